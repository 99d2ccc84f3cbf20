// Grouped expert GEMMs on CTA pairs (tcgen05 cta_group::2, sm_100a): the
// large-batch form of expert_gemm_kernel.
//
// Same work as expert_gemm.cu (the per-expert fp4_gemm / fp8_gemm calls of
// spark_runtime/lazy_official_runtime.py:995-998,1001) with the same operands,
// epilogue and outputs, but one work item is a 256-row segment tile x one
// 256-row weight block computed by a cluster of two CTAs:
//   - CTA r of the pair stages activation rows row0 + 128 r .. + 127 (A) and
//     one 128-row half of the weight block (B): GEMM1 -> w1 rows (r = 0) or
//     the same w3 rows (r = 1); GEMM2 -> w2 rows jb*256 + 128 r;
//   - the leader (r = 0) issues M = 256, N = 256, K = 32 block-scaled MMAs; each
//     CTA's TMEM receives its own 128 rows x 256 columns, exactly the
//     accumulator the single-CTA kernel holds, so the epilogue is the same.
// Per SM and k tile this moves 32 KB into shared memory and reads 32 KB of
// operands out of it, against 48 KB + 48 KB for the single-CTA M = 128 x
// N = 256 tile, and fits 6 stages instead of 4.  Measured on the B200 it is
// bit-identical to the single-CTA kernel and about 5% faster per computed
// row; 256-row tiles pad small segments twice as much, so the host picks it
// only for very large segments (DSV4_BLOCK_N=256 forces it).
//
// Synchronisation (all waits bounded, see common.cuh):
//   full[s]    leader only; its producer posts the byte count of both CTAs'
//              loads, and both CTAs' loads complete on it (.cta_group::2);
//   empty[s]   both CTAs; the leader's MMA commit arrives on both (multicast);
//   acc_full   both CTAs; the leader's MMA commit arrives on both;
//   acc_empty  leader only; one arrival from each CTA's epilogue.
// No load uses cluster multicast.
#include "kernels.cuh"

namespace dsv4 {

template <bool GATED>
struct PairCfg {
  static constexpr int A_BYTES = 128 * 128;      // this CTA's 128 activation rows, one k tile
  static constexpr int B_BYTES = 128 * 128;      // this CTA's 128-row weight half (e2m1 spread)
  static constexpr int TILE_BYTES = A_BYTES + B_BYTES;
  // scale atoms of a group of four k tiles in a two-slot ring (as in
  // expert_gemm.cu): [act 512][weight half 0: 4 x 512][weight half 1: 4 x 512]
  static constexpr int SF_GROUP = 512 + 2 * 2048;
  static constexpr int SF_RING = 2 * SF_GROUP;
  static constexpr int STAGE_BYTES = TILE_BYTES;
  static constexpr int CTRL_BYTES = 256;
  static constexpr int SMEM_MAX = 232448;
  static constexpr int STAGES0 = (SMEM_MAX - 1024 - CTRL_BYTES - SF_RING) / STAGE_BYTES;
  static constexpr int STAGES = STAGES0 > 8 ? 8 : STAGES0;
  static constexpr int SFA_COL = 256;
  static constexpr int SFB_COL = 264;
  static constexpr int TMEM_COLS = 512;
  static constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + SF_RING + CTRL_BYTES;
  static_assert(STAGES >= 2, "need at least two stages");
  static_assert(SMEM_BYTES <= SMEM_MAX, "over the per-CTA shared memory limit");
};

// Tensor maps of the pair kernel: weights (routed arena / shared expert),
// activations, and the three scale-atom buffers viewed as rows of 256 bytes
// (weights: box 256 x 8 = four consecutive 512-byte atoms; activations: box
// 256 x 2 = one atom).
struct PairMaps {
  CUtensorMap w0, w1;    // routed e2m1 arena maps (GEMM1: w1, w3; GEMM2: w2, w2)
  CUtensorMap s0, s1;    // shared expert e4m3 maps (same roles)
  CUtensorMap x;         // activations, box 128 rows
  CUtensorMap sfw;       // routed weight scale atoms (whole arena_sf)
  CUtensorMap sfs;       // shared expert weight scale atoms
  CUtensorMap sfx;       // activation scale atoms (k-packed)
};

template <bool GATED>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    expert_gemm_pair_kernel(const __grid_constant__ PairMaps maps, const GemmArgs args,
                            const long long sfs_row_off0, const long long sfs_row_off1,
                            const long long sfw_row_off0, const long long sfw_row_off1) {
  using C = PairCfg<GATED>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tile_base = smem;
  uint8_t* sf_base = smem + (size_t)C::STAGES * C::TILE_BYTES;
  uint8_t* ctrl = sf_base + C::SF_RING;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_abort = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    *epi_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.w0);
    tma_prefetch_desc(&maps.x);
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int NB = args.nb_count;
  const int KT = args.kt_count;
  const int KT4 = KT >> 2;
  const int total = *args.n_tiles * NB;
  const int cid = (int)(blockIdx.x >> 1);
  const int step = (int)(gridDim.x >> 1);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int sf_slot = 1;  // ring slot of the current k-tile group (flips at each group)
      for (int w = cid; w < total && !*abort_flag; w += step) {
        const int4 tl = args.tiles[w / NB];
        const int jb = w % NB;
        const bool shared = tl.x >= args.n_routed;
        const int slot = shared ? 0 : args.expert_slot[tl.x];
        const int arow = tl.y + 128 * (int)rank;  // this CTA's activation rows
        const int brow = GATED ? jb * 128 : jb * 256 + 128 * (int)rank;
        const CUtensorMap* bmap = shared ? ((GATED && rank) ? &maps.s1 : &maps.s0)
                                         : ((GATED && rank) ? &maps.w1 : &maps.w0);
        // scale atoms of the two 128-row weight halves, in 256-byte rows
        long long sfb_row0, sfb_row1;
        const CUtensorMap* sfmap = shared ? &maps.sfs : &maps.sfw;
        {
          const long long base = shared ? 0 : (long long)slot * (args.sf_slot_stride >> 8);
          const long long o0 = shared ? sfs_row_off0 : sfw_row_off0;
          const long long o1 = shared ? sfs_row_off1 : sfw_row_off1;
          if (GATED) {
            sfb_row0 = base + o0 + (long long)jb * KT * 2;
            sfb_row1 = base + o1 + (long long)jb * KT * 2;
          } else {
            sfb_row0 = base + o0 + (long long)(2 * jb) * KT * 2;
            sfb_row1 = base + o0 + (long long)(2 * jb + 1) * KT * 2;
          }
        }
        const long long sfa_row0 = (long long)(arow >> 5) * KT4 * 2;
        // both CTAs' global bytes: A + B half (e2m1 8 KB / e4m3 16 KB)
        const uint32_t tx_base = 2u * (C::A_BYTES + (shared ? 16384u : 8192u));
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, DSV4_DEVERR_TIMEOUT_PRODUCER)) {
            *abort_flag = 1;
            break;
          }
          // the first k tile of each group of four carries the group's scale atoms
          const bool sf_tile = (kt & 3) == 0;
          if (sf_tile) sf_slot ^= 1;
          const uint32_t bar = mapa_shared(&full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], tx_base + (sf_tile ? 2u * 4608u : 0u));
          uint8_t* st = tile_base + (size_t)stage * C::TILE_BYTES;
          uint8_t* sf = sf_base + (size_t)sf_slot * C::SF_GROUP;
          tma_load_2d_pair(st, &maps.x, bar, kt * 128, arow);
          if (shared)
            tma_load_2d_pair(st + C::A_BYTES, bmap, bar, kt * 128, brow);
          else
            tma_load_3d_pair(st + C::A_BYTES, bmap, bar, kt * 128, brow, slot);
          if (sf_tile) {
            tma_load_2d_pair(sf, &maps.sfx, bar, 0, (int)(sfa_row0 + (kt >> 2) * 2));
            tma_load_2d_pair(sf + 512, sfmap, bar, 0, (int)(sfb_row0 + kt * 2));
            tma_load_2d_pair(sf + 2560, sfmap, bar, 0, (int)(sfb_row1 + kt * 2));
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {
        // let copies already in flight land before the CTA can exit
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 10000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t aphase = 0;
      int sf_slot = 1;  // follows the producer's ring slot
      const uint32_t sfa_t = tmem + C::SFA_COL;
      const uint32_t sfb_t = tmem + C::SFB_COL;
      for (int w = cid; w < total && !*abort_flag; w += step) {
        const int4 tl = args.tiles[w / NB];
        const uint32_t b_fmt = tl.x >= args.n_routed ? 0u : 5u;  // e4m3 shared, e2m1 routed
        if (!mbar_wait_cluster(acc_empty, aphase ^ 1, DSV4_DEVERR_TIMEOUT_MMA)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&full[stage], phase, DSV4_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = tile_base + (size_t)stage * C::TILE_BYTES;
          if ((kt & 3) == 0) sf_slot ^= 1;
          const uint8_t* sf = sf_base + (size_t)sf_slot * C::SF_GROUP;
          const uint32_t sfa_k = sfa_t + 4 * sf_slot;
          const uint32_t sfb_k = sfb_t + 32 * sf_slot + 8 * (kt & 3);
          if ((kt & 3) == 0) {
            tc_cp_sf_pair(sfa_k, sdesc_sf(smem_u32(sf)));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tc_cp_sf_pair(sfb_k + 8 * j, sdesc_sf(smem_u32(sf + 512 + 512 * j)));
              tc_cp_sf_pair(sfb_k + 8 * j + 4, sdesc_sf(smem_u32(sf + 2560 + 512 * j)));
            }
          }
          const uint64_t adesc = sdesc_k_sw128(smem_u32(st));
          const uint64_t bdesc = sdesc_k_sw128(smem_u32(st + C::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t idesc = idesc_mxf8f6f4(0u, b_fmt, 256, kt & 3, kk, 256);
            tc_mma_mxf8f6f4_pair(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, sfa_k, sfb_k,
                                 (kt > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        tc_commit_pair_mc(acc_full, 0x3);
        aphase ^= 1;
      }
      // drain every tcgen05 op of the pair before TMEM is released
      tc_commit_pair(final_bar);
      mbar_wait(final_bar, 0, DSV4_DEVERR_TIMEOUT_MMA);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Thread (warp quarter q, lane) owns row 32q + lane of this CTA's half of
    // the pair tile and the 256 accumulator columns of that row.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    uint32_t aphase = 0;
    const float lim = args.swiglu_limit;
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t acc_empty_leader = mapa_shared(acc_empty, 0);
    for (int w = cid; w < total; w += step) {
      const int4 tl = args.tiles[w / NB];
      const int jb = w % NB;
      const int row0 = tl.y + 128 * (int)rank;
      const int nrows = min(max(tl.z - 128 * (int)rank, 0), 128);
      if (!mbar_wait(acc_full, aphase, DSV4_DEVERR_TIMEOUT_EPILOGUE)) {
        *epi_abort = 1;
        *abort_flag = 1;
      }
      epi_bar();
      const bool stop = *epi_abort != 0;
      epi_bar();
      if (stop) break;
      aphase ^= 1;
      tc_fence_after();
      const bool warp_rows = q * 32 < nrows;
      uint32_t pk[128];
      if (warp_rows) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t a[32], b[32];
          if (GATED) {  // pk[j] = (bf16 g_j, bf16 u_j)
            tmem_ld32_issue(taddr + 32 * c, a);
            tmem_ld32_issue(taddr + 128 + 32 * c, b);
            tmem_wait_ld2(a, b);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const __nv_bfloat162 v =
                  __floats2bfloat162_rn(__uint_as_float(a[i]), __uint_as_float(b[i]));
              pk[32 * c + i] = *reinterpret_cast<const uint32_t*>(&v);
            }
          } else {      // pk[j] = bf16 outputs (2j, 2j+1)
            tmem_ld32_issue(taddr + 64 * c, a);
            tmem_ld32_issue(taddr + 64 * c + 32, b);
            tmem_wait_ld2(a, b);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const __nv_bfloat162 v0 =
                  __floats2bfloat162_rn(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
              const __nv_bfloat162 v1 =
                  __floats2bfloat162_rn(__uint_as_float(b[2 * i]), __uint_as_float(b[2 * i + 1]));
              pk[32 * c + i] = *reinterpret_cast<const uint32_t*>(&v0);
              pk[32 * c + 16 + i] = *reinterpret_cast<const uint32_t*>(&v1);
            }
          }
        }
      }
      tc_fence_before();
      epi_bar();
      if (q == 0 && lane == 0) mbar_arrive_cluster(acc_empty_leader);
      if (warp_rows && r < nrows) {
        const int row = row0 + r;
        if (GATED) {
          const float wr = args.slot_weight[row];
          float amax = 0.f;
#pragma unroll
          for (int j = 0; j < 128; ++j) {
            const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&pk[j]);
            float gb = __low2float(v), ub = __high2float(v);
            if (lim > 0.f) {
              ub = fminf(fmaxf(ub, -lim), lim);
              gb = fminf(gb, lim);
            }
            const float s = __fdividef(gb, 1.0f + __expf(-gb));
            const float hv = bf16_round((s * ub) * wr);
            amax = fmaxf(amax, fabsf(hv));
            pk[j] = __float_as_uint(hv);
          }
          const int e = act_scale_exp(amax);
          const float inv = exp2i(-e);
          uint8_t* dst = args.out_q + (size_t)row * args.out_ld + jb * 128;
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            uint32_t wds[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const float* f = reinterpret_cast<const float*>(&pk[16 * v + 4 * t]);
              wds[t] = e4m3x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
            }
            *reinterpret_cast<uint4*>(dst + 16 * v) = make_uint4(wds[0], wds[1], wds[2], wds[3]);
          }
          write_row_scale(args.out_sf, row, jb, (args.out_ld >> 7) >> 2,
                          static_cast<uint8_t>(e + 127));
        } else {
          uint4* dst = reinterpret_cast<uint4*>(args.out_bf16 + (size_t)row * args.out_ld + jb * 256);
#pragma unroll
          for (int v = 0; v < 32; ++v)
            dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
    }
  }

  // the leader's MMAs write both CTAs' TMEM: neither CTA frees it before the
  // pair is done
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

// Scale atoms as rows of 256 bytes: dims {256, bytes / 256}, box {256, box_rows}.
int make_tmap_atoms(CUtensorMap* m, const void* base, long long bytes, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return DSV4_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 255) || (bytes & 255) || bytes < 256LL * box_rows)
    return DSV4_ERR_ARG;
  cuuint64_t dims[2] = {256, (cuuint64_t)(bytes / 256)};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {256, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSV4_OK : DSV4_ERR_CUDA;
}

// CTA pairs that can be resident at once on this device (cached per device).
int pair_clusters_resident(bool gated) {
  static int cached[2][64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int& c = cached[gated ? 1 : 0][dev];
  if (c > 0) return c;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (gated) {
    cfg.dynamicSmemBytes = PairCfg<true>::SMEM_BYTES;
    if (ensure_smem_attr(reinterpret_cast<const void*>(expert_gemm_pair_kernel<true>),
                         (int)PairCfg<true>::SMEM_BYTES) ||
        cudaOccupancyMaxActiveClusters(&n, expert_gemm_pair_kernel<true>, &cfg) != cudaSuccess)
      n = 0;
  } else {
    cfg.dynamicSmemBytes = PairCfg<false>::SMEM_BYTES;
    if (ensure_smem_attr(reinterpret_cast<const void*>(expert_gemm_pair_kernel<false>),
                         (int)PairCfg<false>::SMEM_BYTES) ||
        cudaOccupancyMaxActiveClusters(&n, expert_gemm_pair_kernel<false>, &cfg) != cudaSuccess)
      n = 0;
  }
  cudaGetLastError();
  c = n;
  return n;
}

// One launch of the pair kernel over `clusters` CTA pairs (grid = 2 x clusters).
int launch_expert_gemm_pair(bool gated, const PairMaps& maps, const GemmArgs& args,
                            long long sfs_row_off0, long long sfs_row_off1,
                            long long sfw_row_off0, long long sfw_row_off1, int clusters,
                            cudaStream_t st) {
  if (clusters <= 0) return DSV4_ERR_UNSUPPORTED;
  const dim3 grid(2 * clusters, 1, 1);
  if (gated)
    launch_k(expert_gemm_pair_kernel<true>, grid, 192, PairCfg<true>::SMEM_BYTES, st, maps, args,
             sfs_row_off0, sfs_row_off1, sfw_row_off0, sfw_row_off1);
  else
    launch_k(expert_gemm_pair_kernel<false>, grid, 192, PairCfg<false>::SMEM_BYTES, st, maps,
             args, sfs_row_off0, sfs_row_off1, sfw_row_off0, sfw_row_off1);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

}  // namespace dsv4
