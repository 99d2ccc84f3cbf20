// Grouped expert GEMMs on the 5th-generation tensor core (tcgen05, sm_100a).
//
// Replaces the per-expert official Expert.forward -> act_quant + fp4_gemm /
// fp8_gemm calls of spark_runtime/lazy_official_runtime.py:995-998,1001
// (official kernel API: scripts/smoke_official_kernels.py:36-50) with one
// launch over every (expert segment, 128-row weight block) of the layer.
//
// Orientation ("swap AB"): the weight is the M = 128 operand (A) and the
// tokens of one expert segment are N (B), so a decode step with one token per
// expert still fills the 128-row MMA and the kernel streams weights at HBM
// speed.  D[weight_row, token] lives in TMEM: one lane per weight row, one
// column per token.
//
// Operands (both K-major, 128-byte swizzle, 128-wide K tiles):
//   A routed : e2m1 weights straight from the expert arena, TMA'd with the
//              16U4_ALIGN16B type (16 packed nibbles -> 16 bytes in smem);
//   A shared : e4m3 weights of the shared expert (the "E-th expert");
//   B        : e4m3 activations of the permuted segment rows;
//   scales   : per-32 ue8m0 for A, per-128 (replicated x4) for B, moved
//              smem -> TMEM with tcgen05.cp; kind::mxf8f6f4.block_scale.
//
// GEMM1 (GATED): two accumulators (w1 and w3 rows of the same inter block);
//   epilogue = bf16(g), bf16(u), clamp, silu(g)*u*route_weight, bf16, per-128
//   act_quant along the inter dim (the 128 TMEM lanes = one scale block) ->
//   e4m3 H rows + scale atoms that feed GEMM2 directly.
// GEMM2: w2; epilogue = bf16 expert output rows O[slot, hidden].
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner and
// MMA issuer, warps 2..5 = epilogue (TMEM lane quarter = warp % 4).
#include "kernels.cuh"

namespace dsv4 {

__host__ __device__ constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

template <int BN, bool GATED>
struct GemmCfg {
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int NA = GATED ? 2 : 1;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int TILE_BYTES = NA * A_BYTES + B_BYTES;  // multiple of 1024
  static constexpr int SFB_OFF = 512 * NA;
  static constexpr int SF_STAGE = 512 * NA + 512;
  static constexpr int STAGE_BYTES = TILE_BYTES + SF_STAGE;
  static constexpr int SMEM_BUDGET = 200 * 1024;
  static constexpr int STAGES0 = SMEM_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES0 > 8 ? 8 : STAGES0;
  static constexpr int ACC_COLS = NA * BN;
  static constexpr int NACC = (2 * ACC_COLS + 12 <= 512) ? 2 : 1;
  static constexpr int SF_COL = NACC * ACC_COLS;
  static constexpr int TMEM_COLS = pow2_at_least(SF_COL + 12);
  static constexpr uint32_t TX_BYTES = NA * A_BYTES + B_BYTES + 512 * NA + 512;
  static constexpr uint32_t TX_BYTES_FP4 = NA * (A_BYTES / 2) + B_BYTES + 512 * NA + 512;
  static constexpr int RED_BYTES = GATED ? 4 * BN * 4 : 0;
  static constexpr int CTRL_BYTES = 256;
  static constexpr size_t SMEM_BYTES =
      1024 + (size_t)STAGES * STAGE_BYTES + CTRL_BYTES + RED_BYTES;
  static_assert(TILE_BYTES % 1024 == 0, "tiles must keep 1024-byte alignment");
  static_assert(SF_COL + 12 <= 512, "TMEM overflow");
  static_assert(BN % 32 == 0 && BN <= 128, "one sliding scale atom covers 128 rows");
  static_assert(STAGES >= 2, "need at least two stages");
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Activation scale atoms use a sliding layout: one 512-byte atom per 32-row
// group g and 128-wide K tile; byte (m0*16 + m1*4 + b) of atom (g, kt) holds
// the scale of row 32*(g+m1) + m0.  A tile starting at any 32-aligned row then
// needs exactly one atom and always lands on TMEM scale column 0.
__device__ __forceinline__ void write_row_scale(uint8_t* atoms, int row, int kt, int KT,
                                                uint32_t scale_byte) {
  const uint32_t word = scale_byte * 0x01010101u;
  const int g = row >> 5;
#pragma unroll
  for (int m1 = 0; m1 < 4; ++m1) {
    if (g - m1 >= 0)
      *reinterpret_cast<uint32_t*>(atoms + ((size_t)(g - m1) * KT + kt) * 512 + (row & 31) * 16 +
                                   m1 * 4) = word;
  }
}

template <int BN, bool GATED>
__global__ void __launch_bounds__(192, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tmA0,
                       const __grid_constant__ CUtensorMap tmA1,
                       const __grid_constant__ CUtensorMap tmS0,
                       const __grid_constant__ CUtensorMap tmS1,
                       const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = GemmCfg<BN, GATED>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tile_base = smem;
  uint8_t* sf_base = smem + (size_t)C::STAGES * C::TILE_BYTES;
  uint8_t* ctrl = sf_base + (size_t)C::STAGES * C::SF_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* final_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_abort = abort_flag + 1;
  float* red = reinterpret_cast<float*>(ctrl + C::CTRL_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    *epi_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA0);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int NB = args.nb_count;
  const int KT = args.kt_count;
  const int total = *args.n_tiles * NB;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x) {
        const int4 tl = args.tiles[w / NB];
        const int jb = w % NB;
        const bool shared = tl.x >= args.n_routed;
        const int slot = shared ? 0 : args.expert_slot[tl.x];
        const uint8_t* sfa0 = shared ? args.sf_shared0
                                     : args.sf_routed + (size_t)slot * args.sf_slot_stride + args.sf_off0;
        const uint8_t* sfa1 = shared ? args.sf_shared1
                                     : args.sf_routed + (size_t)slot * args.sf_slot_stride + args.sf_off1;
        const int row0 = tl.y;
        const size_t g0 = (size_t)(row0 >> 5);
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, DSV4_DEVERR_TIMEOUT_PRODUCER)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* st = tile_base + (size_t)stage * C::TILE_BYTES;
          uint8_t* sf = sf_base + (size_t)stage * C::SF_STAGE;
          // transaction bytes count what the TMA reads: an e2m1 tile is 8 KB in
          // global memory even though it spreads to 16 KB (16U4_ALIGN16B) in smem
          mbar_arrive_expect_tx(&full[stage], shared ? C::TX_BYTES : C::TX_BYTES_FP4);
          if (shared) {
            tma_load_2d(st, &tmS0, &full[stage], kt * 128, jb * 128);
            if (GATED) tma_load_2d(st + C::A_BYTES, &tmS1, &full[stage], kt * 128, jb * 128);
          } else {
            tma_load_3d(st, &tmA0, &full[stage], kt * 128, jb * 128, slot);
            if (GATED) tma_load_3d(st + C::A_BYTES, &tmA1, &full[stage], kt * 128, jb * 128, slot);
          }
          tma_load_2d(st + C::NA * C::A_BYTES, &tmB, &full[stage], kt * 128, row0);
          bulk_load(sf, sfa0 + ((size_t)jb * KT + kt) * 512, 512, &full[stage]);
          if (GATED) bulk_load(sf + 512, sfa1 + ((size_t)jb * KT + kt) * 512, 512, &full[stage]);
          bulk_load(sf + C::SFB_OFF, args.sfb + (g0 * KT + kt) * 512, 512, &full[stage]);
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
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int abuf = 0;
      uint32_t aphase = 0;
      for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x) {
        const int4 tl = args.tiles[w / NB];
        const uint32_t a_fmt = tl.x >= args.n_routed ? 0u : 5u;  // e4m3 shared, e2m1 routed
        if (!mbar_wait(&acc_empty[abuf], aphase ^ 1, DSV4_DEVERR_TIMEOUT_MMA)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + abuf * C::ACC_COLS;
        const uint32_t sfa0_t = tmem + C::SF_COL;
        const uint32_t sfa1_t = tmem + C::SF_COL + 4;
        const uint32_t sfb_t = tmem + C::SF_COL + 8;
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&full[stage], phase, DSV4_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = tile_base + (size_t)stage * C::TILE_BYTES;
          const uint8_t* sf = sf_base + (size_t)stage * C::SF_STAGE;
          tc_cp_sf(sfa0_t, sdesc_sf(smem_u32(sf)));
          if (GATED) tc_cp_sf(sfa1_t, sdesc_sf(smem_u32(sf + 512)));
          tc_cp_sf(sfb_t, sdesc_sf(smem_u32(sf + C::SFB_OFF)));
          const uint64_t a0 = sdesc_k_sw128(smem_u32(st));
          const uint64_t a1 = sdesc_k_sw128(smem_u32(st + C::A_BYTES));
          const uint64_t b = sdesc_k_sw128(smem_u32(st + C::NA * C::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t idesc = idesc_mxf8f6f4(a_fmt, 0u, BN, kk, kk);
            const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
            tc_mma_mxf8f6f4(d0, a0 + 2 * kk, b + 2 * kk, idesc, sfa0_t, sfb_t, acc);
            if (GATED)
              tc_mma_mxf8f6f4(d0 + BN, a1 + 2 * kk, b + 2 * kk, idesc, sfa1_t, sfb_t, acc);
          }
          tc_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        tc_commit(&acc_full[abuf]);
        if (++abuf == C::NACC) {
          abuf = 0;
          aphase ^= 1;
        }
      }
      // drain every tcgen05 op of this CTA before TMEM is released
      tc_commit(final_bar);
      mbar_wait(final_bar, 0, DSV4_DEVERR_TIMEOUT_MMA);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int abuf = 0;
    uint32_t aphase = 0;
    const float lim = args.swiglu_limit;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      const int4 tl = args.tiles[w / NB];
      const int jb = w % NB;
      const int row0 = tl.y, nrows = tl.z;
      // The four epilogue warps take every decision together: a warp whose
      // wait timed out still meets the others at the named barrier, then all
      // of them leave.  (A named barrier with a missing warp would never end.)
      // epi_abort is written only by epilogue warps and read between two
      // barriers, so all four see the same value.
      if (!mbar_wait(&acc_full[abuf], aphase, DSV4_DEVERR_TIMEOUT_EPILOGUE)) {
        *epi_abort = 1;
        *abort_flag = 1;
      }
      epi_bar();
      const bool stop = *epi_abort != 0;
      epi_bar();
      if (stop) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + abuf * C::ACC_COLS;
      const int col = jb * 128 + q * 32 + lane;  // output feature (weight row)
      if (GATED) {
        for (int c = 0; c < BN; c += 16) {
          float g[16], u[16], h[16];
          tmem_ld16(taddr + c, g);
          tmem_ld16(taddr + BN + c, u);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c + i;
            float gb = bf16_round(g[i]);
            float ub = bf16_round(u[i]);
            if (lim > 0.f) {
              ub = fminf(fmaxf(ub, -lim), lim);
              gb = fminf(gb, lim);
            }
            const float s = gb / (1.0f + expf(-gb));
            const float wr = n < nrows ? args.slot_weight[row0 + n] : 0.f;
            float hv = (s * ub) * wr;
            hv = bf16_round(hv);
            h[i] = hv;
            float m = fabsf(hv);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) red[q * BN + n] = m;
          }
          epi_bar();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c + i;
            const float amax =
                fmaxf(fmaxf(red[n], red[BN + n]), fmaxf(red[2 * BN + n], red[3 * BN + n]));
            const int e = act_scale_exp(amax);
            const uint8_t code = f32_to_e4m3(h[i] * exp2i(-e));
            if (n < nrows) {
              args.out_q[(size_t)(row0 + n) * args.out_ld + col] = code;
              if (q == 0 && lane == 0)
                write_row_scale(args.out_sf, row0 + n, jb, args.out_ld >> 7,
                                static_cast<uint32_t>(e + 127));
            }
          }
          epi_bar();
        }
      } else {
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(taddr + c, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c + i;
            if (n < nrows)
              args.out_bf16[(size_t)(row0 + n) * args.out_ld + col] = __float2bfloat16_rn(v[i]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[abuf]);
      if (++abuf == C::NACC) {
        abuf = 0;
        aphase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// FP4 e2m1 weights of every arena slot: dims {K elements, rows, slots}.
int make_tmap_fp4_arena(CUtensorMap* m, const void* base, int K, int rows, int slots,
                        long long slot_stride) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return DSV4_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 31) || (slot_stride & 31) || (K % 128) ||
      ((K / 2) % 32))
    return DSV4_ERR_ARG;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)slots};
  cuuint64_t strides[2] = {(cuuint64_t)(K / 2), (cuuint64_t)slot_stride};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void*>(base), dims,
                   strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSV4_OK : DSV4_ERR_CUDA;
}

// 8-bit row-major matrix [rows][K] (e4m3 weights or activations), box {128, box_rows}.
int make_tmap_u8(CUtensorMap* m, const void* base, int K, int rows, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return DSV4_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K % 128)) return DSV4_ERR_ARG;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSV4_OK : DSV4_ERR_CUDA;
}

template <int BN, bool GATED>
static int launch_one(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& s0,
                      const CUtensorMap& s1, const CUtensorMap& b, const GemmArgs& args, int grid,
                      cudaStream_t st) {
  using C = GemmCfg<BN, GATED>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(expert_gemm_kernel<BN, GATED>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)C::SMEM_BYTES) != cudaSuccess)
      return DSV4_ERR_CUDA;
    attr_set = true;
  }
  expert_gemm_kernel<BN, GATED><<<grid, 192, C::SMEM_BYTES, st>>>(a0, a1, s0, s1, b, args);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_expert_gemm(bool gated, int block_n, const CUtensorMap& a0, const CUtensorMap& a1,
                       const CUtensorMap& s0, const CUtensorMap& s1, const CUtensorMap& b,
                       const GemmArgs& args, int grid, cudaStream_t st) {
  if (gated) {
    switch (block_n) {
      case 32: return launch_one<32, true>(a0, a1, s0, s1, b, args, grid, st);
      case 64: return launch_one<64, true>(a0, a1, s0, s1, b, args, grid, st);
      case 128: return launch_one<128, true>(a0, a1, s0, s1, b, args, grid, st);
      default: return DSV4_ERR_ARG;
    }
  }
  switch (block_n) {
    case 32: return launch_one<32, false>(a0, a1, s0, s1, b, args, grid, st);
    case 64: return launch_one<64, false>(a0, a1, s0, s1, b, args, grid, st);
    case 128: return launch_one<128, false>(a0, a1, s0, s1, b, args, grid, st);
    default: return DSV4_ERR_ARG;
  }
}

}  // namespace dsv4
