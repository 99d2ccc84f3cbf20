// Grouped expert GEMMs on the 5th-generation tensor core (tcgen05, sm_100a).
//
// Replaces the per-expert official Expert.forward -> act_quant + fp4_gemm /
// fp8_gemm calls of spark_runtime/lazy_official_runtime.py:995-998,1001
// (official kernel API: scripts/smoke_official_kernels.py:36-50) with one
// launch over every (expert segment tile, 256-row weight block) of the layer.
//
// Orientation: A = activations of one expert segment tile (M = 128 rows of
// which the first BM are loaded: 32 for decode, 128 for prefill; rows past BM
// read the following smem and land in TMEM lanes nobody reads), B = N = 256
// weight rows (GEMM1: 128 rows of w1 stacked on the same 128 rows of w3;
// GEMM2: 256 rows of w2).  One block-scaled MMA (kind::mxf8f6f4, K = 32)
// therefore covers 4 KB of FP4 weights, and the TMEM accumulator holds, per
// token lane, 256 output columns - so the SwiGLU and the 128-wide fp8
// re-quantization of the epilogue are per-thread work with contiguous stores.
//
// Operands (K-major, 128-byte swizzle, 128-wide k tiles):
//   A            : e4m3 activation rows of the permuted segment (TMA box BM rows);
//   B routed     : e2m1 weights from the expert arena, TMA type 16U4_ALIGN16B
//                  (16 packed nibbles -> 16 bytes in smem);
//   B shared     : e4m3 weights of the shared expert (the E-th segment);
//   scales       : activations per 128 (k-packed: one 32-bit TMEM word holds
//                  four k tiles, selected by the MMA's scale-factor id), weights
//                  per 32 (one word per k tile); both moved smem -> TMEM with
//                  tcgen05.cp.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner and MMA
// issuer, warps 2..5 = epilogue (TMEM lane quarter = warp % 4).
#include "kernels.cuh"

namespace dsv4 {

__host__ __device__ constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// FP4A: GEMM1 on FP4 activations (kind::mxf4).  A k tile is then 256 values,
// still 128 bytes per row for both operands (two e2m1 codes per byte), and
// each stage carries its own scale atoms: two 128-wide windows of the
// activation atoms and of each weight half (3 KB).
template <int BM, bool GATED, bool FP4A = false>
struct GemmCfg {
  static constexpr int A_BYTES = BM * 128;       // activation rows of one k tile
  static constexpr int B_HALF = 128 * 128;       // one 128-row weight box in smem
  static constexpr int B_BYTES = 2 * B_HALF;     // N = 256 weight rows
  static constexpr int TILE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SF_STAGE = FP4A ? 3 * 1024 : 0;
  // scale atoms of a group of four k tiles, loaded with the group's first
  // tile into one of two ring slots: [act 512][weight half 0: 4 x 512][half 1: 4 x 512].
  // A slot is refilled 8 k tiles after its last use, which the producer's
  // stage wait already covers while STAGES <= 8.
  static constexpr int SF_GROUP = 512 + 2 * 2048;
  static constexpr int SF_RING = FP4A ? 0 : 2 * SF_GROUP;
  static constexpr int STAGE_BYTES = TILE_BYTES + SF_STAGE;
  static constexpr int CTRL_BYTES = 256;
  // the whole 227 KB a CTA may hold: decode is bound by the weight bytes in
  // flight per SM, and an e2m1 box takes twice its global bytes in smem
  static constexpr int SMEM_MAX = 232448;
  static constexpr int STAGES0 = (SMEM_MAX - 1024 - CTRL_BYTES - SF_RING) / STAGE_BYTES;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static constexpr int STAGES = STAGES0 > 8 ? 8 : STAGES0;
  static constexpr int ACC_COLS = 256;
  // TMEM scale columns, two sets used by alternate k-tile groups: activation
  // scales 4 columns, weight scales 4 k tiles x 8 columns (256 rows).  FP4A:
  // two sets used by alternate k tiles, each activation 2 windows x 4 columns
  // then weights 2 windows x 8 columns (24 columns from SFA_COL + 24 * set).
  static constexpr int SFA_COL = 256;
  static constexpr int SFB_COL = 264;
  static constexpr int TMEM_COLS = 512;
  static constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + SF_RING + CTRL_BYTES;
  static_assert(A_BYTES % 1024 == 0, "tiles must keep 1024-byte alignment");
  // the M = 128 MMA reads 128 rows (16 KB) from the A base; they must stay in the stage
  static_assert(128 * 128 <= TILE_BYTES, "A window leaves the stage");
  static_assert(BM == 32 || BM == 64 || BM == 128, "activation rows per tile");
  static_assert(STAGES >= 2, "need at least two stages");
  static_assert(SMEM_BYTES <= SMEM_MAX, "over the per-CTA shared memory limit");
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Activation scale atoms use a sliding, k-packed layout: one 512-byte atom per
// 32-row group g and group of four 128-wide k tiles q; byte (m0*16 + m1*4 + b)
// of atom (g, q) holds the scale of row 32*(g+m1) + m0 for k tile 4q + b.  A
// tile starting at any 32-aligned row needs one atom per four k tiles, always
// lands on TMEM scale column 0, and the MMA picks the k tile's byte with its
// scale-factor id.
__device__ __forceinline__ void write_row_scale(uint8_t* atoms, int row, int kt, int KT4,
                                                uint8_t scale_byte) {
  const int g = row >> 5;
#pragma unroll
  for (int m1 = 0; m1 < 4; ++m1) {
    if (g - m1 >= 0)
      atoms[((size_t)(g - m1) * KT4 + (kt >> 2)) * 512 + (row & 31) * 16 + m1 * 4 + (kt & 3)] =
          scale_byte;
  }
}

// Everything the producer needs about one work item (segment tile x 256-row
// weight block).
struct ItemInfo {
  int jb, row0, slot;
  bool shared;
  int r0, r1;               // first row of the two 128-row weight boxes
  const uint8_t* sfb0;      // scale atoms of the two boxes (k tile 0)
  const uint8_t* sfb1;
};

// KW: 128-wide k windows of a weight row block's scale atoms (= the k tiles of
// the e4m3-activation kernel, twice them with FP4 activations).
template <bool GATED>
__device__ __forceinline__ ItemInfo decode_item(const GemmArgs& a, int w, int NB, int KW) {
  ItemInfo it;
  const int4 tl = a.tiles[w / NB];
  it.jb = w % NB;
  it.row0 = tl.y;
  it.shared = tl.x >= a.n_routed;
  it.slot = it.shared ? 0 : a.expert_slot[tl.x];
  const uint8_t* base = it.shared ? nullptr : a.sf_routed + (size_t)it.slot * a.sf_slot_stride;
  const uint8_t* s0 = it.shared ? a.sf_shared0 : base + a.sf_off0;
  const uint8_t* s1 = it.shared ? a.sf_shared1 : base + a.sf_off1;
  if (GATED) {  // w1 rows jb*128.. on top of the same w3 rows
    it.r0 = it.r1 = it.jb * 128;
    it.sfb0 = s0 + (size_t)it.jb * KW * 512;
    it.sfb1 = s1 + (size_t)it.jb * KW * 512;
  } else {      // 256 consecutive w2 rows
    it.r0 = it.jb * 256;
    it.r1 = it.r0 + 128;
    it.sfb0 = s0 + (size_t)(2 * it.jb) * KW * 512;
    it.sfb1 = s0 + (size_t)(2 * it.jb + 1) * KW * 512;
  }
  return it;
}

// TMA producer of the grouped expert GEMMs (one elected thread): per work
// item and 128-wide k tile, the activation box, the two 128-row weight boxes
// and, on the first k tile of each group of four, the group's scale atoms.
// True when an item of tile `shared` is outside args.seg_filter's segments.
__device__ __forceinline__ bool filtered_out(const GemmArgs& a, bool shared) {
  return a.seg_filter != 0 && shared != (a.seg_filter == 2);
}

template <class C, bool GATED, bool FP4A = false>
__device__ __forceinline__ void gemm_produce(const CUtensorMap* tmW0p, const CUtensorMap* tmW1p,
                                             const CUtensorMap* tmS0p, const CUtensorMap* tmS1p,
                                             const CUtensorMap* tmXp, const GemmArgs& args,
                                             uint8_t* tile_base, uint8_t* sf_base, uint64_t* full,
                                             uint64_t* empty, volatile int* abort_flag, int NB,
                                             int KT, int KT4, int total, int step) {
  int stage = 0;
  uint32_t phase = 0;
  int sf_slot = 1;  // ring slot of the current k-tile group (flips at each group)
  const int S = args.k_split, KTS = KT / S;  // k-range slices per item, k tiles per slice
  const int KW = FP4A ? 2 * KT : KT;         // 128-wide scale windows per row block
  ItemInfo cur, nxt;
  if ((int)blockIdx.x < total) cur = decode_item<GATED>(args, blockIdx.x / S, NB, KW);
  // work units are (item, slice); slices start on a group of four k tiles, so
  // the scale-atom ring flips at the same k tiles as without a split
  for (int w = blockIdx.x; w < total && !*abort_flag; w += step) {
    // the next unit's descriptor loads are issued now and used one unit
    // later, so their latency hides behind this unit's k loop
    if (w + step < total) nxt = decode_item<GATED>(args, (w + step) / S, NB, KW);
    if (filtered_out(args, cur.shared)) {
      cur = nxt;
      continue;
    }
    const size_t g0 = (size_t)(cur.row0 >> 5);
    // transaction bytes count what the TMA reads from global memory: an e2m1
    // box is 8 KB there even though it spreads to 16 KB (16U4_ALIGN16B) in smem
    const uint32_t tx_base = C::A_BYTES + 2u * (cur.shared ? C::B_HALF : C::B_HALF / 2);
    const int kt0 = (w % S) * KTS;
    for (int kt = kt0; kt < kt0 + KTS; ++kt) {
      if (!mbar_wait(&empty[stage], phase ^ 1, DSV4_DEVERR_TIMEOUT_PRODUCER)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* st = tile_base + (size_t)stage * C::STAGE_BYTES;
      if constexpr (FP4A) {
        // packed boxes are as many bytes in global memory as in smem; the
        // stage's scale atoms: activation windows 2kt, 2kt+1, then each
        // weight half's
        mbar_arrive_expect_tx(&full[stage], C::A_BYTES + 2u * C::B_HALF + 3072u);
        tma_load_2d(st, tmXp, &full[stage], kt * 128, cur.row0);
        uint8_t* b = st + C::A_BYTES;
        tma_load_3d(b, tmW0p, &full[stage], kt * 128, cur.r0, cur.slot);
        tma_load_3d(b + C::B_HALF, GATED ? tmW1p : tmW0p, &full[stage], kt * 128, cur.r1, cur.slot);
        uint8_t* sfs = st + C::TILE_BYTES;
        bulk_load(sfs, args.sfb + (g0 * KW + 2 * kt) * 512, 1024, &full[stage]);
        bulk_load(sfs + 1024, cur.sfb0 + (size_t)(2 * kt) * 512, 1024, &full[stage]);
        bulk_load(sfs + 2048, cur.sfb1 + (size_t)(2 * kt) * 512, 1024, &full[stage]);
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
        continue;
      }
      // the first k tile of each group of four carries the group's scale atoms
      const bool sf_tile = (kt & 3) == 0;
      if (sf_tile) sf_slot ^= 1;
      uint8_t* sf = sf_base + (size_t)sf_slot * C::SF_GROUP;
      mbar_arrive_expect_tx(&full[stage], tx_base + (sf_tile ? 512u + 4096u : 0u));
      tma_load_2d(st, tmXp, &full[stage], kt * 128, cur.row0);
      uint8_t* b = st + C::A_BYTES;
      if (cur.shared) {
        tma_load_2d(b, tmS0p, &full[stage], kt * 128, cur.r0);
        tma_load_2d(b + C::B_HALF, GATED ? tmS1p : tmS0p, &full[stage], kt * 128, cur.r1);
      } else {
        tma_load_3d(b, tmW0p, &full[stage], kt * 128, cur.r0, cur.slot);
        tma_load_3d(b + C::B_HALF, GATED ? tmW1p : tmW0p, &full[stage], kt * 128, cur.r1,
                    cur.slot);
      }
      if (sf_tile) {
        bulk_load(sf, args.sfb + (g0 * KT4 + (kt >> 2)) * 512, 512, &full[stage]);
        bulk_load(sf + 512, cur.sfb0 + (size_t)kt * 512, 2048, &full[stage]);
        bulk_load(sf + 2560, cur.sfb1 + (size_t)kt * 512, 2048, &full[stage]);
      }
      if (++stage == C::STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    cur = nxt;
  }
  if (*abort_flag) {
    // let copies already in flight land before the CTA can exit
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 10000000ull) {
    }
  }
}

// Split-K epilogue of one (item, slice) unit.  Every thread drains its row's
// 256 fp32 accumulator columns and stores those of valid rows to the slice's
// partial rows; then the CTA counts the slice as finished.  The CTA whose
// slice is the item's last adds the item's S partial rows in slice order
// (the same sum whichever CTA is last) and applies the single-pass epilogue
// arithmetic: four warps take rows in turn, each lane 8 of the 256 columns.
template <bool GATED>
__device__ __forceinline__ void split_epilogue(const GemmArgs& args, uint32_t taddr, bool warp_rows,
                                               int r, int q, int lane, int item, int slice,
                                               const int4& tl, int jb, uint64_t* acc_empty,
                                               volatile int* split_last) {
  const int S = args.k_split, nrows = tl.z;
  if (warp_rows) {
    float* prow = args.partial + ((size_t)slice * args.part_rows + tl.w + r) * args.part_ld + jb * 256;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t a[32], b[32];
      tmem_ld32_issue(taddr + 64 * c, a);
      tmem_ld32_issue(taddr + 64 * c + 32, b);
      tmem_wait_ld2(a, b);
      if (r < nrows) {
        float4* d = reinterpret_cast<float4*>(prow + 64 * c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          d[i] = make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                             __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3]));
          d[8 + i] = make_float4(__uint_as_float(b[4 * i]), __uint_as_float(b[4 * i + 1]),
                                 __uint_as_float(b[4 * i + 2]), __uint_as_float(b[4 * i + 3]));
        }
      }
    }
  }
  tc_fence_before();
  mbar_arrive(acc_empty);
  // The barrier orders every epilogue thread's partial stores before the one
  // counting atomic, whose release (gpu scope, cumulative) publishes them; the
  // CTA that sees the count complete acquires through the same atomic, and the
  // barrier after it orders its threads' partial loads behind that acquire.
  epi_bar();
  if (threadIdx.x == 64) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(old)
                 : "l"(args.item_done + item)
                 : "memory");
    *split_last = old == S - 1;
  }
  epi_bar();
  const bool last = *split_last != 0;
  epi_bar();  // everyone read the flag before the next unit may overwrite it
  if (!last) return;
  for (int rr = q; rr < nrows; rr += 4) {
    // four slices' loads in flight at a time (L2: other SMs wrote them), then
    // their sum in slice order
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    for (int s0 = 0; s0 < S; s0 += 4) {
      float4 x[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (s0 + j < S) {
          const float4* p = reinterpret_cast<const float4*>(
              args.partial + ((size_t)(s0 + j) * args.part_rows + tl.w + rr) * args.part_ld + jb * 256 +
              8 * lane);
          x[2 * j] = __ldcg(p);
          x[2 * j + 1] = __ldcg(p + 1);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (s0 + j < S) {
          v[0] += x[2 * j].x; v[1] += x[2 * j].y; v[2] += x[2 * j].z; v[3] += x[2 * j].w;
          v[4] += x[2 * j + 1].x; v[5] += x[2 * j + 1].y; v[6] += x[2 * j + 1].z; v[7] += x[2 * j + 1].w;
        }
      }
    }
    const int row = tl.y + rr;
    if (GATED) {
      // lanes 0..15 hold g columns 8*lane.., lanes 16..31 the u columns of the same units
      float gb[8], ub[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        gb[i] = bf16_round(v[i]);
        ub[i] = __shfl_down_sync(0xffffffffu, gb[i], 16);
      }
      const float lim = args.swiglu_limit;
      const float wr = args.slot_weight[row];
      float hv[8], amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float g = gb[i], u = ub[i];
        if (lim > 0.f) {
          u = fminf(fmaxf(u, -lim), lim);
          g = fminf(g, lim);
        }
        const float sg = __fdividef(g, 1.0f + __expf(-g));
        hv[i] = bf16_round((sg * u) * wr);
        amax = fmaxf(amax, fabsf(hv[i]));
      }
      if (lane >= 16) amax = 0.f;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      amax = __shfl_sync(0xffffffffu, amax, 0);
      const int e = act_scale_exp(amax);
      const float inv = exp2i(-e);
      if (lane < 16) {
        uint8_t* dst = args.out_q + (size_t)row * args.out_ld + jb * 128 + 8 * lane;
        *reinterpret_cast<uint2*>(dst) =
            make_uint2(e4m3x4(hv[0] * inv, hv[1] * inv, hv[2] * inv, hv[3] * inv),
                       e4m3x4(hv[4] * inv, hv[5] * inv, hv[6] * inv, hv[7] * inv));
      }
      if (lane == 0)
        write_row_scale(args.out_sf, row, jb, (args.out_ld >> 7) >> 2, static_cast<uint8_t>(e + 127));
    } else {
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        pk[i] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      *reinterpret_cast<uint4*>(args.out_bf16 + (size_t)row * args.out_ld + jb * 256 + 8 * lane) =
          make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
}

template <int BM, bool GATED, bool FP4A = false>
__global__ void __launch_bounds__(192, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tmW0,
                       const __grid_constant__ CUtensorMap tmW1,
                       const __grid_constant__ CUtensorMap tmS0,
                       const __grid_constant__ CUtensorMap tmS1,
                       const __grid_constant__ CUtensorMap tmX, const GemmArgs args) {
  using C = GemmCfg<BM, GATED, FP4A>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tile_base = smem;
  uint8_t* sf_base = smem + (size_t)C::STAGES * C::STAGE_BYTES;
  uint8_t* ctrl = sf_base + C::SF_RING;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_abort = abort_flag + 1;
  volatile int* split_last = epi_abort + 1;  // this CTA finished the item's last slice
  volatile int* epi_dry = split_last + 1;    // [4] per epilogue warp: its next pass is the dry one

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    *epi_abort = 0;
    for (int i = 0; i < 4; ++i) epi_dry[i] = 1;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    // every map a first k tile may need: its descriptor fetch is otherwise
    // in series with that tile's loads
    tma_prefetch_desc(&tmW0);
    tma_prefetch_desc(&tmW1);
    tma_prefetch_desc(&tmS0);
    tma_prefetch_desc(&tmS1);
    tma_prefetch_desc(&tmX);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int NB = args.nb_count;
  const int KT = args.kt_count;
  const int KT4 = KT >> 2;
  const int S = args.k_split;
  const int KTS = KT / S;
  const int total = *args.n_tiles * NB * S;
  const int step = (int)gridDim.x;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0)
      gemm_produce<C, GATED, FP4A>(&tmW0, &tmW1, &tmS0, &tmS1, &tmX, args, tile_base, sf_base, full, empty,
                                   abort_flag, NB, KT, KT4, total, step);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // acc_empty's first phase is the epilogue's dry pass (below), so the
      // first item waits for it to have read TMEM
      uint32_t aphase = 1;
      int sf_slot = 1;  // follows the producer's ring slot
      uint32_t sf_set = 0;  // FP4A: TMEM scale column set of the next k tile
      const uint32_t sfa_t = tmem + C::SFA_COL;
      const uint32_t sfb_t = tmem + C::SFB_COL;
      int4 tl_next = make_int4(0, 0, 0, 0);
      if ((int)blockIdx.x < total) tl_next = args.tiles[blockIdx.x / S / NB];
      for (int w = blockIdx.x; w < total && !*abort_flag; w += step) {
        const int4 tl = tl_next;
        if (w + step < total) tl_next = args.tiles[(w + step) / S / NB];
        if (filtered_out(args, tl.x >= args.n_routed)) continue;
        const int kt0 = (w % S) * KTS;
        const uint32_t b_fmt = tl.x >= args.n_routed ? 0u : 5u;  // e4m3 shared, e2m1 routed
        if (!mbar_wait(acc_empty, aphase ^ 1, DSV4_DEVERR_TIMEOUT_MMA)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kt = kt0; kt < kt0 + KTS; ++kt) {
          if (!mbar_wait(&full[stage], phase, DSV4_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = tile_base + (size_t)stage * C::STAGE_BYTES;
          if constexpr (FP4A) {
            // the stage's atoms into the column set the previous k tile's
            // MMAs are not reading; K = 64 per MMA: window kk / 2, scale
            // bytes {0,1} or {2,3} of it
            const uint8_t* sfs = st + C::TILE_BYTES;
            const uint32_t sfa_k = sfa_t + 24 * sf_set, sfb_k = sfa_k + 8;
            tc_cp_sf(sfa_k, sdesc_sf(smem_u32(sfs)));
            tc_cp_sf(sfa_k + 4, sdesc_sf(smem_u32(sfs + 512)));
            tc_cp_sf(sfb_k, sdesc_sf(smem_u32(sfs + 1024)));       // weight rows 0-127 (w1), window 0
            tc_cp_sf(sfb_k + 8, sdesc_sf(smem_u32(sfs + 1536)));   // rows 0-127, window 1
            tc_cp_sf(sfb_k + 4, sdesc_sf(smem_u32(sfs + 2048)));   // rows 128-255 (w3), window 0
            tc_cp_sf(sfb_k + 12, sdesc_sf(smem_u32(sfs + 2560)));  // rows 128-255, window 1
            const uint64_t adesc = sdesc_k_sw128(smem_u32(st));
            const uint64_t bdesc = sdesc_k_sw128(smem_u32(st + C::A_BYTES));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t id = (kk & 1) * 2;
              tc_mma_mxf4(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc_mxf4(256, id, id), sfa_k + 4 * (kk >> 1),
                          sfb_k + 8 * (kk >> 1), (kt > kt0 || kk > 0) ? 1u : 0u);
            }
            sf_set ^= 1;
            tc_commit(&empty[stage]);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          // one burst of scale copies per four k tiles, into the column set the
          // previous group's MMAs are not reading
          if ((kt & 3) == 0) sf_slot ^= 1;
          const uint8_t* sf = sf_base + (size_t)sf_slot * C::SF_GROUP;
          const uint32_t set = sf_slot;
          const uint32_t sfa_k = sfa_t + 4 * set;
          const uint32_t sfb_k = sfb_t + 32 * set + 8 * (kt & 3);
          if ((kt & 3) == 0) {
            tc_cp_sf(sfa_k, sdesc_sf(smem_u32(sf)));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tc_cp_sf(sfb_k + 8 * j, sdesc_sf(smem_u32(sf + 512 + 512 * j)));
              tc_cp_sf(sfb_k + 8 * j + 4, sdesc_sf(smem_u32(sf + 2560 + 512 * j)));
            }
          }
          const uint64_t adesc = sdesc_k_sw128(smem_u32(st));
          const uint64_t bdesc = sdesc_k_sw128(smem_u32(st + C::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t idesc = idesc_mxf8f6f4(0u, b_fmt, 256, kt & 3, kk);
            tc_mma_mxf8f6f4(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, sfa_k, sfb_k,
                            (kt > kt0 || kk > 0) ? 1u : 0u);
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
        tc_commit(acc_full);
        aphase ^= 1;
      }
      // drain every tcgen05 op of this CTA before TMEM is released
      tc_commit(final_bar);
      mbar_wait(final_bar, 0, DSV4_DEVERR_TIMEOUT_MMA);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Thread (warp quarter q, lane) owns token row 32q + lane of the tile and
    // the 256 accumulator columns of that row.  It copies them out of TMEM
    // (as packed bf16), releases the accumulator to the MMA warp, then does
    // the arithmetic and the stores while the next item's MMAs run.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    uint32_t aphase = 0;
    const float lim = args.swiglu_limit;
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    // The first pass is dry: the CTA's first item again, on whatever TMEM
    // holds before any MMA, without waiting for the accumulator.  It runs the
    // epilogue's instructions once while that item's MMAs are still
    // microseconds off, so that the real passes do not fetch them cold (the
    // unrolled GEMM1 arithmetic is thousands of instructions, and a decode
    // CTA's only item otherwise waits on those fetches).  Its release of the
    // accumulator is the first phase the MMA warp waits for, so no MMA writes
    // TMEM before the dry pass has read it.  Its stores go to the rows and
    // scale bytes that the same threads store again, later in program order,
    // in the item's real pass; nothing reads them before the kernel ends.  The
    // flag is read from shared memory so that the dry pass stays the same
    // code as the real ones.
    for (int w = (int)blockIdx.x - step; w < total; w += step) {
      const bool dry = epi_dry[q] != 0;
      __syncwarp();
      if (dry && lane == 0) epi_dry[q] = 0;
      const int wi = dry ? w + step : w;
      if (wi >= total) continue;  // dry pass of a CTA without items
      const int item = wi / S;
      const int4 tl = args.tiles[item / NB];
      if (filtered_out(args, tl.x >= args.n_routed)) {
        if (dry) {  // the MMA warp still counts the dry pass's release
          tc_fence_before();
          mbar_arrive(acc_empty);
        }
        continue;
      }
      const int jb = item % NB;
      const int row0 = tl.y, nrows = tl.z;
      // epi_abort is written only by epilogue warps and read between two
      // barriers, so all four see the same value.
      if (!dry && !mbar_wait(acc_full, aphase, DSV4_DEVERR_TIMEOUT_EPILOGUE)) {
        *epi_abort = 1;
        *abort_flag = 1;
      }
      epi_bar();
      const bool stop = *epi_abort != 0;
      epi_bar();
      if (stop) break;
      if (!dry) aphase ^= 1;
      tc_fence_after();
      const bool warp_rows = q * 32 < nrows;  // TMEM lanes of this quarter hold real rows
      if (S > 1) {
        if (dry) {
          tc_fence_before();
          mbar_arrive(acc_empty);
        } else {
          split_epilogue<GATED>(args, taddr, warp_rows, r, q, lane, item, wi % S, tl, jb, acc_empty,
                                split_last);
        }
        continue;
      }
      uint32_t pk[128];                       // packed bf16 pairs out of TMEM
      if (warp_rows) {
        // 64 columns in flight per wait: the accumulator goes back to the MMA
        // warp after four load round trips instead of sixteen
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t a[32], b[32];
          if (GATED) {  // pk[j] = (bf16 g_j, bf16 u_j) for j = 32c .. 32c+31
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
      mbar_arrive(acc_empty);
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
            // silu with the hardware exp2 and reciprocal: a few ulp of fp32, far
            // below the bf16 rounding of h that follows
            const float s = __fdividef(gb, 1.0f + __expf(-gb));
            const float hv = bf16_round((s * ub) * wr);
            amax = fmaxf(amax, fabsf(hv));
            pk[j] = __float_as_uint(hv);
          }
          if constexpr (FP4A) {
            // FP4 h for the FP4 GEMM2: four 32-value blocks (fp4_act_quant
            // semantics), 64 packed bytes per row of this 128-wide window jb,
            // scale bytes into the per-32 atoms of window jb
            (void)amax;
            uint8_t* dst = args.out_q + (size_t)row * (args.out_ld / 2) + jb * 64;
            const int KW = args.out_ld >> 7, g = row >> 5;
#pragma unroll
            for (int blk = 0; blk < 4; ++blk) {
              float v32[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) v32[i] = __uint_as_float(pk[32 * blk + i]);
              uint4 packed;
              const int e4 = fp4_block_quant(v32, packed);
              *reinterpret_cast<uint4*>(dst + 16 * blk) = packed;
#pragma unroll
              for (int m1 = 0; m1 < 4; ++m1)
                if (g - m1 >= 0)
                  args.out_sf[((size_t)(g - m1) * KW + jb) * 512 + (row & 31) * 16 + m1 * 4 + blk] =
                      static_cast<uint8_t>(e4 + 127);
            }
          } else {
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
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(args.out_bf16 + (size_t)row * args.out_ld + jb * 256);
#pragma unroll
          for (int v = 0; v < 32; ++v)
            dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
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
                        long long slot_stride, int l2_promotion) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return DSV4_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 31) || (slot_stride & 31) || (K % 128) ||
      ((K / 2) % 32))
    return DSV4_ERR_ARG;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)slots};
  cuuint64_t strides[2] = {(cuuint64_t)(K / 2), (cuuint64_t)slot_stride};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  const CUtensorMapL2promotion promo =
      l2_promotion >= 256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
      : l2_promotion >= 128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
      : l2_promotion >= 64  ? CU_TENSOR_MAP_L2_PROMOTION_L2_64B
                            : CU_TENSOR_MAP_L2_PROMOTION_NONE;
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void*>(base), dims,
                   strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSV4_OK : DSV4_ERR_CUDA;
}

// FP4 e2m1 weights of every arena slot read as packed bytes (two codes per
// byte, for kind::mxf4): dims {K/2 bytes, rows, slots}, box {128 bytes = 256
// values, 128 rows, 1}.
int make_tmap_fp4_packed_arena(CUtensorMap* m, const void* base, int K, int rows, int slots,
                               long long slot_stride, int l2_promotion) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return DSV4_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (slot_stride & 15) || (K % 256)) return DSV4_ERR_ARG;
  cuuint64_t dims[3] = {(cuuint64_t)(K / 2), (cuuint64_t)rows, (cuuint64_t)slots};
  cuuint64_t strides[2] = {(cuuint64_t)(K / 2), (cuuint64_t)slot_stride};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  const CUtensorMapL2promotion promo =
      l2_promotion >= 256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
      : l2_promotion >= 128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
      : l2_promotion >= 64  ? CU_TENSOR_MAP_L2_PROMOTION_L2_64B
                            : CU_TENSOR_MAP_L2_PROMOTION_NONE;
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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

// bf16 row-major matrix [rows][K], box {64 elements = 128 bytes, box_rows}.
int make_tmap_bf16(CUtensorMap* m, const void* base, int K, int rows, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return DSV4_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K % 64)) return DSV4_ERR_ARG;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSV4_OK : DSV4_ERR_CUDA;
}

template <int BM, bool GATED>
static int launch_one(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& s0,
                      const CUtensorMap& s1, const CUtensorMap& b, const GemmArgs& args, int grid,
                      cudaStream_t st) {
  using C = GemmCfg<BM, GATED>;
  if (ensure_smem_attr(reinterpret_cast<const void*>(expert_gemm_kernel<BM, GATED>),
                       (int)C::SMEM_BYTES))
    return DSV4_ERR_CUDA;
  launch_k(expert_gemm_kernel<BM, GATED>, grid, 192, C::SMEM_BYTES, st,
           a0, a1, s0, s1, b, args);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

template <int BM, bool GATED>
static int launch_one_fp4(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b, const GemmArgs& args,
                          int grid, cudaStream_t st) {
  using C = GemmCfg<BM, GATED, true>;
  if (ensure_smem_attr(reinterpret_cast<const void*>(expert_gemm_kernel<BM, GATED, true>), (int)C::SMEM_BYTES))
    return DSV4_ERR_CUDA;
  launch_k(expert_gemm_kernel<BM, GATED, true>, grid, 192, C::SMEM_BYTES, st, a0, a1, a0, a1, b, args);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_expert_gemm_fp4(bool gated, int block_n, const CUtensorMap& a0, const CUtensorMap& a1,
                           const CUtensorMap& b, const GemmArgs& args, int grid, cudaStream_t st) {
  if (args.seg_filter != 1 || args.k_split != 1) return DSV4_ERR_ARG;  // routed items, unsplit
  if (gated) {
    switch (block_n) {
      case 32: return launch_one_fp4<32, true>(a0, a1, b, args, grid, st);
      case 64: return launch_one_fp4<64, true>(a0, a1, b, args, grid, st);
      case 128: return launch_one_fp4<128, true>(a0, a1, b, args, grid, st);
      default: return DSV4_ERR_ARG;
    }
  }
  switch (block_n) {
    case 32: return launch_one_fp4<32, false>(a0, a1, b, args, grid, st);
    case 64: return launch_one_fp4<64, false>(a0, a1, b, args, grid, st);
    case 128: return launch_one_fp4<128, false>(a0, a1, b, args, grid, st);
    default: return DSV4_ERR_ARG;
  }
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
