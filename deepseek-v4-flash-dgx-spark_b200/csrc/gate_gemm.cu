// Gate on the tensor core for large batches: logits = x . Wg^T (bf16 x bf16,
// fp32 accumulate, tcgen05 kind::f16) with the whole routing step fused into
// the epilogue.
//
// Orientation: A = BM token rows of x (M = 128 MMA; rows past BM read the
// following smem and land in TMEM lanes nobody reads), B = all E = 256 gate
// rows (N = 256).  Each epilogue thread therefore holds the 256 logits of its
// token and does, in registers, exactly what gate_topk_kernel does: canonical
// sigmoid, + correction bias, top-k with ties to the lower expert id,
// renormalise in rank order, x route_scale - the same bits.  It also writes
// the fp32 logits row.  Replaces the official Gate.forward called at
// spark_runtime/lazy_official_runtime.py:983.  Small batches use the split
// form (64-expert blocks x K slices, partial logits summed by
// gate_topk_kernel) so that many SMs share the 2 MB of gate weights.
#include "kernels.cuh"

namespace dsv4 {

template <int BM, int NE>
struct GateCfg {
  static constexpr int KT_ELEMS = 64;            // bf16 per 128-byte row of a k tile
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = NE * 128;       // NE gate rows (experts) per item
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 6 ? 6 : (200 * 1024) / STAGE_BYTES;
  // The M = 128 MMA reads a 16 KB A window from every stage's A base; for the
  // last stage it reaches past the ring into the control block and this pad,
  // which keeps it inside the CTA's shared memory.
  static constexpr int A_WINDOW_PAD = 128 * 128;
  static constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256 + A_WINDOW_PAD;
  static constexpr int TMEM_COLS = NE < 32 ? 32 : NE;
  static_assert(A_BYTES % 1024 == 0, "1024-byte aligned tiles");
};

// FUSED: NE = 256 experts per item, whole K, routing in the epilogue.
// Otherwise: items = (token tile, NE-expert block, K slice); the epilogue
// writes fp32 partial logits partial[slice][token][expert] that
// gate_topk_kernel sums in slice order.
template <int BM, int NE, bool FUSED>
__global__ void __launch_bounds__(192, 1)
    gate_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     int T, int H, int E, int ksplit, const float* __restrict__ bias, int k,
                     float route_scale, float* __restrict__ logits, float* __restrict__ weights,
                     int64_t* __restrict__ indices) {
  using C = GateCfg<BM, NE>;
  static_assert(!FUSED || NE == 256, "fused routing needs every expert in one accumulator");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ctrl = smem + (size_t)C::STAGES * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_abort = abort_flag + 1;

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
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int KT = H / C::KT_ELEMS;
  const int KTS = KT / ksplit;                 // k tiles per slice
  const int n_eb = E / NE;
  const int n_items = (T + BM - 1) / BM * n_eb * ksplit;
  const int step = (int)gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int it = blockIdx.x; it < n_items && !*abort_flag; it += step) {
        const int ks = it % ksplit, eb = (it / ksplit) % n_eb, tt = it / (ksplit * n_eb);
        for (int kt = ks * KTS; kt < (ks + 1) * KTS; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, DSV4_DEVERR_TIMEOUT_PRODUCER)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* st = smem + (size_t)stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::A_BYTES + C::B_BYTES);
          tma_load_2d(st, &tmX, &full[stage], kt * C::KT_ELEMS, tt * BM);
          tma_load_2d(st + C::A_BYTES, &tmW, &full[stage], kt * C::KT_ELEMS, eb * NE);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 10000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, aphase = 0;
      const uint32_t idesc = idesc_bf16(NE);
      for (int it = blockIdx.x; it < n_items && !*abort_flag; it += step) {
        if (!mbar_wait(acc_empty, aphase ^ 1, DSV4_DEVERR_TIMEOUT_MMA)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kt = 0; kt < KTS; ++kt) {
          if (!mbar_wait(&full[stage], phase, DSV4_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + (size_t)stage * C::STAGE_BYTES;
          const uint64_t adesc = sdesc_k_sw128(smem_u32(st));
          const uint64_t bdesc = sdesc_k_sw128(smem_u32(st + C::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // K = 16 bf16 (32 bytes) per MMA
            tc_mma_f16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
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
      tc_commit(final_bar);
      mbar_wait(final_bar, 0, DSV4_DEVERR_TIMEOUT_MMA);
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t aphase = 0;
    for (int it = blockIdx.x; it < n_items; it += step) {
      if (!mbar_wait(acc_full, aphase, DSV4_DEVERR_TIMEOUT_EPILOGUE)) {
        *epi_abort = 1;
        *abort_flag = 1;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const bool stop = *epi_abort != 0;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (stop) break;
      aphase ^= 1;
      tc_fence_after();
      const int ks = it % ksplit, eb = (it / ksplit) % n_eb, tt = it / (ksplit * n_eb);
      const int t = tt * BM + r;
      const bool live = (q * 32 < BM) && (tt * BM + q * 32 < T);  // warp holds real rows
      if (!FUSED) {
        if (live) {
#pragma unroll 1
          for (int c = 0; c < NE; c += 16) {
            float v[16];
            tmem_ld16(taddr + c, v);
            if (t < T) {
              float4* lp = reinterpret_cast<float4*>(logits + ((size_t)ks * T + t) * E + eb * NE + c);
              lp[0] = make_float4(v[0], v[1], v[2], v[3]);
              lp[1] = make_float4(v[4], v[5], v[6], v[7]);
              lp[2] = make_float4(v[8], v[9], v[10], v[11]);
              lp[3] = make_float4(v[12], v[13], v[14], v[15]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(acc_empty);
        continue;
      }
      // running top-k of (score + bias): descending, ties to the lower id
      float tsel[8], tscore[8];
      int tidx[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        tsel[j] = -INFINITY;
        tscore[j] = 0.f;
        tidx[j] = 0x7fffffff;
      }
      if (live) {
#pragma unroll 1
        for (int c = 0; c < 256; c += 16) {
          float v[16];
          tmem_ld16(taddr + c, v);
          if (t < T) {
            float4* lp = reinterpret_cast<float4*>(logits + (size_t)t * 256 + c);
            lp[0] = make_float4(v[0], v[1], v[2], v[3]);
            lp[1] = make_float4(v[4], v[5], v[6], v[7]);
            lp[2] = make_float4(v[8], v[9], v[10], v[11]);
            lp[3] = make_float4(v[12], v[13], v[14], v[15]);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = c + i;
            const float s = sigmoid_canonical(v[i]);
            const float sel = bias ? __fadd_rn(s, bias[e]) : s;
            // insert after every entry with sel >= this one (earlier ids win ties)
            if (sel > tsel[7]) {
              float cs = sel, cc = s;
              int ce = e;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (cs > tsel[j]) {
                  const float ts = tsel[j], tc = tscore[j];
                  const int te = tidx[j];
                  tsel[j] = cs;
                  tscore[j] = cc;
                  tidx[j] = ce;
                  cs = ts;
                  cc = tc;
                  ce = te;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
      if (live && t < T) {
        float total = tscore[0];
#pragma unroll
        for (int j = 1; j < 8; ++j)
          if (j < k) total = __fadd_rn(total, tscore[j]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j < k) {
            weights[(size_t)t * k + j] = __fmul_rn(__fdiv_rn(tscore[j], total), route_scale);
            indices[(size_t)t * k + j] = tidx[j];
          }
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

int make_tmap_bf16(CUtensorMap* m, const void* base, int K, int rows, int box_rows);

template <int BM, int NE, bool FUSED>
static int launch_gate_gemm_cfg(const void* x, const void* w, int T, int H, int E, int ksplit,
                                const float* bias, int k, float route_scale, float* out,
                                float* weights, int64_t* indices, int num_sms, cudaStream_t st) {
  using C = GateCfg<BM, NE>;
  CUtensorMap tx, tw;
  int rc;
  if ((rc = make_tmap_bf16(&tx, x, H, T, BM))) return rc;
  if ((rc = make_tmap_bf16(&tw, w, H, E, NE))) return rc;
  if (ensure_smem_attr(reinterpret_cast<const void*>(gate_gemm_kernel<BM, NE, FUSED>),
                       (int)C::SMEM_BYTES))
    return DSV4_ERR_CUDA;
  const int items = (T + BM - 1) / BM * (E / NE) * ksplit;
  const int grid = items < num_sms ? items : num_sms;
  launch_k(gate_gemm_kernel<BM, NE, FUSED>, grid, 192, C::SMEM_BYTES, st,
           tx, tw, T, H, E, ksplit, bias, k, route_scale, out, weights, indices);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

// Split configuration of the small-batch gate: 64-expert blocks x K slices,
// enough items to cover the SMs, slices of at least 4 k tiles.
void gate_gemm_split_shape(int T, int H, int E, int num_sms, int* bm, int* ksplit) {
  const int b = T <= 32 ? 32 : (T <= 64 ? 64 : 128);
  const int tiles = (T + b - 1) / b;
  int s = 1;
  const int kt = H / 64;
  while (s * 2 * tiles * (E / 64) <= num_sms && kt % (s * 2) == 0 && kt / (s * 2) >= 4) s *= 2;
  *bm = b;
  *ksplit = s;
}

int launch_gate_gemm_partials(const void* x, const void* w, int T, int H, int E, float* partials,
                              int num_sms, cudaStream_t st) {
  int bm, ks;
  gate_gemm_split_shape(T, H, E, num_sms, &bm, &ks);
  switch (bm) {
    case 32: return launch_gate_gemm_cfg<32, 64, false>(x, w, T, H, E, ks, nullptr, 0, 0.f, partials,
                                                        nullptr, nullptr, num_sms, st);
    case 64: return launch_gate_gemm_cfg<64, 64, false>(x, w, T, H, E, ks, nullptr, 0, 0.f, partials,
                                                        nullptr, nullptr, num_sms, st);
    default: return launch_gate_gemm_cfg<128, 64, false>(x, w, T, H, E, ks, nullptr, 0, 0.f,
                                                         partials, nullptr, nullptr, num_sms, st);
  }
}

int launch_gate_gemm_topk(const void* x, const void* w, int T, int H, const float* bias, int k,
                          float route_scale, float* logits, float* weights, int64_t* indices,
                          int num_sms, cudaStream_t st) {
  // 64-row tiles until they would leave SMs idle with 128-row tiles
  if ((T + 127) / 128 >= num_sms)
    return launch_gate_gemm_cfg<128, 256, true>(x, w, T, H, 256, 1, bias, k, route_scale, logits,
                                                weights, indices, num_sms, st);
  return launch_gate_gemm_cfg<64, 256, true>(x, w, T, H, 256, 1, bias, k, route_scale, logits,
                                             weights, indices, num_sms, st);
}

}  // namespace dsv4
