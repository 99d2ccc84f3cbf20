// Gate: logits = x . Wg^T (fp32), then sigmoid scores, correction bias, top-k,
// renormalise, routed scale.  Replaces the official Gate.forward(x, input_ids)
// that the reference calls at spark_runtime/lazy_official_runtime.py:983.
#include "kernels.cuh"

namespace dsv4 {

// ---------------------------------------------------------------------------
// Canonical fp32 sigmoid.  exp() is Cody & Waite range reduction with the
// two-constant split of ln 2 used by Moshier's Cephes expf (C1 = 355/512,
// C2 = -2.12194440e-4) and the degree-7 Taylor polynomial of e^r in Horner
// form.  Every step is a single round-to-nearest fp32 operation (no FMA
// contraction), so the CPU restatement reproduces it bit for bit.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float exp_canonical(float t) {
  const float n = rintf(__fmul_rn(t, 1.4426950408889634f));
  float r = __fsub_rn(t, __fmul_rn(n, 0.693359375f));
  r = __fsub_rn(r, __fmul_rn(n, -2.12194440e-4f));
  float p = 1.0f / 5040.0f;
  p = __fadd_rn(__fmul_rn(p, r), 1.0f / 720.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f / 120.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f / 24.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f / 6.0f);
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  return __fmul_rn(p, exp2i(static_cast<int>(n)));
}

__device__ __forceinline__ float sigmoid_canonical(float x) {
  const float t = fminf(fmaxf(-x, -80.0f), 80.0f);
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_canonical(t)));
}

// ---------------------------------------------------------------------------
// Logits.  Each CTA owns EPC experts: their gate rows are staged in shared
// memory as fp32, then each warp walks tokens and accumulates EPC dot
// products with 16-byte loads of x, reduced across the warp.
// ---------------------------------------------------------------------------
constexpr int kGateEPC = 2;
constexpr int kGateThreads = 256;

template <bool W_FP32>
__global__ void __launch_bounds__(kGateThreads) gate_logits_kernel(
    const __nv_bfloat16* __restrict__ x, const void* __restrict__ w, int T, int H, int E,
    float* __restrict__ logits) {
  extern __shared__ float ws[];  // [kGateEPC][H] fp32
  const int e0 = blockIdx.x * kGateEPC;
  const int ne = min(kGateEPC, E - e0);
  // Stage the gate rows with 16-byte loads, every load of a thread issued
  // before any is used (the rows come from DRAM: latency, not bandwidth).
  const int vec = W_FP32 ? 4 : 8;  // elements per 16-byte load
  const int nvec = kGateEPC * H / vec;
  constexpr int kMaxPerThread = 16;
  uint4 buf[kMaxPerThread];
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) {
    const int v = threadIdx.x + u * kGateThreads;
    buf[u] = make_uint4(0, 0, 0, 0);
    if (v < nvec && (v * vec) / H < ne) {
      const char* base = static_cast<const char*>(w) + (size_t)e0 * H * (W_FP32 ? 4 : 2);
      buf[u] = __ldg(reinterpret_cast<const uint4*>(base) + v);
    }
  }
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) {
    const int v = threadIdx.x + u * kGateThreads;
    if (v < nvec) {
      float* dst = ws + v * vec;
      if (W_FP32) {
        *reinterpret_cast<uint4*>(dst) = buf[u];
      } else {
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&buf[u]);
        float4 lo, hi;
        lo.x = __bfloat162float(b[0]); lo.y = __bfloat162float(b[1]);
        lo.z = __bfloat162float(b[2]); lo.w = __bfloat162float(b[3]);
        hi.x = __bfloat162float(b[4]); hi.y = __bfloat162float(b[5]);
        hi.z = __bfloat162float(b[6]); hi.w = __bfloat162float(b[7]);
        reinterpret_cast<float4*>(dst)[0] = lo;
        reinterpret_cast<float4*>(dst)[1] = hi;
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = kGateThreads >> 5;
  for (int t = warp; t < T; t += nwarps) {
    float acc[kGateEPC];
#pragma unroll
    for (int j = 0; j < kGateEPC; ++j) acc[j] = 0.f;
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)t * H);
#pragma unroll 4
    for (int c = lane; c < H / 8; c += 32) {
      const uint4 raw = __ldg(xr + c);
      const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&raw);
      float xf[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) xf[i] = __bfloat162float(xv[i]);
#pragma unroll
      for (int j = 0; j < kGateEPC; ++j) {
        const float4* wr = reinterpret_cast<const float4*>(ws + j * H + c * 8);
        const float4 a = wr[0], b = wr[1];
        acc[j] = fmaf(xf[0], a.x, acc[j]);
        acc[j] = fmaf(xf[1], a.y, acc[j]);
        acc[j] = fmaf(xf[2], a.z, acc[j]);
        acc[j] = fmaf(xf[3], a.w, acc[j]);
        acc[j] = fmaf(xf[4], b.x, acc[j]);
        acc[j] = fmaf(xf[5], b.y, acc[j]);
        acc[j] = fmaf(xf[6], b.z, acc[j]);
        acc[j] = fmaf(xf[7], b.w, acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kGateEPC; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    if (lane == 0) {
      for (int j = 0; j < ne; ++j) logits[(size_t)t * E + e0 + j] = acc[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Top-k.  One CTA per token.  The selecting warp's lane l holds experts l,
// l+32, ...; k rounds of a warp arg-max on (score + bias), ties to the lower
// expert id.
// ---------------------------------------------------------------------------
constexpr int kMaxExpertsPerLane = 16;  // E <= 512
constexpr int kMaxTopk = 8;
constexpr int kSliceBatch = 8;  // split-K slices loaded together

// The logit at src from nsplit split-K partial slices `slice` floats apart,
// summed in slice order in fp32 (loads issued kSliceBatch at a time).
__device__ __forceinline__ float sum_slices(const float* src, int nsplit, size_t slice) {
  float lg = src[0];
  for (int sl0 = 1; sl0 < nsplit; sl0 += kSliceBatch) {
    float v[kSliceBatch];
#pragma unroll
    for (int j = 0; j < kSliceBatch; ++j) v[j] = sl0 + j < nsplit ? src[(size_t)(sl0 + j) * slice] : 0.f;
#pragma unroll
    for (int j = 0; j < kSliceBatch; ++j)
      if (sl0 + j < nsplit) lg = __fadd_rn(lg, v[j]);
  }
  return lg;
}

// Top-k of one token by one warp, from its sigmoid scores (s_score) and
// selection values (s_sel = score + bias) in shared memory: k rounds of a warp
// arg-max on s_sel, ties to the lower expert id; lane r < k gets the rank-r
// expert and its weight (its score over the sum of the k picked scores, summed
// in rank order, times route_scale).
__device__ __forceinline__ void warp_topk(const float* s_score, const float* s_sel, int E, int k,
                                          float route_scale, int lane, float* w_out, int* e_out) {
  float score[kMaxExpertsPerLane], sel[kMaxExpertsPerLane];
  const int per = (E + 31) / 32;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    if (i < per && e < E) {
      score[i] = s_score[e];
      sel[i] = s_sel[e];
    } else {
      score[i] = 0.f;
      sel[i] = -INFINITY;
    }
  }
  float total = 0.f;
  float my_w = 0.f;  // lane r keeps the rank-r pick
  int my_e = 0;
#pragma unroll
  for (int r = 0; r < kMaxTopk; ++r) {
    if (r >= k) break;
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      // experts of a lane increase with i, so '>' keeps the lower id on ties
      if (sel[i] > best) {
        best = sel[i];
        best_e = lane + 32 * i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    // the owning lane retires the winner and broadcasts its raw score
    float w = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      if (lane + 32 * i == best_e) {
        w = score[i];
        sel[i] = -INFINITY;
      }
    }
    w = __shfl_sync(0xffffffffu, w, best_e & 31);
    total = (r == 0) ? w : __fadd_rn(total, w);
    if (lane == r) {
      my_w = w;
      my_e = best_e;
    }
  }
  float w = 0.f;
  if (lane < k) w = __fmul_rn(__fdiv_rn(my_w, total), route_scale);
  *w_out = w;
  *e_out = my_e;
}

// With nsplit > 1, `logits` holds nsplit partial slices [nsplit][T][E] that are
// summed in slice order (fp32) and the sums are written to logits_out.
__global__ void __launch_bounds__(512) gate_topk_kernel(const float* __restrict__ logits,
                                                        int nsplit, float* __restrict__ logits_out,
                                                        const float* __restrict__ bias, int T,
                                                        int E, int k, float route_scale,
                                                        float* __restrict__ weights,
                                                        int64_t* __restrict__ indices,
                                                        const int64_t* __restrict__ hash_table,
                                                        const int64_t* __restrict__ input_ids,
                                                        long long vocab) {
  // One CTA per token, one thread per expert: each thread sums its expert's
  // split-K slices in slice order (loads issued kSliceBatch at a time so they
  // are in flight together), then warp 0 selects the top k from shared memory.
  __shared__ float s_score[kMaxExpertsPerLane * 32], s_sel[kMaxExpertsPerLane * 32];
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const float lg = sum_slices(logits + (size_t)t * E + e, nsplit, (size_t)T * E);
    if (logits_out) logits_out[(size_t)t * E + e] = lg;
    const float s = sigmoid_canonical(lg);
    s_score[e] = s;
    s_sel[e] = bias ? __fadd_rn(s, bias[e]) : s;
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  if (hash_table) {
    // hash-routed layer: the experts are the table row of the token id (rank
    // order of the row), the weights their scores renormalised in that order
    const long long id = input_ids[t];
    int e = -1;
    if (lane < k) {
      if (id >= 0 && id < vocab) {
        const int64_t v = hash_table[id * k + lane];
        if (v >= 0 && v < E) e = static_cast<int>(v);
      }
      if (e < 0) record_error(DSV4_DEVERR_BAD_INDEX);
    }
    const float w = e >= 0 ? s_score[e] : 0.f;
    float total = 0.f;
    for (int r = 0; r < k; ++r) {
      const float wr = __shfl_sync(0xffffffffu, w, r);
      total = (r == 0) ? wr : __fadd_rn(total, wr);
    }
    if (lane < k) {
      weights[(size_t)t * k + lane] = e >= 0 ? __fmul_rn(__fdiv_rn(w, total), route_scale) : 0.f;
      indices[(size_t)t * k + lane] = e;
    }
    return;
  }
  float w;
  int e;
  warp_topk(s_score, s_sel, E, k, route_scale, lane, &w, &e);
  if (lane < k) {
    weights[(size_t)t * k + lane] = w;
    indices[(size_t)t * k + lane] = e;
  }
}

int launch_gate_logits(const void* x, const void* w, int w_is_fp32, int T, int H, int E,
                       float* logits, cudaStream_t st) {
  const int grid = (E + kGateEPC - 1) / kGateEPC;
  const size_t smem = (size_t)kGateEPC * H * sizeof(float);
  if (w_is_fp32) {
    if (ensure_smem_attr(reinterpret_cast<const void*>(gate_logits_kernel<true>), (int)smem))
      return DSV4_ERR_CUDA;
    launch_k(gate_logits_kernel<true>, grid, kGateThreads, smem, st,
             static_cast<const __nv_bfloat16*>(x), w, T,
                                                      H, E, logits);
  } else {
    if (ensure_smem_attr(reinterpret_cast<const void*>(gate_logits_kernel<false>), (int)smem))
      return DSV4_ERR_CUDA;
    launch_k(gate_logits_kernel<false>, grid, kGateThreads, smem, st,
             static_cast<const __nv_bfloat16*>(x), w,
                                                       T, H, E, logits);
  }
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_gate_topk(const float* logits, const float* bias, int T, int E, int k,
                     float route_scale, float* weights, int64_t* indices, cudaStream_t st,
                     int nsplit, float* logits_out, const int64_t* hash_table,
                     const int64_t* input_ids, long long vocab) {
  const int threads = std::min(kMaxExpertsPerLane * 32, (E + 31) / 32 * 32);
  if (T > 0) {
    launch_k(gate_topk_kernel, T, threads, 0, st, logits, nsplit, logits_out, bias, T, E, k,
             route_scale, weights, indices, hash_table, input_ids, vocab);
  }
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

}  // namespace dsv4
