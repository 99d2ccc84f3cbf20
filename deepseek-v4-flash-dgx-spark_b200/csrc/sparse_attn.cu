// Sparse attention of the DeepSeek-V4 attention block on the tensor core.
//
// Replaces the official kernel.sparse_attn (TileLang; its shared-memory
// request fails at h=64, d=512 on GB10, LOG.md E025) and the reference's
// per-token Python fallback spark_runtime/lazy_official_runtime.py:1024-1049:
//
//   out[b,s,h] = sum_j p[h,j] kv[b, idx_j]   over the valid (>= 0) indices of
//   topk_idxs[b,s], with p[h,j] = exp(z[h,j] - m[h]) / (sum_j exp(z - m)
//   + exp(sink[h] - m)), z[h,j] = scale * q[b,s,h] . kv[b,idx_j],
//   m[h] = max(max_j z[h,j], sink[h]); zeros when no index is valid.
//
// One KV row serves every head (kv [B,N,D], q [B,S,H,D], H = 64, D = 512), so
// each query token is two small GEMMs over the gathered rows:
//   S^T[j,h] = C[j,:] . Q[h,:]     M = 128 gathered rows, N = 64 heads, K = 512
//   O^T[d,h] += C^T[d,j] . P[h,j]  M = 128 of the 512 d, N = 64 heads, K = 128 rows
// C (128 gathered rows, K-major, 128-byte swizzled 64-element k tiles) is read
// by the second product as an MN-major operand: the same bytes are the
// canonical MN-major layout of C^T (64-element d chunks 16 KB apart, 8-row
// groups 1 KB apart), so no transpose is ever written.  Both products run on
// tcgen05 (kind::f16, bf16 inputs, fp32 accumulators in TMEM).
//
// Each CTA takes one query token and a range of 128-row chunks of its index
// list (a split).  Pass 1 computes the scores chunk by chunk and keeps the
// running per-head max and sum of exponentials; pass 2 recomputes the scores,
// forms the final probabilities in bf16 and accumulates O^T in TMEM.  A token
// with one split writes out directly; several splits write fp32 partials
// (max, sum, unnormalised O) that sparse_attn_combine_kernel merges with the
// sink term.
//
// Warp roles (256 threads): all warps gather rows (cp.async, 16 B); warp 0,
// lane 0 issues the MMAs; warps 0-3 own the TMEM lane quarters (lane = gathered
// row in the score product, = d in the output product).
#include "kernels.cuh"

namespace dsv4 {

constexpr int kSaHeads = 64;
constexpr int kSaDim = 512;
constexpr int kSaChunk = 128;                  // gathered rows per chunk
constexpr int kSaThreads = 256;
constexpr int kSaQBytes = kSaHeads * kSaDim * 2;   // 64 KB: Q, 8 k tiles of [64 rows][128 B]
constexpr int kSaCBytes = kSaChunk * kSaDim * 2;   // 128 KB: C, 8 k tiles of [128 rows][128 B]
constexpr int kSaPBytes = kSaHeads * kSaChunk * 2; // 16 KB: P, 2 k tiles of [64 rows][128 B]
constexpr int kSaCtrl = 4096;  // barrier, TMEM slot, 128 row indices, reductions
constexpr size_t kSaSmem = 1024 + kSaQBytes + kSaCBytes + kSaPBytes + kSaCtrl;
constexpr int kSaTmemCols = 512;  // S: cols 0..63; O^T: 4 d tiles x 64 cols at 256..511

// Byte offset of element (row, col) of a K-major tile set: 64-element k tiles of
// [rows][128 B], 128-byte swizzle (16-byte unit index XOR row % 8).
__device__ __forceinline__ uint32_t sw128_offset(int rows, int row, int col) {
  const int kt = col >> 6, unit = (col & 63) >> 3;
  return (uint32_t)kt * rows * 128 + row * 128 + ((unit ^ (row & 7)) << 4) + ((col & 7) << 1);
}

// Descriptor of a K-major, 128-byte swizzled operand (as sdesc_k_sw128) and of
// the MN-major view of the same layout: MN chunks of 64 elements LBO bytes
// apart, groups of 8 K rows 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor: bf16 A and B, fp32 D, M = 128, N = n;
// a_mn / b_mn select the MN-major form of A / B.
__host__ __device__ constexpr uint32_t idesc_bf16_major(uint32_t n, uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) |
         ((128u >> 4) << 24);
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(reinterpret_cast<uint64_t>(g))
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Load 64 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t a[32], b[32];
  tmem_ld32_issue(taddr, a);
  tmem_ld32_issue(taddr + 32, b);
  tmem_wait_ld2(a, b);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = __uint_as_float(a[i]);
    v[32 + i] = __uint_as_float(b[i]);
  }
}

struct SaArgs {
  const __nv_bfloat16* q;     // [B,S,H,D]
  const __nv_bfloat16* kv;    // [B,N,D]
  const float* sink;          // [H]
  const int* idx;             // [B,S,K]
  __nv_bfloat16* out;         // [B,S,H,D]
  float* part_o;              // [tokens][splits][H][D] (splits > 1)
  float* part_ml;             // [tokens][splits][H][2]: max, sum (splits > 1)
  int S, N, K;                // query positions per batch, kv rows per batch, indices per query
  int splits, chunks_per_split;
  float scale;
};

__global__ void __launch_bounds__(kSaThreads, 1) sparse_attn_kernel(const SaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sC = sQ + kSaQBytes;
  uint8_t* sP = sC + kSaCBytes;
  uint8_t* ctrl = sP + kSaPBytes;
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(ctrl);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 8);
  int* s_idx = reinterpret_cast<int*>(ctrl + 16);            // [128] this chunk's kv rows (-1 invalid)
  // [4 quarters][64] partial reductions, [64] reduced, [64] final max, [64] final 1 / sum: 448 floats
  float* s_red = reinterpret_cast<float*>(ctrl + 16 + 4 * kSaChunk);
  static_assert(16 + 4 * kSaChunk + 448 * 4 <= kSaCtrl, "control block too small");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int token = blockIdx.x / a.splits, split = blockIdx.x % a.splits;
  const int b = token / a.S;
  const int n_chunks = (a.K + kSaChunk - 1) / kSaChunk;
  const int c_begin = split * a.chunks_per_split;
  const int c_end = min(n_chunks, c_begin + a.chunks_per_split);
  const __nv_bfloat16* kvb = a.kv + (size_t)b * a.N * kSaDim;
  const int* idx = a.idx + (size_t)token * a.K;

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kSaTmemCols);
    tmem_relinquish();
  }
  // Q of this token: 64 rows x 512, swizzled K-major
  const __nv_bfloat16* qt = a.q + (size_t)token * kSaHeads * kSaDim;
  for (int u = tid; u < kSaHeads * kSaDim / 8; u += kSaThreads) {
    const int row = u / (kSaDim / 8), col = (u % (kSaDim / 8)) * 8;
    cp_async16(smem_u32(sQ + sw128_offset(kSaHeads, row, col)), qt + (size_t)row * kSaDim + col);
  }
  cp_async_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem;          // scores: 64 columns
  const uint32_t t_o = tmem + 256;    // O^T: 4 x 64 columns
  const int q4 = warp & 3;            // TMEM lane quarter of warps 0-3 and 4-7
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const bool tmem_warp = warp < 4;    // warps 0-3 read the accumulators (lanes = their quarter)

  float m_run = -INFINITY, l_run = 0.f;  // per head (thread h < 64 of warps 0-1 keeps head h)
  uint32_t mma_phase = 0;
  bool any_valid = false;
  // A wait that runs out fails the whole CTA at once (every thread leaves the
  // chunk loops at the same point, so no barrier is left waiting).
  bool failed = false;

  // gather chunk c into sC (K-major swizzled), indices into s_idx
  auto gather = [&](int c) {
    for (int j = tid; j < kSaChunk; j += kSaThreads) {
      const int p = c * kSaChunk + j;
      int r = p < a.K ? idx[p] : -1;
      if (r >= a.N) {
        record_error(DSV4_DEVERR_BAD_INDEX);
        r = -1;
      }
      s_idx[j] = r;
    }
    __syncthreads();
    for (int u = tid; u < kSaChunk * kSaDim / 8; u += kSaThreads) {
      const int row = u / (kSaDim / 8), col = (u % (kSaDim / 8)) * 8;
      const int r = s_idx[row];
      const uint32_t dst = smem_u32(sC + sw128_offset(kSaChunk, row, col));
      if (r >= 0)
        cp_async16(dst, kvb + (size_t)r * kSaDim + col);
      else
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
    }
    cp_async_wait_all();
    fence_proxy_async_shared();  // the generic-proxy writes, before the tensor core reads them
    __syncthreads();
  };

  // S^T = C . Q^T into t_s; waits for completion (bounded)
  auto scores = [&]() -> bool {
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_major(kSaHeads, 0, 0);
#pragma unroll 1
      for (int kt = 0; kt < kSaDim / 64; ++kt) {
        const uint64_t ad = sdesc_k_sw128(smem_u32(sC + kt * kSaChunk * 128));
        const uint64_t bd = sdesc_k_sw128(smem_u32(sQ + kt * kSaHeads * 128));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc_mma_f16(t_s, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) ? 1u : 0u);
      }
      tc_commit(mma_bar);
    }
    __syncwarp();
    const bool ok = mbar_wait(mma_bar, mma_phase, DSV4_DEVERR_TIMEOUT_MMA);
    mma_phase ^= 1;
    failed = __syncthreads_or(!ok) != 0;
    tc_fence_after();
    return !failed;
  };

  // per-head max (mode 0) or sum (mode 1) over the 128 rows of v[64] held by
  // the threads of warps 0-3 (thread = row); result for head h at s_red[h]
  auto head_reduce = [&](float* v, int mode) {
    if (tmem_warp) {
#pragma unroll 8
      for (int h = 0; h < kSaHeads; ++h) {
        float x = v[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float y = __shfl_xor_sync(0xffffffffu, x, o);
          x = mode == 0 ? fmaxf(x, y) : x + y;
        }
        if (lane == 0) s_red[q4 * kSaHeads + h] = x;  // [4 quarters][64], 1 KB
      }
    }
    __syncthreads();
    if (tid < kSaHeads) {
      float x = s_red[tid];
      for (int w = 1; w < 4; ++w) x = mode == 0 ? fmaxf(x, s_red[w * kSaHeads + tid]) : x + s_red[w * kSaHeads + tid];
      s_red[4 * kSaHeads + tid] = x;
    }
    __syncthreads();
  };

  float z[kSaHeads];
  // ---------------------------------------------------------------- pass 1
  for (int c = c_begin; c < c_end && !failed; ++c) {
    gather(c);
    if (!scores()) break;
    bool valid = false;
    if (tmem_warp) {
      tmem_ld64(t_s + lane_base, z);
      valid = s_idx[q4 * 32 + lane] >= 0;
#pragma unroll
      for (int h = 0; h < kSaHeads; ++h) z[h] = valid ? z[h] * a.scale : -INFINITY;
    }
    any_valid |= __syncthreads_or(valid);
    head_reduce(z, 0);
    // every thread needs the new running max of every head: read s_red[256 + h]
    if (tmem_warp) {
#pragma unroll
      for (int h = 0; h < kSaHeads; ++h) {
        const float mn = s_red[4 * kSaHeads + h];
        z[h] = (valid && mn > -INFINITY) ? __expf(z[h] - mn) : 0.f;
      }
    }
    // the chunk's max must be read by all before the sums overwrite s_red
    float cmax = tid < kSaHeads ? s_red[4 * kSaHeads + tid] : 0.f;
    __syncthreads();
    head_reduce(z, 1);
    if (tid < kSaHeads) {
      const float csum = s_red[4 * kSaHeads + tid];
      if (cmax > -INFINITY) {
        const float mn = fmaxf(m_run, cmax);
        l_run = (m_run > -INFINITY ? l_run * __expf(m_run - mn) : 0.f) + csum * __expf(cmax - mn);
        m_run = mn;
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  // the per-head max and sum of this split: published for pass 2 (and the
  // sink folded in when this split is the token's only one)
  float* s_m = s_red + 5 * kSaHeads;  // [64] final max
  float* s_l = s_m + kSaHeads;        // [64] final 1 / denominator (or sum)
  if (tid < kSaHeads) {
    float m = m_run, l = l_run;
    if (a.splits == 1) {
      const float sk = a.sink[tid];
      const float mn = fmaxf(m, sk);
      l = (m > -INFINITY ? l * __expf(m - mn) : 0.f) + __expf(sk - mn);
      m = mn;
    }
    s_m[tid] = m;
    s_l[tid] = l > 0.f ? 1.0f / l : 0.f;
    if (a.splits > 1) {
      float* ml = a.part_ml + ((size_t)token * a.splits + split) * kSaHeads * 2;
      ml[2 * tid] = m_run;
      ml[2 * tid + 1] = l_run;
    }
  }
  __syncthreads();

  // ---------------------------------------------------------------- pass 2
  bool first = true;
  for (int c = c_begin; c < c_end && !failed; ++c) {
    gather(c);
    if (!scores()) break;
    if (tmem_warp) {
      tmem_ld64(t_s + lane_base, z);
      const int j = q4 * 32 + lane;
      const bool valid = s_idx[j] >= 0;
      // P[h][j] (bf16, K-major over j: 2 k tiles of [64 rows][128 B])
#pragma unroll 8
      for (int h = 0; h < kSaHeads; ++h) {
        const float p = valid ? __expf(z[h] * a.scale - s_m[h]) * s_l[h] : 0.f;
        *reinterpret_cast<__nv_bfloat16*>(sP + sw128_offset(kSaHeads, h, j)) = __float2bfloat16_rn(p);
      }
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      // O^T[d, h] += C^T[d, j] P[h, j]: A = C as MN-major (d chunks 16 KB apart), B = P K-major
      const uint32_t idesc = idesc_bf16_major(kSaHeads, 1, 0);
#pragma unroll 1
      for (int dt = 0; dt < kSaDim / 128; ++dt) {
#pragma unroll 1
        for (int kt = 0; kt < kSaChunk / 64; ++kt) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // rows j = 64 kt + 16 kk .. +15 of C, d = 128 dt .. +127 (k tiles 2 dt, 2 dt + 1)
            const uint32_t a_addr = smem_u32(sC + (2 * dt) * kSaChunk * 128 + (64 * kt + 16 * kk) * 128);
            const uint64_t ad = sdesc_mn_sw128(a_addr, kSaChunk * 128);
            const uint64_t bd = sdesc_k_sw128(smem_u32(sP + kt * kSaHeads * 128)) + 2 * kk;
            tc_mma_f16(t_o + 64 * dt, ad, bd, idesc, (!first || kt || kk) ? 1u : 0u);
          }
        }
      }
      tc_commit(mma_bar);
    }
    __syncwarp();
    const bool ok = mbar_wait(mma_bar, mma_phase, DSV4_DEVERR_TIMEOUT_MMA);
    mma_phase ^= 1;
    failed = __syncthreads_or(!ok) != 0;
    tc_fence_after();
    first = false;
  }

  // ---------------------------------------------------------------- output
  // thread (quarter q4, lane) of warps 0-3 holds d = 128 dt + 32 q4 + lane
  if (tmem_warp && !failed) {
    const int tok_out = token;
#pragma unroll 1
    for (int dt = 0; dt < kSaDim / 128; ++dt) {
      float o[kSaHeads];
      if (!first) tmem_ld64(t_o + 64 * dt + lane_base, o);
      const int d = 128 * dt + 32 * q4 + lane;
      if (a.splits == 1) {
        __nv_bfloat16* dst = a.out + (size_t)tok_out * kSaHeads * kSaDim + d;
#pragma unroll 8
        for (int h = 0; h < kSaHeads; ++h)
          dst[(size_t)h * kSaDim] = __float2bfloat16_rn((first || !any_valid) ? 0.f : o[h]);
      } else {
        // unnormalised partial: O * sum (so the combine can rescale by max)
        float* dst = a.part_o + ((size_t)tok_out * a.splits + split) * kSaHeads * kSaDim + d;
#pragma unroll 8
        for (int h = 0; h < kSaHeads; ++h) {
          const float l = s_l[h] > 0.f ? 1.0f / s_l[h] : 0.f;
          dst[(size_t)h * kSaDim] = first ? 0.f : o[h] * l;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kSaTmemCols);
  }
}

// Merge the splits of each (token, head): M = max(max_s m_s, sink), denominator
// = sum_s l_s exp(m_s - M) + exp(sink - M), out = sum_s O_s exp(m_s - M) / den.
__global__ void __launch_bounds__(kSaDim / 4) sparse_attn_combine_kernel(const SaArgs a) {
  const int token = blockIdx.x / kSaHeads, h = blockIdx.x % kSaHeads;
  const float* ml = a.part_ml + (size_t)token * a.splits * kSaHeads * 2;
  float M = a.sink[h];
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, ml[(s * kSaHeads + h) * 2]);
  float den = __expf(a.sink[h] - M);
  for (int s = 0; s < a.splits; ++s) {
    const float m = ml[(s * kSaHeads + h) * 2];
    if (m > -INFINITY) den += ml[(s * kSaHeads + h) * 2 + 1] * __expf(m - M);
  }
  bool any = false;
  for (int s = 0; s < a.splits; ++s) any |= ml[(s * kSaHeads + h) * 2] > -INFINITY;
  for (int d = threadIdx.x; d < kSaDim; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float m = ml[(s * kSaHeads + h) * 2];
      if (m > -INFINITY)
        acc += a.part_o[(((size_t)token * a.splits + s) * kSaHeads + h) * kSaDim + d] * __expf(m - M);
    }
    a.out[((size_t)token * kSaHeads + h) * kSaDim + d] = __float2bfloat16_rn(any ? acc / den : 0.f);
  }
}

long long sparse_attn_workspace(int tokens, int K, int num_sms, int* splits_out, int* cps_out) {
  const int n_chunks = (K + kSaChunk - 1) / kSaChunk;
  // enough CTAs to cover the SMs twice; one split when the tokens already do
  int splits = tokens >= 2 * num_sms ? 1 : (2 * num_sms + tokens - 1) / tokens;
  if (splits > n_chunks) splits = n_chunks;
  if (splits < 1) splits = 1;
  const int cps = (n_chunks + splits - 1) / splits;
  splits = (n_chunks + cps - 1) / cps;
  if (splits_out) *splits_out = splits;
  if (cps_out) *cps_out = cps;
  if (splits == 1) return 0;
  return (long long)tokens * splits * kSaHeads * (kSaDim + 2) * 4;
}

int launch_sparse_attn(const void* q, const void* kv, const float* sink, const int* idx, int B, int S,
                       int N, int K, float scale, void* out, void* ws, long long ws_bytes, int num_sms,
                       cudaStream_t st) {
  const int tokens = B * S;
  int splits, cps;
  const long long need = sparse_attn_workspace(tokens, K, num_sms, &splits, &cps);
  if (need > ws_bytes || (need > 0 && !ws)) return DSV4_ERR_WORKSPACE;
  SaArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kv = static_cast<const __nv_bfloat16*>(kv);
  a.sink = sink;
  a.idx = idx;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.part_o = need ? static_cast<float*>(ws) : nullptr;
  a.part_ml = need ? static_cast<float*>(ws) + (size_t)tokens * splits * kSaHeads * kSaDim : nullptr;
  a.S = S;
  a.N = N;
  a.K = K;
  a.splits = splits;
  a.chunks_per_split = cps;
  a.scale = scale;
  if (ensure_smem_attr(reinterpret_cast<const void*>(sparse_attn_kernel), (int)kSaSmem)) return DSV4_ERR_CUDA;
  launch_k(sparse_attn_kernel, tokens * splits, kSaThreads, kSaSmem, st, a);
  if (splits > 1) launch_k(sparse_attn_combine_kernel, tokens * kSaHeads, kSaDim / 4, 0, st, a);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

}  // namespace dsv4
