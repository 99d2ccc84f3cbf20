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
// list (a split), in one pass with an online softmax: per chunk the rows are
// gathered (cp.async, 16 B; the next chunk's rows are prefetched to L2 while
// the tensor core works), the scores land in TMEM, every thread reads its row's
// scores for 32 heads, P = exp(z - m) goes to shared memory in bf16 and the
// output product accumulates O^T in TMEM.  The running max m of a head is
// raised only when a score exceeds it by more than kSaRescaleLog (then O^T and
// the partial sums are rescaled); the per-head max is a recursive-halving
// reduction over the warp's lanes plus a 4-way combine in shared memory.  A
// token with one split writes out directly with the sink folded into the
// denominator; several splits write fp32 partials (max, sum, O relative to the
// max) that sparse_attn_combine_kernel merges with the sink term.
//
// Warp roles (256 threads): all warps gather rows; warp 0, lane 0 issues the
// MMAs; warp w reads TMEM lane quarter w % 4 (lane = gathered row in the score
// product, = d in the output product) for heads 32 (w / 4) .. +31.
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
constexpr float kSaRescaleLog = 8.0f;  // headroom of the running max (natural log)

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

// Load 32 consecutive fp32 columns of this thread's TMEM lane and wait.
__device__ __forceinline__ void tmem_ld32_wait(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32_issue(taddr, r);
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]) : : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 32 consecutive fp32 columns of this thread's TMEM lane (tcgen05.wait::st
// before the tensor core reads them).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
               :: "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31])) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Reduce 32 values per lane over the warp's 32 lanes (max, or sum when kSum) by
// recursive halving: at each step a lane keeps one half of its values, sends
// the other half to its partner and combines (31 shuffles in all).  Afterwards
// lane l holds the reduction of value l, which is returned.
template <bool kSum>
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? v[i] : v[i + o];
      const float keep = up ? v[i + o] : v[i];
      const float r = __shfl_xor_sync(0xffffffffu, send, o);
      v[i] = kSum ? keep + r : fmaxf(keep, r);
    }
  }
  return v[0];
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
  int* s_idx = reinterpret_cast<int*>(ctrl + 16);                 // [128] this chunk's kv rows (-1 invalid)
  float* s_red = reinterpret_cast<float*>(ctrl + 16 + 4 * kSaChunk);  // [4 quarters][64] partial reductions
  float* s_m = s_red + 4 * kSaHeads;                             // [64] running max per head
  float* s_f = s_m + kSaHeads;                                   // [64] rescale factor, then output factor
  static_assert(16 + 4 * kSaChunk + 6 * kSaHeads * 4 <= kSaCtrl, "control block too small");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q4 = warp & 3;           // TMEM lane quarter: rows 32 q4 .. +31 of a chunk (or of a d tile)
  const int h0 = (warp >> 2) * 32;   // warps 0-3 take heads 0-31, warps 4-7 heads 32-63
  const int row = q4 * 32 + lane;    // this thread's gathered row (scores) and d within a d tile (output)
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const int token = blockIdx.x / a.splits, split = blockIdx.x % a.splits;
  const int b = token / a.S;
  const int n_chunks = (a.K + kSaChunk - 1) / kSaChunk;
  const int c_begin = split * a.chunks_per_split;
  const int c_end = min(n_chunks, c_begin + a.chunks_per_split);
  const __nv_bfloat16* kvb = a.kv + (size_t)b * a.N * kSaDim;
  const int* idx = a.idx + (size_t)token * a.K;
  const __nv_bfloat16* qt = a.q + (size_t)token * kSaHeads * kSaDim;

  auto load_index = [&](int c) -> int {
    const int p = c * kSaChunk + tid;
    int r = p < a.K ? __ldg(idx + p) : -1;
    if (r >= a.N) {
      record_error(DSV4_DEVERR_BAD_INDEX);
      r = -1;
    }
    return r;
  };

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kSaTmemCols);
    tmem_relinquish();
  }
  if (tid < kSaHeads) s_m[tid] = -INFINITY;
  int next_row = (tid < kSaChunk && c_begin < c_end) ? load_index(c_begin) : -1;

  // Online softmax over the chunks: this thread keeps, for its row and its 32
  // heads, the running max (the same in every thread of the head half) and a
  // partial sum of the bf16 probabilities; O^T accumulates in TMEM relative to
  // the running max.  The max is raised (and O, the sums rescaled) only when a
  // score exceeds it by more than kSaRescaleLog, so probabilities stay below
  // e^kSaRescaleLog and most chunks need no reduction at all.
  float m_run[32], l_run[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
  }
  uint32_t mma_phase = 0;
  bool first = true, any_valid = false;
  // A wait that runs out fails the whole CTA at once (every thread leaves the
  // chunk loop at the same point, so no barrier is left waiting).
  bool failed = false;
  uint32_t tmem = 0;

  for (int c = c_begin; c < c_end; ++c) {
    if (!first) {
      // the previous chunk's output product is done with sC and sP
      const bool ok = mbar_wait(mma_bar, mma_phase, DSV4_DEVERR_TIMEOUT_MMA);
      mma_phase ^= 1;
      failed = __syncthreads_or(!ok) != 0;
      if (failed) break;
    }
    if (tid < kSaChunk) s_idx[tid] = next_row;
    __syncthreads();
    if (c == c_begin) {
      for (int u = tid; u < kSaHeads * kSaDim / 8; u += kSaThreads) {
        const int r = u / (kSaDim / 8), col = (u % (kSaDim / 8)) * 8;
        cp_async16(smem_u32(sQ + sw128_offset(kSaHeads, r, col)), qt + (size_t)r * kSaDim + col);
      }
    }
    for (int u = tid; u < kSaChunk * kSaDim / 8; u += kSaThreads) {
      const int r = u / (kSaDim / 8), col = (u % (kSaDim / 8)) * 8;
      const int kr = s_idx[r];
      const uint32_t dst = smem_u32(sC + sw128_offset(kSaChunk, r, col));
      if (kr >= 0)
        cp_async16(dst, kvb + (size_t)kr * kSaDim + col);
      else
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
    }
    // the next chunk's indices load while this one is gathered
    next_row = (tid < kSaChunk && c + 1 < c_end) ? load_index(c + 1) : -1;
    cp_async_wait_all();
    fence_proxy_async_shared();  // the generic-proxy writes, before the tensor core reads them
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem = *tmem_slot;
    const uint32_t t_s = tmem, t_o = tmem + 256;

    // S^T[j, h] = C[j, :] . Q[h, :]
    if (tid == 0) {
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
    // the next chunk's rows start towards L2 while the tensor core works
    if (tid < kSaChunk && next_row >= 0) {
      const char* src = reinterpret_cast<const char*>(kvb + (size_t)next_row * kSaDim);
#pragma unroll
      for (int l = 0; l < kSaDim * 2 / 128; ++l)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(src + l * 128)));
    }
    __syncwarp();
    {
      const bool ok = mbar_wait(mma_bar, mma_phase, DSV4_DEVERR_TIMEOUT_MMA);
      mma_phase ^= 1;
      failed = __syncthreads_or(!ok) != 0;
    }
    tc_fence_after();
    if (failed) break;

    float z[32];
    tmem_ld32_wait(t_s + lane_base + h0, z);
    const bool valid = s_idx[row] >= 0;
    any_valid |= valid;
    bool raise = false;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      z[i] = valid ? z[i] * a.scale : -INFINITY;
      raise |= z[i] > m_run[i] + kSaRescaleLog;
    }
    if (__syncthreads_or(raise)) {
      float t[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) t[i] = z[i];
      s_red[q4 * kSaHeads + h0 + lane] = warp_reduce_scatter32<false>(t, lane);
      __syncthreads();
      if (tid < kSaHeads) {
        float cm = s_red[tid];
#pragma unroll
        for (int w = 1; w < 4; ++w) cm = fmaxf(cm, s_red[w * kSaHeads + tid]);
        const float mo = s_m[tid], mn = fmaxf(mo, cm);
        s_f[tid] = mo == -INFINITY ? 0.f : __expf(mo - mn);
        s_m[tid] = mn;
      }
      __syncthreads();
      float alpha[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        alpha[i] = s_f[h0 + i];
        m_run[i] = s_m[h0 + i];
        l_run[i] *= alpha[i];
      }
      if (!first) {
        // O^T columns of this thread's heads, in each of the 4 d tiles
#pragma unroll 1
        for (int dt = 0; dt < kSaDim / 128; ++dt) {
          float o[32];
          tmem_ld32_wait(t_o + 64 * dt + h0 + lane_base, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha[i];
          tmem_st32(t_o + 64 * dt + h0 + lane_base, o);
        }
        tmem_wait_st();
      }
    }
    // P[h][j] in bf16 (K-major over j: 2 k tiles of [64 rows][128 B])
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const __nv_bfloat16 pb = __float2bfloat16_rn(valid ? __expf(z[i] - m_run[i]) : 0.f);
      l_run[i] += __bfloat162float(pb);
      *reinterpret_cast<__nv_bfloat16*>(sP + sw128_offset(kSaHeads, h0 + i, row)) = pb;
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
    first = false;
  }
  if (!first && !failed) {
    const bool ok = mbar_wait(mma_bar, mma_phase, DSV4_DEVERR_TIMEOUT_MMA);
    mma_phase ^= 1;
    failed = __syncthreads_or(!ok) != 0;
  }
  tc_fence_after();

  // ---------------------------------------------------------------- output
  // per-head sums over the 128 rows, then the factor each head's O^T column
  // is scaled by: the sink folded in when this split is the token's only one
  {
    float t[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) t[i] = l_run[i];
    s_red[q4 * kSaHeads + h0 + lane] = warp_reduce_scatter32<true>(t, lane);
  }
  const bool any = __syncthreads_or(any_valid) != 0;
  if (tid < kSaHeads) {
    const float l = s_red[tid] + s_red[kSaHeads + tid] + s_red[2 * kSaHeads + tid] + s_red[3 * kSaHeads + tid];
    const float m = s_m[tid];
    if (a.splits == 1) {
      const float sk = a.sink[tid];
      const float M = fmaxf(m, sk);
      const float den = (m > -INFINITY ? l * __expf(m - M) : 0.f) + __expf(sk - M);
      s_f[tid] = (any && m > -INFINITY) ? __expf(m - M) / den : 0.f;
    } else {
      float* ml = a.part_ml + ((size_t)token * a.splits + split) * kSaHeads * 2;
      ml[2 * tid] = m;
      ml[2 * tid + 1] = l;
    }
  }
  __syncthreads();
  if (!failed) {
#pragma unroll 1
    for (int dt = 0; dt < kSaDim / 128; ++dt) {
      float o[32];
      if (!first) {
        tmem_ld32_wait((*tmem_slot + 256) + 64 * dt + h0 + lane_base, o);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
      }
      const int d = 128 * dt + row;
      if (a.splits == 1) {
        __nv_bfloat16* dst = a.out + ((size_t)token * kSaHeads + h0) * kSaDim + d;
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[(size_t)i * kSaDim] = __float2bfloat16_rn(o[i] * s_f[h0 + i]);
      } else {
        // O relative to this split's running max (the combine rescales it)
        float* dst = a.part_o + (((size_t)token * a.splits + split) * kSaHeads + h0) * kSaDim + d;
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[(size_t)i * kSaDim] = o[i];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(*tmem_slot, kSaTmemCols);
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
