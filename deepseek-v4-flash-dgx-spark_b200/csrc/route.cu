// Routing plan, permutation with fused activation quantization, and the
// weighted combine back to token order.
//
// Replaces, in spark_runtime/lazy_official_runtime.py:980-1002 (LazyMoE.forward):
//   counts = torch.bincount(indices).tolist()        (:985, a host sync)
//   idx, top = torch.where(indices == i); x[idx]      (:997-998, one select per expert)
//   y[idx] += expert(...); y += shared(x); y.type_as(x) (:984,998-1002)
// with device-only kernels: no host round trip between routing and the GEMMs.
#include "kernels.cuh"

namespace dsv4 {

// ---------------------------------------------------------------------------
// Route plan: a stable counting sort of the T*k (token, rank) routes into
// per-expert segments, in three launches that use the whole GPU:
//   route_count    per chunk of `chunk` tokens, a histogram over experts
//   route_scan     per expert, exclusive scan of its chunk counts (token
//                  order); the last CTA to finish lays out the segments
//   route_scatter  per chunk, each route's rank among earlier routes of the
//                  chunk with the same expert gives its slot; the chunk's token
//                  rows are quantized once and written to all their slots
// Inside a segment rows follow token order, which is the order torch.where
// gives.  Segment sizes are padded to 32 rows so every GEMM tile starts on a
// 32-row boundary of the activation scale atoms.  The shared expert is
// segment E and holds the first `shared_rows` tokens.
//
// ctrl[0] counts finished route_scan CTAs, ctrl[1] flags an invalid index,
// ctrl[2] flags a failed plan; the caller zeroes ctrl before route_count.
// ---------------------------------------------------------------------------
constexpr int kSegAlign = 32;
constexpr int kMaxK = 8;
constexpr int kMaxChunk = 32;  // tokens per chunk (chunk * k <= 256 threads)
constexpr int kScanThreads = 256;
constexpr int kMaxSegments = 513;

__global__ void __launch_bounds__(256) route_count_kernel(const int64_t* __restrict__ indices,
                                                          int T, int k, int E, int allow_skip,
                                                          int chunk, int nchunks,
                                                          int* __restrict__ chunk_cnt,
                                                          int* __restrict__ ctrl) {
  __shared__ int hist[kMaxSegments];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int c = blockIdx.x;
  const int r1 = min(T, (c + 1) * chunk) * k;
  for (int i = c * chunk * k + threadIdx.x; i < r1; i += blockDim.x) {
    const int64_t v = indices[i];
    if (v >= 0 && v < E) atomicAdd(&hist[v], 1);
    else if (!(allow_skip && v == -1)) atomicOr(&ctrl[1], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_cnt[(size_t)e * nchunks + c] = hist[e];
}

// Segment layout of one CTA from the per-segment counts s_cnt[0..NS) (shared
// memory): padded segment starts, tile bases and valid-row bases by a
// block-wide scan (each thread sums a contiguous run of segments, warps scan
// the thread sums with shuffles, warp 0 scans the warp totals), then the tile
// list, the padding rows and the published counts.  A thread writes the tiles
// of its own run (it holds the run's valid-row base in a register, so no
// per-segment array beyond s_start and s_tbase is needed); a warp writes a
// segment's padding rows.  A failed plan (an invalid index seen earlier, or more
// rows / tiles than the workspace holds) records a device error, sets ctrl[2]
// and emits no tiles.
__device__ void plan_layout(int* s_cnt, int* s_start, int* s_tbase, int NS, int block_n,
                            int max_rows, int max_tiles, int bad, int* __restrict__ counts,
                            int* __restrict__ seg_start, int4* __restrict__ tiles,
                            int* __restrict__ n_tiles, int* __restrict__ slot_token,
                            float* __restrict__ slot_weight, int* __restrict__ ctrl,
                            int* __restrict__ zero_ptr, int n_zero) {
  __shared__ int s_fail;
  __shared__ int s_wsum[3][32];  // per warp: padded rows, tiles, valid rows (then their exclusive scan)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int nwarps = (nthr + 31) >> 5;
  __syncthreads();
  const int per = (NS + nthr - 1) / nthr;
  const int s_lo = min(tid * per, NS), s_hi = min(s_lo + per, NS);
  int r_own = 0, t_own = 0, v_own = 0;
  for (int s = s_lo; s < s_hi; ++s) {
    const int c = s_cnt[s];
    r_own += (c + kSegAlign - 1) / kSegAlign * kSegAlign;
    t_own += (c + block_n - 1) / block_n;
    v_own += c;
  }
  int r_inc = r_own, t_inc = t_own, v_inc = v_own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, r_inc, o);
    const int b = __shfl_up_sync(0xffffffffu, t_inc, o);
    const int d = __shfl_up_sync(0xffffffffu, v_inc, o);
    if (lane >= o) {
      r_inc += a;
      t_inc += b;
      v_inc += d;
    }
  }
  if (lane == 31) {
    s_wsum[0][warp] = r_inc;
    s_wsum[1][warp] = t_inc;
    s_wsum[2][warp] = v_inc;
  }
  __syncthreads();
  if (warp == 0) {
    const int r0 = lane < nwarps ? s_wsum[0][lane] : 0;
    const int t0 = lane < nwarps ? s_wsum[1][lane] : 0;
    const int v0 = lane < nwarps ? s_wsum[2][lane] : 0;
    int r = r0, t = t0, v = v0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, r, o);
      const int b = __shfl_up_sync(0xffffffffu, t, o);
      const int d = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) {
        r += a;
        t += b;
        v += d;
      }
    }
    if (lane < nwarps) {
      s_wsum[0][lane] = r - r0;
      s_wsum[1][lane] = t - t0;
      s_wsum[2][lane] = v - v0;
    }
    if (lane == 31) {
      s_start[NS] = r;
      s_tbase[NS] = t;
      s_fail = bad || r > max_rows || t > max_tiles;
      if (s_fail) record_error(bad ? DSV4_DEVERR_BAD_INDEX : DSV4_DEVERR_PLAN_OVERFLOW);
      ctrl[2] = s_fail;
    }
  }
  __syncthreads();
  // exclusive bases of this thread's first segment
  int r_run = s_wsum[0][warp] + r_inc - r_own;
  int t_run = s_wsum[1][warp] + t_inc - t_own;
  const int v_base = s_wsum[2][warp] + v_inc - v_own;
  for (int s = s_lo; s < s_hi; ++s) {
    const int c = s_cnt[s];
    s_start[s] = r_run;
    s_tbase[s] = t_run;
    r_run += (c + kSegAlign - 1) / kSegAlign * kSegAlign;
    t_run += (c + block_n - 1) / block_n;
  }
  __syncthreads();
  if (s_fail) {
    if (tid == 0) *n_tiles = 0;
    return;
  }
  for (int s = tid; s <= NS; s += nthr) {
    seg_start[s] = s_start[s];
    if (s < NS) counts[s] = s_cnt[s];
  }
  // split-K item counters of the GEMMs start at zero on every call
  for (int i = tid; i < n_zero; i += nthr) zero_ptr[i] = 0;
  // tile = {segment, first plan row, valid rows, compact index of the first row};
  // the compact index counts the valid rows of earlier segments
  int vb = v_base;
  for (int s = s_lo; s < s_hi; ++s) {
    const int c = s_cnt[s], base = s_start[s], tb = s_tbase[s], nt = s_tbase[s + 1] - tb;
    for (int m = 0; m < nt; ++m)
      tiles[tb + m] = make_int4(s, base + m * block_n, min(block_n, c - m * block_n), vb + m * block_n);
    vb += c;
  }
  // padding rows: one warp per segment, consecutive lanes on consecutive rows
  for (int s = warp; s < NS; s += nwarps)
    for (int r = s_start[s] + s_cnt[s] + lane; r < s_start[s + 1]; r += 32) {
      slot_token[r] = -1;
      slot_weight[r] = 0.f;
    }
  if (tid == 0) *n_tiles = s_tbase[NS];
}

// Small batches: count, per-chunk scan and layout in one CTA, every count in
// shared memory ([nchunks][E], at most kSmallPlanInts).  Produces the same
// plan and chunk offsets as route_count + route_scan.
constexpr int kSmallPlanInts = 10240;  // with the layout arrays, under 48 KB of static smem

__global__ void __launch_bounds__(1024) route_plan_small_kernel(
    const int64_t* __restrict__ indices, int T, int k, int E, int allow_skip, int shared_rows,
    int chunk, int nchunks, int block_n, int max_rows, int max_tiles,
    int* __restrict__ chunk_base, int* __restrict__ counts, int* __restrict__ seg_start,
    int4* __restrict__ tiles, int* __restrict__ n_tiles, int* __restrict__ slot_token,
    float* __restrict__ slot_weight, int* __restrict__ ctrl, int* __restrict__ zero_ptr, int n_zero) {
  __shared__ int cnt[kSmallPlanInts];
  __shared__ int s_cnt[kMaxSegments], s_start[kMaxSegments + 1], s_tbase[kMaxSegments + 1];
  __shared__ int s_bad;
  const int tid = threadIdx.x;
  for (int i = tid; i < nchunks * E; i += blockDim.x) cnt[i] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  for (int i = tid; i < T * k; i += blockDim.x) {
    const int64_t v = indices[i];
    if (v >= 0 && v < E) atomicAdd(&cnt[(i / k / chunk) * E + (int)v], 1);
    else if (!(allow_skip && v == -1)) s_bad = 1;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    int run = 0;
    for (int c = 0; c < nchunks; ++c) {
      chunk_base[(size_t)e * nchunks + c] = run;
      run += cnt[c * E + e];
    }
    s_cnt[e] = run;
  }
  if (tid == 0) s_cnt[E] = shared_rows;
  plan_layout(s_cnt, s_start, s_tbase, E + 1, block_n, max_rows, max_tiles, s_bad, counts,
              seg_start, tiles, n_tiles, slot_token, slot_weight, ctrl, zero_ptr, n_zero);
}

__global__ void __launch_bounds__(kScanThreads) route_scan_kernel(
    const int* __restrict__ chunk_cnt, int nchunks, int E, int shared_rows, int block_n,
    int max_rows, int max_tiles, int* __restrict__ chunk_base, int* __restrict__ counts,
    int* __restrict__ seg_start, int4* __restrict__ tiles, int* __restrict__ n_tiles,
    int* __restrict__ slot_token, float* __restrict__ slot_weight, int* __restrict__ ctrl,
    int* __restrict__ zero_ptr, int n_zero) {
  __shared__ int s_cnt[kMaxSegments], s_start[kMaxSegments + 1], s_tbase[kMaxSegments + 1];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // one warp per expert: exclusive scan of its chunk counts in chunk (token) order
  const int e = blockIdx.x * (kScanThreads / 32) + warp;
  if (e < E) {
    const int* src = chunk_cnt + (size_t)e * nchunks;
    int* dst = chunk_base + (size_t)e * nchunks;
    int run = 0;
    for (int c0 = 0; c0 < nchunks; c0 += 32) {
      const int c = c0 + lane;
      const int v = c < nchunks ? src[c] : 0;
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += a;
      }
      if (c < nchunks) dst[c] = run + inc - v;
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) counts[e] = run;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&ctrl[0], 1) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // the last CTA: padded segment offsets, tiles, padding rows
  for (int s = tid; s < E; s += kScanThreads) s_cnt[s] = __ldcg(counts + s);
  if (tid == 0) s_cnt[E] = shared_rows;
  plan_layout(s_cnt, s_start, s_tbase, E + 1, block_n, max_rows, max_tiles, __ldcg(ctrl + 1), counts,
              seg_start, tiles, n_tiles, slot_token, slot_weight, ctrl, zero_ptr, n_zero);
}

// Per-128 act_quant of one token row by one warp, the codes and scales written
// to every slot in `slots` (smem, -1 = none).  The row is walked in quads of
// four 128-wide k tiles: lane l owns elements 16l..16l+15 of a quad (k tile
// 4q + l/8), so the 8 lanes of a k tile reduce its amax in 3 shuffles, codes
// leave as one 16-byte store per lane and slot, and the quad's four scales as
// one 32-bit word.  Scales go to the sliding k-packed atoms: atom (g, q) holds
// rows 32g .. 32g+127 for k tiles 4q .. 4q+3, row r / tile kt at byte
// (r%32)*16 + ((r/32)-g)*4 + kt%4, so one quad of one row is 4 consecutive
// bytes in each of the (up to) four atoms that contain the row.
// act_quant of one quad (4 k tiles) of a row held as 16 bf16 per lane (lane l:
// elements 16l..16l+15): codes of the lane's 16 elements and, in every lane,
// the biased ue8m0 scale byte of its k tile (l / 8).
__device__ __forceinline__ void quad_quant(const uint4 raw[2], int lane, uint4* code, uint32_t* sc) {
  float v[16];
  const __nv_bfloat16* b0 = reinterpret_cast<const __nv_bfloat16*>(&raw[0]);
  const __nv_bfloat16* b1 = reinterpret_cast<const __nv_bfloat16*>(&raw[1]);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = __bfloat162float(b0[i]);
    v[8 + i] = __bfloat162float(b1[i]);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const int e = act_scale_exp(amax);
  const float inv = exp2i(-e);
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = e4m3x4(v[4 * j] * inv, v[4 * j + 1] * inv, v[4 * j + 2] * inv, v[4 * j + 3] * inv);
  *code = make_uint4(w[0], w[1], w[2], w[3]);
  *sc = static_cast<uint32_t>(e + 127);
}

constexpr int kQuadsInFlight = 2;
constexpr int kQuantGroup = 8;  // k tiles of loads in flight in quant_row; the least a scatter CTA takes

__device__ __forceinline__ void scatter_row(const __nv_bfloat16* __restrict__ xrow,
                                            const uint8_t* __restrict__ qrow, int q0, int q1,
                                            int KT, int H, const int* slots, int nslots, int lane,
                                            uint8_t* __restrict__ xq, uint8_t* __restrict__ sfb) {
  for (int qa = q0; qa < q1; qa += kQuadsInFlight) {
    uint4 raw[kQuadsInFlight][2];
    uint4 code[kQuadsInFlight];
    uint32_t sc[kQuadsInFlight];
#pragma unroll
    for (int g = 0; g < kQuadsInFlight; ++g) {
      raw[g][0] = raw[g][1] = code[g] = make_uint4(0, 0, 0, 0);
      sc[g] = 0;
      if (qa + g < q1) {
        const size_t e0 = (size_t)(qa + g) * 512 + lane * 16;
        if (xrow) {
          raw[g][0] = *reinterpret_cast<const uint4*>(xrow + e0);
          raw[g][1] = *reinterpret_cast<const uint4*>(xrow + e0 + 8);
        } else {
          code[g] = *reinterpret_cast<const uint4*>(qrow + e0);
          sc[g] = qrow[H + (qa + g) * 4 + (lane >> 3)];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kQuadsInFlight; ++g) {
      if (qa + g >= q1) break;
      if (xrow) quad_quant(raw[g], lane, &code[g], &sc[g]);
      // the quad's four scales, k tile j held by lane 8j
      const uint32_t s4 = __shfl_sync(0xffffffffu, sc[g], 0) | (__shfl_sync(0xffffffffu, sc[g], 8) << 8) |
                          (__shfl_sync(0xffffffffu, sc[g], 16) << 16) |
                          (__shfl_sync(0xffffffffu, sc[g], 24) << 24);
      for (int d = 0; d < nslots; ++d) {
        const int slot = slots[d];
        if (slot < 0) continue;
        *reinterpret_cast<uint4*>(xq + (size_t)slot * H + (size_t)(qa + g) * 512 + lane * 16) = code[g];
        if (lane < 4) {
          const int ga = (slot >> 5) - lane;
          if (ga >= 0)
            *reinterpret_cast<uint32_t*>(sfb + ((size_t)ga * (KT >> 2) + (qa + g)) * 512 + (slot & 31) * 16 +
                                         lane * 4) = s4;
        }
      }
    }
  }
}

// grid (nchunks, ksplit): CTA (c, y) places chunk c's routes and writes quads
// [y*KQ/ksplit, (y+1)*KQ/ksplit) (KQ = H/512) of its token rows.  Tokens t < n_x_rows are
// quantized from x (bf16); later tokens are fp8 rows of `rows_in` (codes, then
// H/128 scale bytes) copied as they are.
__global__ void __launch_bounds__(256) route_scatter_kernel(
    const __nv_bfloat16* __restrict__ x, int n_x_rows, const uint8_t* __restrict__ rows_in,
    long long rows_in_stride, const int64_t* __restrict__ indices, const float* __restrict__ weights,
    int T, int k, int E, int H, int shared_rows, int chunk, int nchunks,
    const int* __restrict__ seg_start, const int* __restrict__ chunk_base, const int* __restrict__ ctrl,
    int* __restrict__ route_slot, int* __restrict__ slot_token, float* __restrict__ slot_weight,
    uint8_t* __restrict__ xq, uint8_t* __restrict__ sfb) {
  __shared__ int s_e[kMaxChunk * kMaxK];
  __shared__ int s_slot[kMaxChunk][kMaxK + 1];
  if (__ldcg(ctrl + 2)) return;
  const int c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = c * chunk;
  const int nt = min(chunk, T - t0);
  const int nr = nt * k, i0 = t0 * k;
  const bool owner = blockIdx.y == 0;
  if (tid < nr) {
    const int64_t v = indices[i0 + tid];
    s_e[tid] = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
  }
  __syncthreads();
  if (tid < nr) {
    const int e = s_e[tid];
    int slot = -1;
    if (e >= 0) {
      int rank = 0;
      for (int j = 0; j < tid; ++j) rank += s_e[j] == e;
      slot = seg_start[e] + chunk_base[(size_t)e * nchunks + c] + rank;
      if (owner) {
        slot_token[slot] = t0 + tid / k;
        slot_weight[slot] = weights[i0 + tid];
      }
    }
    if (owner) route_slot[i0 + tid] = slot;
    s_slot[tid / k][tid % k] = slot;
  }
  if (tid < nt) {
    const int t = t0 + tid;
    int slot = -1;
    if (t < shared_rows) {
      slot = seg_start[E] + t;
      if (owner) {
        slot_token[slot] = t;
        slot_weight[slot] = 1.0f;
      }
    }
    s_slot[tid][k] = slot;
  }
  __syncthreads();
  const int KT = H / 128, KQ = KT / 4;
  const int per = (KQ + gridDim.y - 1) / gridDim.y;
  const int q0 = blockIdx.y * per, q1 = min(KQ, q0 + per);
  for (int lt = warp; lt < nt; lt += blockDim.x / 32) {
    const int t = t0 + lt;
    const __nv_bfloat16* xrow = t < n_x_rows ? x + (size_t)t * H : nullptr;
    const uint8_t* qrow = t < n_x_rows ? nullptr : rows_in + (size_t)(t - n_x_rows) * rows_in_stride;
    scatter_row(xrow, qrow, q0, q1, KT, H, s_slot[lt], k + 1, lane, xq, sfb);
  }
}

// ---------------------------------------------------------------------------
// Decode batches of at most kFusedMaxTokens tokens: the gate's top-k (from the
// split-K partial logits), the route plan and the scatter + act_quant in one
// CTA, with the same results as gate_topk_kernel + route_plan_small_kernel +
// route_scatter_kernel (one chunk): the three launches and their round trips
// through global memory become one.
// ---------------------------------------------------------------------------
constexpr int kFusedMaxTokens = 8;
constexpr int kFusedMaxExperts = 512;

__global__ void __launch_bounds__(512) route_small_fused_kernel(
    const float* __restrict__ partials, int nsplit, float* __restrict__ logits_out, const float* __restrict__ bias,
    int T, int E, int k, float route_scale, float* __restrict__ weights, int64_t* __restrict__ indices,
    const __nv_bfloat16* __restrict__ x, int H, int shared_rows, int block_n, int max_rows, int max_tiles,
    int* __restrict__ chunk_base, int* __restrict__ counts, int* __restrict__ seg_start, int4* __restrict__ tiles,
    int* __restrict__ n_tiles, int* __restrict__ slot_token, float* __restrict__ slot_weight,
    int* __restrict__ ctrl, int* __restrict__ zero_ptr, int n_zero, int* __restrict__ route_slot,
    uint8_t* __restrict__ xq, uint8_t* __restrict__ sfb) {
  __shared__ float s_score[kFusedMaxTokens * kFusedMaxExperts], s_sel[kFusedMaxTokens * kFusedMaxExperts];
  __shared__ int cnt[kFusedMaxExperts];
  __shared__ int s_cnt[kMaxSegments], s_start[kMaxSegments + 1], s_tbase[kMaxSegments + 1];
  __shared__ int s_e[kFusedMaxTokens * kMaxK];
  __shared__ float s_w[kFusedMaxTokens * kMaxK];
  __shared__ int s_slot[kFusedMaxTokens][kMaxK + 1];
  __shared__ int s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_bad = 0;
  // scores of every (token, expert): a thread takes kFusedPairs pairs a
  // block apart and keeps all their slice loads in flight together; each
  // logit still adds its slices in slice order (as sum_slices does)
  constexpr int kFusedPairs = 4;
  const size_t slice = (size_t)T * E;
  const int n_pairs = T * E;
  for (int i0 = tid; i0 < n_pairs; i0 += blockDim.x * kFusedPairs) {
    float acc[kFusedPairs];
#pragma unroll
    for (int p = 0; p < kFusedPairs; ++p) {
      const int i = i0 + p * blockDim.x;
      acc[p] = i < n_pairs ? partials[i] : 0.f;
    }
    for (int sl0 = 1; sl0 < nsplit; sl0 += kSliceBatch) {
      float v[kFusedPairs][kSliceBatch];
#pragma unroll
      for (int p = 0; p < kFusedPairs; ++p) {
        const int i = i0 + p * blockDim.x;
#pragma unroll
        for (int j = 0; j < kSliceBatch; ++j)
          v[p][j] = (i < n_pairs && sl0 + j < nsplit) ? partials[i + (size_t)(sl0 + j) * slice] : 0.f;
      }
#pragma unroll
      for (int p = 0; p < kFusedPairs; ++p)
#pragma unroll
        for (int j = 0; j < kSliceBatch; ++j)
          if (sl0 + j < nsplit) acc[p] = __fadd_rn(acc[p], v[p][j]);
    }
#pragma unroll
    for (int p = 0; p < kFusedPairs; ++p) {
      const int i = i0 + p * blockDim.x;
      if (i >= n_pairs) continue;
      const int t = i / E, e = i % E;
      logits_out[i] = acc[p];
      const float sc = sigmoid_canonical(acc[p]);
      s_score[t * kFusedMaxExperts + e] = sc;
      s_sel[t * kFusedMaxExperts + e] = bias ? __fadd_rn(sc, bias[e]) : sc;
    }
  }
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  // top-k: warp t takes token t
  if (warp < T) {
    float w;
    int e;
    warp_topk(s_score + warp * kFusedMaxExperts, s_sel + warp * kFusedMaxExperts, E, k, route_scale, lane, &w, &e);
    if (lane < k) {
      weights[(size_t)warp * k + lane] = w;
      indices[(size_t)warp * k + lane] = e;
      s_e[warp * k + lane] = e;
      s_w[warp * k + lane] = w;
      if (e >= 0 && e < E)
        atomicAdd(&cnt[e], 1);
      else
        s_bad = 1;  // no finite selection value (NaN logits): the plan fails as the separate kernels' does
    }
  }
  __syncthreads();
  // plan (one chunk: every chunk offset is 0)
  for (int e = tid; e < E; e += blockDim.x) {
    chunk_base[e] = 0;
    s_cnt[e] = cnt[e];
  }
  if (tid == 0) s_cnt[E] = shared_rows;
  plan_layout(s_cnt, s_start, s_tbase, E + 1, block_n, max_rows, max_tiles, s_bad, counts, seg_start, tiles,
              n_tiles, slot_token, slot_weight, ctrl, zero_ptr, n_zero);
  __syncthreads();
  if (__ldcg(ctrl + 2)) return;
  // slots: route i of expert e goes to seg_start[e] + (its rank among e's routes, in route order)
  const int nr = T * k;
  if (tid < nr) {
    const int e = s_e[tid];
    int rank = 0;
    for (int j = 0; j < tid; ++j) rank += s_e[j] == e;
    const int slot = s_start[e] + rank;
    slot_token[slot] = tid / k;
    slot_weight[slot] = s_w[tid];
    route_slot[tid] = slot;
    s_slot[tid / k][tid % k] = slot;
  }
  if (tid < T) {
    int slot = -1;
    if (tid < shared_rows) {
      slot = s_start[E] + tid;
      slot_token[slot] = tid;
      slot_weight[slot] = 1.0f;
    }
    s_slot[tid][k] = slot;
  }
  __syncthreads();
  // quantize every token once and write its k + 1 rows: warps take (token,
  // pair of 512-wide quads) units
  const int KT = H / 128, KQ = KT / 4, units_per_token = (KQ + 1) / 2;
  for (int u = warp; u < T * units_per_token; u += blockDim.x / 32) {
    const int t = u / units_per_token, q0 = (u % units_per_token) * 2;
    scatter_row(x + (size_t)t * H, nullptr, q0, min(KQ, q0 + 2), KT, H, s_slot[t], k + 1, lane, xq, sfb);
  }
}

// ---------------------------------------------------------------------------
// Per-128 act_quant of k tiles [kt_begin, kt_end) of one row by one warp into a
// single destination row (the expert forward's identity plan, the linear layer
// and the plain act_quant entry point).
// ---------------------------------------------------------------------------

template <typename ScaleSink>
__device__ __forceinline__ void quant_row(const __nv_bfloat16* __restrict__ src, bool valid,
                                          uint8_t* __restrict__ dst, int kt_begin, int KT, int lane,
                                          ScaleSink sink) {
  for (int k0 = kt_begin; k0 < KT; k0 += kQuantGroup) {
    uint2 raw[kQuantGroup];
#pragma unroll
    for (int g = 0; g < kQuantGroup; ++g) {
      raw[g] = make_uint2(0, 0);
      if (valid && k0 + g < KT)
        raw[g] = *reinterpret_cast<const uint2*>(src + (size_t)(k0 + g) * 128 + lane * 4);
    }
#pragma unroll
    for (int g = 0; g < kQuantGroup; ++g) {
      if (k0 + g >= KT) break;
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw[g]);
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(b[i]);
      float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const int e = act_scale_exp(amax);
      const float inv = exp2i(-e);
      uint32_t packed = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        packed |= static_cast<uint32_t>(f32_to_e4m3(v[i] * inv)) << (8 * i);
      *reinterpret_cast<uint32_t*>(dst + (size_t)(k0 + g) * 128 + lane * 4) = packed;
      sink(k0 + g, static_cast<uint32_t>(e + 127));
    }
  }
}

// Activation scales go to the sliding k-packed atoms: atom (g, q) holds rows
// 32g .. 32g+127 for k tiles 4q .. 4q+3, row r / tile kt at byte
// (r%32)*16 + ((r/32)-g)*4 + kt%4.
__global__ void __launch_bounds__(256) permute_quant_kernel(
    const __nv_bfloat16* __restrict__ x, int H, const int* __restrict__ slot_token,
    const int* __restrict__ total_rows_ptr, uint8_t* __restrict__ xq, uint8_t* __restrict__ sfb) {
  const int lane = threadIdx.x & 31;
  const int total = *total_rows_ptr;
  const int KT = H / 128;
  // blockIdx.y takes one share of every row's k tiles (few rows: more warps)
  const int per = (KT + gridDim.y - 1) / gridDim.y;
  const int kb = blockIdx.y * per, ke = min(KT, kb + per);
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < total; row += nwarps) {
    const int t = slot_token[row];
    quant_row(x + (size_t)(t < 0 ? 0 : t) * H, t >= 0, xq + (size_t)row * H, kb, ke, lane,
              [&](int kt, uint32_t s) {
                if (lane < 4) {
                  const int m1 = lane;
                  const int g = (row >> 5) - m1;
                  if (g >= 0)
                    sfb[((size_t)g * (KT >> 2) + (kt >> 2)) * 512 + (row & 31) * 16 + m1 * 4 +
                        (kt & 3)] = static_cast<uint8_t>(s);
                }
              });
  }
}

__global__ void __launch_bounds__(256) act_quant_kernel(const __nv_bfloat16* __restrict__ x, int M,
                                                        int K, uint8_t* __restrict__ q,
                                                        uint8_t* __restrict__ s) {
  const int lane = threadIdx.x & 31;
  const int KT = K / 128;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < M; row += nwarps) {
    quant_row(x + (size_t)row * K, true, q + (size_t)row * K, 0, KT, lane, [&](int kt, uint32_t sc) {
      if (lane == 0) s[(size_t)row * KT + kt] = static_cast<uint8_t>(sc);
    });
  }
}

// ---------------------------------------------------------------------------
// FP4 activations (fp4_block_quant): one thread per 32-value block.
// fp4_act_quant_kernel: plain rows -> packed codes [M][K/2] + scale bytes
// [M][K/32] (the official fp4_act_quant's outputs).
// fp4_scatter_quant_kernel: the layer's routed rows -> packed codes
// [rows][H/2] and per-32 scale atoms for the tensor core: atom (g, w) holds
// rows 32g .. 32g+127 for the 128-wide k window w, row r / block b of the
// window at byte (r%32)*16 + ((r/32)-g)*4 + b (each row written to its four
// overlapping atoms, as the per-128 atoms are).  Each token's block is
// quantized once and written to the token's routed slots (route_slot [T][k],
// -1 = skipped); the shared expert's rows keep e4m3 and get none.  Padding
// rows are left unwritten: a row of A reaches only its own accumulator lane,
// and the epilogue never stores those lanes.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fp4_act_quant_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                                                            uint8_t* __restrict__ q, uint8_t* __restrict__ s) {
  const int nb = K / 32;
  const long long n = (long long)M * nb;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / nb), b = (int)(i % nb);
    float v[32];
    load_bf16x32(x + (size_t)row * K + 32 * b, v);
    uint4 packed;
    const int e = fp4_block_quant(v, packed);
    *reinterpret_cast<uint4*>(q + (size_t)row * (K / 2) + 16 * b) = packed;
    s[(size_t)row * nb + b] = static_cast<uint8_t>(e + 127);
  }
}

__global__ void __launch_bounds__(256) fp4_scatter_quant_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int H, int k, const int* __restrict__ route_slot, int max_rows,
    uint8_t* __restrict__ xq4, uint8_t* __restrict__ atoms) {
  const int nb = H / 32, KW = H / 128;
  const long long n = (long long)T * nb;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / nb), b = (int)(i % nb);
    float v[32];
    load_bf16x32(x + (size_t)t * H + 32 * b, v);
    uint4 packed;
    const uint8_t sbyte = static_cast<uint8_t>(fp4_block_quant(v, packed) + 127);
    const int w = b >> 2;
    for (int j = 0; j < k; ++j) {
      const int row = route_slot[(size_t)t * k + j];
      if (row < 0 || row >= max_rows) continue;
      *reinterpret_cast<uint4*>(xq4 + (size_t)row * (H / 2) + 16 * b) = packed;
      const int g = row >> 5;
#pragma unroll
      for (int m1 = 0; m1 < 4; ++m1)
        if (g - m1 >= 0) atoms[((size_t)(g - m1) * KW + w) * 512 + (row & 31) * 16 + m1 * 4 + (b & 3)] = sbyte;
    }
  }
}


// ---------------------------------------------------------------------------
// Combine: y[t] = bf16( sum over t's routes in ascending expert id of O[slot]
// (fp32) + O[shared slot] ).  Routing weights were applied inside the expert
// (before w2), so this is a plain ordered sum.  One CTA per token, one thread
// per 8-element chunk: a thread's k+1 row loads are all in flight at once.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) combine_kernel(const __nv_bfloat16* __restrict__ O, int H,
                                                      const int* __restrict__ route_slot,
                                                      const int64_t* __restrict__ indices, int T,
                                                      int k, const int* __restrict__ shared_base,
                                                      const __nv_bfloat16* __restrict__ Osh,
                                                      __nv_bfloat16* __restrict__ y) {
  const int t = blockIdx.x;
  if (t >= T) return;
  int se[kMaxK], ss[kMaxK];
#pragma unroll
  for (int r = 0; r < kMaxK; ++r) {
    se[r] = 0x7fffffff;
    ss[r] = -1;
    if (r < k) {
      se[r] = static_cast<int>(indices[(size_t)t * k + r]);
      ss[r] = route_slot[(size_t)t * k + r];
    }
  }
  // insertion sort by expert id (ids of one token are distinct)
#pragma unroll
  for (int a = 1; a < kMaxK; ++a) {
#pragma unroll
    for (int b = a; b > 0; --b) {
      if (se[b] < se[b - 1]) {
        const int te = se[b], ts = ss[b];
        se[b] = se[b - 1];
        ss[b] = ss[b - 1];
        se[b - 1] = te;
        ss[b - 1] = ts;
      }
    }
  }
  const int sh = shared_base ? (*shared_base + t) : -1;
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxK; ++r) {
      if (ss[r] < 0) continue;
      const uint4 raw = *reinterpret_cast<const uint4*>(O + (size_t)ss[r] * H + c * 8);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __bfloat162float(b[i]));
    }
    if (sh >= 0) {
      const uint4 raw = *reinterpret_cast<const uint4*>(Osh + (size_t)sh * H + c * 8);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __bfloat162float(b[i]));
    }
    uint4 out;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
    for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(acc[i]);
    *reinterpret_cast<uint4*>(y + (size_t)t * H + c * 8) = out;
  }
}

// ---------------------------------------------------------------------------
// Identity plan for one expert over T rows (official Expert.forward(x, weights)):
// row r = token r, weight w[r] (1 when w is NULL), ceil(T/block_n) tiles of
// segment `seg`.  Also publishes the padded row count and the expert->slot map.
// ---------------------------------------------------------------------------
__global__ void single_segment_plan_kernel(int T, int seg, int block_n, int rows_pad,
                                           const float* __restrict__ w, int* __restrict__ slot_token,
                                           float* __restrict__ slot_weight, int4* __restrict__ tiles,
                                           int* __restrict__ n_tiles, int* __restrict__ total_rows) {
  const int nt = (T + block_n - 1) / block_n;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows_pad; r += gridDim.x * blockDim.x) {
    slot_token[r] = r < T ? r : -1;
    slot_weight[r] = r < T ? (w ? w[r] : 1.0f) : 0.f;
    if (r < nt) tiles[r] = make_int4(seg, r * block_n, min(block_n, T - r * block_n), r * block_n);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *n_tiles = nt;
    *total_rows = rows_pad;
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
int route_chunk_tokens(int T) { return T <= 1024 ? 8 : kMaxChunk; }

int launch_route_plan(const int64_t* indices, int T, int k, int E, int allow_skip,
                      int shared_rows, int block_n, int max_rows, int max_tiles, int* chunk_cnt,
                      int* chunk_base, int* ctrl, int* counts, int* seg_start, int4* tiles,
                      int* n_tiles, int* slot_token, float* slot_weight, cudaStream_t st,
                      int* zero_ptr, int n_zero) {
  if (T <= 0 || k > kMaxK || E + 1 > kMaxSegments) return DSV4_ERR_ARG;
  const int chunk = route_chunk_tokens(T);
  const int nchunks = (T + chunk - 1) / chunk;
  if (nchunks * E <= kSmallPlanInts) {
    launch_k(route_plan_small_kernel, 1, 1024, 0, st,
             indices, T, k, E, allow_skip, shared_rows, chunk,
                                                nchunks, block_n, max_rows, max_tiles, chunk_base,
                                                counts, seg_start, tiles, n_tiles, slot_token,
                                                slot_weight, ctrl, zero_ptr, n_zero);
    return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
  }
  if (cudaMemsetAsync(ctrl, 0, 4 * sizeof(int), st) != cudaSuccess) return DSV4_ERR_CUDA;
  launch_k(route_count_kernel, nchunks, 256, 0, st,
           indices, T, k, E, allow_skip, chunk, nchunks,
                                              chunk_cnt, ctrl);
  launch_k(route_scan_kernel, (E + kScanThreads / 32 - 1) / (kScanThreads / 32), kScanThreads, 0, st,
           chunk_cnt, nchunks, E, shared_rows, block_n,
                                                max_rows, max_tiles, chunk_base, counts, seg_start,
                                                tiles, n_tiles, slot_token, slot_weight, ctrl, zero_ptr,
                                                n_zero);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_route_small_fused(const float* partials, int nsplit, float* logits_out, const float* bias, int T, int E,
                             int k, float route_scale, float* weights, int64_t* indices, const void* x, int H,
                             int shared_rows, int block_n, int max_rows, int max_tiles, int* chunk_base, int* counts,
                             int* seg_start, int4* tiles, int* n_tiles, int* slot_token, float* slot_weight,
                             int* ctrl, int* zero_ptr, int n_zero, int* route_slot, uint8_t* xq, uint8_t* sfb,
                             cudaStream_t st) {
  if (T <= 0 || T > kFusedMaxTokens || k > kMaxK || E > kFusedMaxExperts || E + 1 > kMaxSegments || H % 512)
    return DSV4_ERR_ARG;
  launch_k(route_small_fused_kernel, 1, 512, 0, st, partials, nsplit, logits_out, bias, T, E, k, route_scale,
           weights, indices, static_cast<const __nv_bfloat16*>(x), H, shared_rows, block_n, max_rows, max_tiles,
           chunk_base, counts, seg_start, tiles, n_tiles, slot_token, slot_weight, ctrl, zero_ptr, n_zero,
           route_slot, xq, sfb);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_route_scatter(const void* x, int n_x_rows, const uint8_t* rows_in,
                         long long rows_in_stride, const int64_t* indices, const float* weights,
                         int T, int k, int E, int H, int shared_rows, const int* seg_start,
                         const int* chunk_base, const int* ctrl, int* route_slot, int* slot_token,
                         float* slot_weight, uint8_t* xq, uint8_t* sfb, int num_sms,
                         cudaStream_t st) {
  if (T <= 0) return DSV4_OK;
  const int chunk = route_chunk_tokens(T);
  const int nchunks = (T + chunk - 1) / chunk;
  const int KT = H / 128;
  int ksplit = (4 * num_sms) / nchunks;
  ksplit = ksplit < 1 ? 1 : (ksplit > KT / kQuantGroup ? KT / kQuantGroup : ksplit);
  if (ksplit < 1) ksplit = 1;
  launch_k(route_scatter_kernel, dim3(nchunks, ksplit), 256, 0, st,
           static_cast<const __nv_bfloat16*>(x), n_x_rows, rows_in, rows_in_stride, indices, weights, T,
      k, E, H, shared_rows, chunk, nchunks, seg_start, chunk_base, ctrl, route_slot, slot_token,
      slot_weight, xq, sfb);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_permute_quant(const void* x, int H, const int* slot_token, const int* total_rows_ptr,
                         int max_rows, uint8_t* xq, uint8_t* sfb, int num_sms, cudaStream_t st) {
  const int warps = 8;
  int grid = (max_rows + warps - 1) / warps;
  grid = grid < num_sms * 8 ? grid : num_sms * 8;
  if (grid < 1) grid = 1;
  // few rows: split each row's k tiles (whole groups of kQuantGroup) over
  // blockIdx.y, up to about two CTAs per SM
  const int KT = H / 128;
  int ky = (2 * num_sms + grid - 1) / grid;
  const int kmax = (KT + kQuantGroup - 1) / kQuantGroup;
  ky = ky < kmax ? ky : kmax;
  if (ky < 1) ky = 1;
  while (ky > 1 && ((KT + ky - 1) / ky) % kQuantGroup) --ky;
  launch_k(permute_quant_kernel, dim3(grid, ky), warps * 32, 0, st,
           static_cast<const __nv_bfloat16*>(x), H,
                                                    slot_token, total_rows_ptr, xq, sfb);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_single_segment_plan(int T, int seg, int block_n, int rows_pad, const float* w,
                               int* slot_token, float* slot_weight, int4* tiles, int* n_tiles,
                               int* total_rows, cudaStream_t st) {
  const int grid = (rows_pad + 255) / 256;
  const int grid1 = grid > 0 ? grid : 1;
  launch_k(single_segment_plan_kernel, grid1, 256, 0, st,
           T, seg, block_n, rows_pad, w, slot_token, slot_weight, tiles, n_tiles, total_rows);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* s, int num_sms,
                     cudaStream_t st) {
  const int warps = 8;
  int grid = (M + warps - 1) / warps;
  grid = grid < num_sms * 8 ? grid : num_sms * 8;
  if (grid < 1) return DSV4_OK;
  launch_k(act_quant_kernel, grid, warps * 32, 0, st,
           static_cast<const __nv_bfloat16*>(x), M, K, q, s);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_fp4_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* s, int num_sms, cudaStream_t st) {
  const long long n = (long long)M * (K / 32);
  if (n <= 0) return DSV4_OK;
  long long grid = (n + 255) / 256;
  if (grid > 8LL * num_sms) grid = 8LL * num_sms;
  launch_k(fp4_act_quant_kernel, (unsigned)grid, 256, 0, st, static_cast<const __nv_bfloat16*>(x), M, K, q, s);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_fp4_scatter_quant(const void* x, int T, int H, int k, const int* route_slot, int max_rows, uint8_t* xq4,
                             uint8_t* atoms, int num_sms, cudaStream_t st) {
  const long long n = (long long)T * (H / 32);
  if (n <= 0) return DSV4_OK;
  long long grid = (n + 255) / 256;
  if (grid > 8LL * num_sms) grid = 8LL * num_sms;
  launch_k(fp4_scatter_quant_kernel, (unsigned)grid, 256, 0, st, static_cast<const __nv_bfloat16*>(x), T, H, k,
           route_slot, max_rows, xq4, atoms);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}


int launch_combine(const void* O, int H, const int* route_slot, const int64_t* indices, int T,
                   int k, const int* shared_base, void* y, cudaStream_t st, const void* O_shared) {
  if (T <= 0) return DSV4_OK;
  const __nv_bfloat16* o = static_cast<const __nv_bfloat16*>(O);
  const __nv_bfloat16* osh = O_shared ? static_cast<const __nv_bfloat16*>(O_shared) : o;
  const int threads = H / 8 < 512 ? H / 8 : 512;
  launch_k(combine_kernel, T, threads, 0, st,
           o, H, route_slot, indices, T, k, shared_base,
                                                          osh, static_cast<__nv_bfloat16*>(y));
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

}  // namespace dsv4
