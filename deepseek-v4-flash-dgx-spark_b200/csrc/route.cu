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
// Route plan (one CTA).  Stable counting sort of the T*k (token, rank) routes
// into per-expert segments: inside a segment rows follow token order, which is
// the order torch.where gives.  Segment sizes are padded to 32 rows so every
// GEMM tile starts on a 32-row boundary of the activation scale atoms.  The
// shared expert is segment E and holds every token.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kSegAlign = 32;

__global__ void __launch_bounds__(kPlanThreads) route_plan_kernel(
    const int64_t* __restrict__ indices, const float* __restrict__ weights, int T, int k, int E,
    int include_shared, int block_n, int max_rows, int max_tiles, int* __restrict__ counts,
    int* __restrict__ seg_start, int* __restrict__ route_slot, int* __restrict__ slot_token,
    float* __restrict__ slot_weight, int4* __restrict__ tiles, int* __restrict__ n_tiles) {
  extern __shared__ int sm[];
  const int NS = E + 1;                  // segments: E routed + shared
  int* cnt = sm;                         // [NS]
  int* tbase = cnt + NS;                 // [NS + 1] tile base per segment
  int* warp_cnt = tbase + NS + 1;        // [kPlanWarps][NS]
  __shared__ int s_total_rows, s_total_tiles, s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < NS; i += kPlanThreads) cnt[i] = 0;
  for (int i = tid; i < kPlanWarps * NS; i += kPlanThreads) warp_cnt[i] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();

  const int n_routes = T * k;
  for (int base = 0; base < n_routes; base += kPlanThreads) {
    const int i = base + tid;
    int e = -1;
    if (i < n_routes) {
      const int64_t v = indices[i];
      if (v >= 0 && v < E) e = static_cast<int>(v);
      else s_bad = 1;
    }
    const unsigned mask = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(mask & ((1u << lane) - 1u));
    const bool leader = (__ffs(mask) - 1) == lane;
    if (leader && e >= 0) warp_cnt[warp * NS + e] = __popc(mask);
    __syncthreads();
    for (int s = tid; s < E; s += kPlanThreads) {
      int run = cnt[s];
      for (int w = 0; w < kPlanWarps; ++w) {
        const int c = warp_cnt[w * NS + s];
        if (c) {
          warp_cnt[w * NS + s] = run;
          run += c;
        }
      }
      cnt[s] = run;
    }
    __syncthreads();
    if (e >= 0) route_slot[i] = warp_cnt[warp * NS + e] + rank_w;  // rank inside segment
    __syncthreads();
    if (leader && e >= 0) warp_cnt[warp * NS + e] = 0;
    __syncthreads();
  }
  if (tid == 0) cnt[E] = include_shared ? T : 0;
  __syncthreads();

  // exclusive scans of padded row counts and of tile counts (warp 0)
  if (warp == 0) {
    int row_run = 0, tile_run = 0;
    for (int s0 = 0; s0 < NS; s0 += 32) {
      const int s = s0 + lane;
      const int c = s < NS ? cnt[s] : 0;
      const int rows = (c + kSegAlign - 1) / kSegAlign * kSegAlign;
      const int nt = (c + block_n - 1) / block_n;
      int r_inc = rows, t_inc = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, r_inc, o);
        const int b = __shfl_up_sync(0xffffffffu, t_inc, o);
        if (lane >= o) {
          r_inc += a;
          t_inc += b;
        }
      }
      if (s < NS) {
        seg_start[s] = row_run + r_inc - rows;
        tbase[s] = tile_run + t_inc - nt;
      }
      row_run += __shfl_sync(0xffffffffu, r_inc, 31);
      tile_run += __shfl_sync(0xffffffffu, t_inc, 31);
    }
    if (lane == 0) {
      seg_start[NS] = row_run;
      tbase[NS] = tile_run;
      s_total_rows = row_run;
      s_total_tiles = tile_run;
    }
  }
  __syncthreads();
  if (s_total_rows > max_rows || s_total_tiles > max_tiles || s_bad) {
    if (tid == 0) {
      record_error(s_bad ? DSV4_DEVERR_BAD_INDEX : DSV4_DEVERR_PLAN_OVERFLOW);
      *n_tiles = 0;
    }
    return;
  }

  for (int i = tid; i < n_routes; i += kPlanThreads) {
    const int e = static_cast<int>(indices[i]);
    const int slot = seg_start[e] + route_slot[i];
    route_slot[i] = slot;
    slot_token[slot] = i / k;
    slot_weight[slot] = weights[i];
  }
  if (include_shared) {
    for (int t = tid; t < T; t += kPlanThreads) {
      slot_token[seg_start[E] + t] = t;
      slot_weight[seg_start[E] + t] = 1.0f;
    }
  }
  for (int s = tid; s < NS; s += kPlanThreads) {
    const int c = cnt[s];
    counts[s] = c;
    for (int r = seg_start[s] + c; r < seg_start[s + 1]; ++r) {
      slot_token[r] = -1;
      slot_weight[r] = 0.f;
    }
    const int nt = tbase[s + 1] - tbase[s];
    for (int m = 0; m < nt; ++m)
      tiles[tbase[s] + m] = make_int4(s, seg_start[s] + m * block_n, min(block_n, c - m * block_n), 0);
  }
  if (tid == 0) *n_tiles = s_total_tiles;
}

// ---------------------------------------------------------------------------
// Per-128 act_quant of one row by one warp: lane l owns elements 4l..4l+3 of
// each 128-wide block.  Blocks are processed 8 at a time with all 8 loads in
// flight before any is used (the rows come from L2/DRAM: latency-bound).
// ---------------------------------------------------------------------------
constexpr int kQuantGroup = 8;

template <typename ScaleSink>
__device__ __forceinline__ void quant_row(const __nv_bfloat16* __restrict__ src, bool valid,
                                          uint8_t* __restrict__ dst, int KT, int lane,
                                          ScaleSink sink) {
  for (int k0 = 0; k0 < KT; k0 += kQuantGroup) {
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
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < total; row += nwarps) {
    const int t = slot_token[row];
    quant_row(x + (size_t)(t < 0 ? 0 : t) * H, t >= 0, xq + (size_t)row * H, KT, lane,
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
    quant_row(x + (size_t)row * K, true, q + (size_t)row * K, KT, lane, [&](int kt, uint32_t sc) {
      if (lane == 0) s[(size_t)row * KT + kt] = static_cast<uint8_t>(sc);
    });
  }
}

// ---------------------------------------------------------------------------
// Combine: y[t] = bf16( sum over t's routes in ascending expert id of O[slot]
// (fp32) + O[shared slot] ).  Routing weights were applied inside the expert
// (before w2), so this is a plain ordered sum.  One CTA per token, one thread
// per 8-element chunk: a thread's k+1 row loads are all in flight at once.
// ---------------------------------------------------------------------------
constexpr int kMaxK = 8;

__global__ void __launch_bounds__(512) combine_kernel(const __nv_bfloat16* __restrict__ O, int H,
                                                      const int* __restrict__ route_slot,
                                                      const int64_t* __restrict__ indices, int T,
                                                      int k, const int* __restrict__ shared_base,
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
      const uint4 raw = *reinterpret_cast<const uint4*>(O + (size_t)sh * H + c * 8);
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
    if (r < nt) tiles[r] = make_int4(seg, r * block_n, min(block_n, T - r * block_n), 0);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *n_tiles = nt;
    *total_rows = rows_pad;
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
int launch_route_plan(const int64_t* indices, const float* weights, int T, int k, int E,
                      int include_shared, int block_n, int max_rows, int max_tiles, int* counts,
                      int* seg_start, int* route_slot, int* slot_token, float* slot_weight,
                      int4* tiles, int* n_tiles, cudaStream_t st) {
  const int NS = E + 1;
  const size_t smem = (size_t)(NS + NS + 1 + kPlanWarps * NS) * sizeof(int);
  if (cudaFuncSetAttribute(route_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return DSV4_ERR_CUDA;
  route_plan_kernel<<<1, kPlanThreads, smem, st>>>(indices, weights, T, k, E, include_shared,
                                                   block_n, max_rows, max_tiles, counts, seg_start,
                                                   route_slot, slot_token, slot_weight, tiles,
                                                   n_tiles);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_permute_quant(const void* x, int H, const int* slot_token, const int* total_rows_ptr,
                         int max_rows, uint8_t* xq, uint8_t* sfb, int num_sms, cudaStream_t st) {
  const int warps = 8;
  int grid = (max_rows + warps - 1) / warps;
  grid = grid < num_sms * 8 ? grid : num_sms * 8;
  if (grid < 1) grid = 1;
  permute_quant_kernel<<<grid, warps * 32, 0, st>>>(static_cast<const __nv_bfloat16*>(x), H,
                                                    slot_token, total_rows_ptr, xq, sfb);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_single_segment_plan(int T, int seg, int block_n, int rows_pad, const float* w,
                               int* slot_token, float* slot_weight, int4* tiles, int* n_tiles,
                               int* total_rows, cudaStream_t st) {
  const int grid = (rows_pad + 255) / 256;
  single_segment_plan_kernel<<<grid > 0 ? grid : 1, 256, 0, st>>>(
      T, seg, block_n, rows_pad, w, slot_token, slot_weight, tiles, n_tiles, total_rows);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* s, int num_sms,
                     cudaStream_t st) {
  const int warps = 8;
  int grid = (M + warps - 1) / warps;
  grid = grid < num_sms * 8 ? grid : num_sms * 8;
  if (grid < 1) return DSV4_OK;
  act_quant_kernel<<<grid, warps * 32, 0, st>>>(static_cast<const __nv_bfloat16*>(x), M, K, q, s);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_combine(const void* O, int H, const int* route_slot, const int64_t* indices, int T,
                   int k, const int* shared_base, void* y, cudaStream_t st) {
  if (T <= 0) return DSV4_OK;
  combine_kernel<<<T, H / 8 < 512 ? H / 8 : 512, 0, st>>>(static_cast<const __nv_bfloat16*>(O), H, route_slot, indices,
                                    T, k, shared_base, static_cast<__nv_bfloat16*>(y));
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

}  // namespace dsv4
