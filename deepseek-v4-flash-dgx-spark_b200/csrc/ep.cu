// Expert parallelism: all-to-all dispatch of FP8 token rows to the ranks that
// own their experts, and the return of every route's bf16 output row.
//
// Replaces the reference's replicated-token expert parallelism
// (spark_runtime/lazy_official_runtime.py:956-965: every rank holds every
// token, computes its own experts, then dist.all_reduce(y) at :999-1000) with
// a dispatch/combine pair that moves only routed rows:
//
//   source rank          dsv4_ep_dispatch: each token is quantized once and
//                        written once per destination rank that owns any of
//                        its experts, with its routes in a metadata tail
//   (exchange)           counts, then rows, by the host (NCCL all-to-all)
//   owning rank          dsv4_ep_expert_forward: the received rows go through
//                        the same plan / scatter / grouped GEMMs as the single
//                        GPU layer (plus the rank's own tokens for the shared
//                        expert); every route's output row goes to a return
//                        buffer, grouped by source rank
//   (exchange)           return rows, by the host
//   source rank          dsv4_ep_combine: the single GPU combine over the
//                        returned rows (ascending expert id) + shared row
//
// Each route's output row is computed by exactly the arithmetic of the single
// GPU layer, and the combine sums the same rows in the same order, so the
// expert-parallel layer is bit-identical to the single GPU one.
//
// Send row layout (row_bytes, a multiple of 16):
//   [0, H)                 e4m3 codes of act_quant(x[t]) (per-128 blocks)
//   [H, H + H/128)         ue8m0 scale bytes, one per 128-wide block
//   [H + H/128, +12k)      k route entries: int32 expert id (-1 = routed to
//                          another rank), f32 routing weight, int32 index of
//                          the route's output row in the return block
//                          (routes to this rank in token order, then k order)
#include "kernels.cuh"

namespace dsv4 {

constexpr int kEpChunk = 256;  // tokens per dispatch chunk (8 warps, one token per lane)
constexpr int kEpMaxWorld = 8;
constexpr int kEpMetaEntry = 12;

// Exchange buffer of one rank (peer-memory expert parallelism), all offsets in
// bytes from its base:
//   [0, 32)        int32 disp_flag[8]: = epoch once source s's rows (and its
//                  info below) are in place
//   [32, 64)       int32 ret_flag[8]: = epoch once owner r's return rows are in place
//   [64, 192)      int32 info[8][4] per source s: rows, routes, offset of its
//                  return block from this rank in s's return region, unused
//   [192, 196)     int32 call counter: the epoch of this rank's current call
//                  when the caller passes epoch 0 (device-side counting, so a
//                  captured CUDA graph replays with a fresh epoch each time)
//   [1024, ...)    receive region: source s's rows at s * cap_tokens rows
//   then           return region: this rank's routes' bf16 output rows
//                  (cap_tokens * topk rows of H), in owner-rank blocks
constexpr int kEpHeaderBytes = 1024;
constexpr int kEpRetFlagOff = 32;
constexpr int kEpInfoOff = 64;
constexpr int kEpEpochOff = 192;

long long ep_row_bytes(int H, int k) { return ((long long)H + H / 128 + (long long)kEpMetaEntry * k + 15) / 16 * 16; }

// Where the send row `pos` for destination rank d lives.  Exchanged through
// host collectives (bases == nullptr): row pos of the local send buffer.  Over
// peer memory: row (pos - dst_base[2d]) of this rank's region in rank d's
// exchange buffer (bases[d] = that buffer as mapped here, IPC for peers).
struct EpPeerRows {
  const uint64_t* bases;  // [world] exchange buffer base of every rank, or nullptr
  int rank;               // this (source) rank
  long long cap_bytes;    // one source region: cap_tokens * row_bytes
  __device__ __forceinline__ uint8_t* row(uint8_t* send, int d, int pos, const int* dst_base,
                                          long long row_bytes) const {
    if (!bases) return send + (size_t)pos * row_bytes;
    return reinterpret_cast<uint8_t*>(bases[d]) + kEpHeaderBytes + (long long)rank * cap_bytes +
           (long long)(pos - dst_base[2 * d]) * row_bytes;
  }
};

__device__ __forceinline__ int warp_excl_scan(int v, int lane, int* total) {
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += a;
  }
  *total = __shfl_sync(0xffffffffu, inc, 31);
  return inc - v;
}

// Destination rank of each of token t's k routes (-1 for an invalid index).
__device__ __forceinline__ void route_dsts(const int64_t* __restrict__ indices, int t, int T, int k,
                                           int E, int per_rank, int* dst, int* expert,
                                           int* __restrict__ ctrl) {
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    dst[j] = -1;
    expert[j] = -1;
    if (t < T && j < k) {
      const int64_t v = indices[(size_t)t * k + j];
      if (v >= 0 && v < E) {
        expert[j] = static_cast<int>(v);
        dst[j] = static_cast<int>(v) / per_rank;
      } else {
        atomicOr(&ctrl[1], 1);
        record_error(DSV4_DEVERR_BAD_INDEX);
      }
    }
  }
}

// Per chunk and destination: rows (tokens with >= 1 route there) and routes.
// cc[(d * 2 + m) * nchunks + c], m = 0 rows, 1 routes.  The last CTA scans the
// chunk counts of each series (cb, exclusive) and totals them per destination
// (send_counts [world][2]; dst_base [world][2] exclusive over destinations).
__global__ void __launch_bounds__(kEpChunk) ep_count_kernel(
    const int64_t* __restrict__ indices, int T, int k, int E, int world, int nchunks,
    int* __restrict__ cc, int* __restrict__ cb, int* __restrict__ send_counts,
    int* __restrict__ dst_base, int* __restrict__ ctrl) {
  __shared__ int s_part[kEpChunk / 32][2 * kEpMaxWorld];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, c = blockIdx.x;
  const int t = c * kEpChunk + tid;
  int dst[kMaxK], expert[kMaxK];
  route_dsts(indices, t, T, k, E, E / world, dst, expert, ctrl);
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) {
    if (d >= world) break;
    int n = 0;
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) n += dst[j] == d;
    const int rows = __popc(__ballot_sync(0xffffffffu, n > 0));
    int routes = n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) routes += __shfl_xor_sync(0xffffffffu, routes, o);
    if (lane == 0) {
      s_part[warp][2 * d] = rows;
      s_part[warp][2 * d + 1] = routes;
    }
  }
  __syncthreads();
  if (tid < 2 * world) {
    int sum = 0;
    for (int w = 0; w < kEpChunk / 32; ++w) sum += s_part[w][tid];
    cc[(size_t)tid * nchunks + c] = sum;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&ctrl[0], 1) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // one warp per series (2 * world <= 16 series over 8 warps)
  for (int sr = warp; sr < 2 * world; sr += kEpChunk / 32) {
    int run = 0;
    for (int c0 = 0; c0 < nchunks; c0 += 32) {
      const int ci = c0 + lane;
      const int v = ci < nchunks ? __ldcg(cc + (size_t)sr * nchunks + ci) : 0;
      int total;
      const int ex = warp_excl_scan(v, lane, &total);
      if (ci < nchunks) cb[(size_t)sr * nchunks + ci] = run + ex;
      run += total;
    }
    if (lane == 0) send_counts[sr] = run;
  }
  __threadfence();
  __syncthreads();
  if (tid < 2) {  // tid 0: rows, tid 1: routes
    int run = 0;
    for (int d = 0; d < world; ++d) {
      dst_base[2 * d + tid] = run;
      run += __ldcg(send_counts + 2 * d + tid);
    }
  }
}

// Positions: the send row of every (token, destination) pair, the metadata
// tail of each send row, and ret_pos[t*k+j] = the row of the source's return
// buffer that will hold route j of token t (return blocks in rank order).
__global__ void __launch_bounds__(kEpChunk) ep_plan_kernel(
    const int64_t* __restrict__ indices, const float* __restrict__ weights, int T, int k, int E,
    int world, int H, long long row_bytes, int nchunks, const int* __restrict__ cb,
    const int* __restrict__ dst_base, int* __restrict__ row_pos, uint8_t* __restrict__ send,
    int* __restrict__ ret_pos, int* __restrict__ ctrl, EpPeerRows peer) {
  __shared__ int s_part[kEpChunk / 32][2 * kEpMaxWorld];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, c = blockIdx.x;
  const int t = c * kEpChunk + tid;
  int dst[kMaxK], expert[kMaxK];
  route_dsts(indices, t, T, k, E, E / world, dst, expert, ctrl);
  int rrank[kEpMaxWorld], rbase[kEpMaxWorld], cnt[kEpMaxWorld];
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) {
    cnt[d] = 0;
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) cnt[d] += dst[j] == d;
    const unsigned b = __ballot_sync(0xffffffffu, cnt[d] > 0);
    rrank[d] = __popc(b & ((1u << lane) - 1u));
    int total;
    rbase[d] = warp_excl_scan(cnt[d], lane, &total);
    if (lane == 0 && d < world) {
      s_part[warp][2 * d] = __popc(b);
      s_part[warp][2 * d + 1] = total;
    }
  }
  if (t < T)
    for (int j = 0; j < k; ++j) ret_pos[(size_t)t * k + j] = -1;
  __syncthreads();
  if (__ldcg(ctrl + 1) || t >= T) {
    if (t < T)
      for (int d = 0; d < world; ++d) row_pos[(size_t)t * world + d] = -1;
    return;
  }
  const size_t meta_off = (size_t)H + H / 128;
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) {
    if (d >= world) break;
    int pos = -1;
    if (cnt[d] > 0) {
      int wrow = 0, wroute = 0;
      for (int w = 0; w < warp; ++w) {
        wrow += s_part[w][2 * d];
        wroute += s_part[w][2 * d + 1];
      }
      pos = dst_base[2 * d] + cb[(size_t)(2 * d) * nchunks + c] + wrow + rrank[d];
      // route index inside the return block from rank d
      int ridx = cb[(size_t)(2 * d + 1) * nchunks + c] + wroute + rbase[d];
      uint8_t* meta = peer.row(send, d, pos, dst_base, row_bytes) + meta_off;
#pragma unroll
      for (int j = 0; j < kMaxK; ++j) {
        if (j >= k) break;
        int32_t e = -1, ri = -1;
        float w = 0.f;
        if (dst[j] == d) {
          e = expert[j];
          w = weights[(size_t)t * k + j];
          ri = ridx++;
          ret_pos[(size_t)t * k + j] = dst_base[2 * d + 1] + ri;
        }
        reinterpret_cast<int32_t*>(meta + kEpMetaEntry * j)[0] = e;
        reinterpret_cast<float*>(meta + kEpMetaEntry * j)[1] = w;
        reinterpret_cast<int32_t*>(meta + kEpMetaEntry * j)[2] = ri;
      }
    }
    row_pos[(size_t)t * world + d] = pos;
  }
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The call counter in this rank's own buffer.
__device__ __forceinline__ int* ep_counter(const uint64_t* bases, int rank) {
  return reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bases[rank]) + kEpEpochOff);
}

// Source, one warp: tell owner d how many rows / routes arrived from this
// rank and where their returns go, then raise disp_flag[rank] in d's buffer
// (release, system scope).  Lane d takes destination d.  epoch <= 0: this
// call's epoch is the own call counter plus one (stored back).  The caller has
// made every row store visible at system scope first.
__device__ __forceinline__ void signal_dispatch(const uint64_t* __restrict__ bases, int rank, int world,
                                                const int* __restrict__ send_counts,
                                                const int* __restrict__ dst_base, int epoch) {
  const int d = threadIdx.x & 31;
  if (epoch <= 0) {
    int e = 0;
    if (d == 0) {
      int* ctr = ep_counter(bases, rank);
      e = *ctr + 1;
      *ctr = e;
    }
    epoch = __shfl_sync(0xffffffffu, e, 0);
  }
  if (d >= world) return;
  uint8_t* b = reinterpret_cast<uint8_t*>(bases[d]);
  int* info = reinterpret_cast<int*>(b + kEpInfoOff) + 4 * rank;
  info[0] = __ldcg(send_counts + 2 * d);
  info[1] = __ldcg(send_counts + 2 * d + 1);
  info[2] = __ldcg(dst_base + 2 * d + 1);
  __threadfence_system();
  st_release_sys(reinterpret_cast<int*>(b) + rank, epoch);
}

// A source with no rows to send (one warp): the counts and offsets are zeros.
__global__ void ep_signal_dispatch_kernel(const uint64_t* __restrict__ bases, int rank, int world,
                                          const int* __restrict__ send_counts,
                                          const int* __restrict__ dst_base, int epoch) {
  signal_dispatch(bases, rank, world, send_counts, dst_base, epoch);
}

// Data: one warp per (token, group of quads) quantizes the row once and writes
// codes + scale bytes into each of its send rows.  Over peer memory the kernel
// also publishes them: every thread fences its stores at system scope, each
// CTA then counts itself done (pack_ctr, zeroed by the dispatch), and the CTA
// that completes the count raises the owners' flags (signal_dispatch).
__global__ void __launch_bounds__(256) ep_pack_kernel(const __nv_bfloat16* __restrict__ x, int T,
                                                      int H, int world, long long row_bytes,
                                                      const int* __restrict__ row_pos,
                                                      int qsplit, uint8_t* __restrict__ send,
                                                      const int* __restrict__ dst_base,
                                                      EpPeerRows peer, int* __restrict__ pack_ctr,
                                                      const int* __restrict__ send_counts, int epoch) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int t = gw / qsplit, part = gw % qsplit;
  const int KQ = H / 512;
  const int per = (KQ + qsplit - 1) / qsplit;
  const int q0 = part * per, q1 = min(KQ, q0 + per);
  int pos[kEpMaxWorld];
  int np = 0;
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) {
    pos[d] = (t < T && d < world) ? row_pos[(size_t)t * world + d] : -1;
    np += pos[d] >= 0;
  }
  const __nv_bfloat16* xrow = x + (size_t)(t < T ? t : 0) * H;
  for (int q = q0; np > 0 && q < q1; q += 2) {
    uint4 raw[2][2];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      raw[g][0] = raw[g][1] = make_uint4(0, 0, 0, 0);
      if (q + g < q1) {
        raw[g][0] = *reinterpret_cast<const uint4*>(xrow + (size_t)(q + g) * 512 + lane * 16);
        raw[g][1] = *reinterpret_cast<const uint4*>(xrow + (size_t)(q + g) * 512 + lane * 16 + 8);
      }
    }
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      if (q + g >= q1) break;
      uint4 code;
      uint32_t sc;
      quad_quant(raw[g], lane, &code, &sc);
      const uint32_t s4 = __shfl_sync(0xffffffffu, sc, 0) | (__shfl_sync(0xffffffffu, sc, 8) << 8) |
                          (__shfl_sync(0xffffffffu, sc, 16) << 16) |
                          (__shfl_sync(0xffffffffu, sc, 24) << 24);
#pragma unroll
      for (int d = 0; d < kEpMaxWorld; ++d) {
        if (pos[d] < 0) continue;
        uint8_t* row = peer.row(send, d, pos[d], dst_base, row_bytes);
        *reinterpret_cast<uint4*>(row + (size_t)(q + g) * 512 + lane * 16) = code;
        if (lane == 0) *reinterpret_cast<uint32_t*>(row + H + (q + g) * 4) = s4;
      }
    }
  }
  if (!peer.bases) return;  // host exchange: nothing to publish
  __shared__ int s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(pack_ctr, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();  // every CTA's rows (and the plan kernel's row tails) before the flags
  if (threadIdx.x < 32) signal_dispatch(peer.bases, peer.rank, world, send_counts, dst_base, epoch);
}

// Receiver: routing of the T_own + R local rows.  Rows t < T_own are this
// rank's own tokens (shared expert only); row T_own + i is received row i.
// Route j of a received row becomes local expert e - e_begin and its output
// row goes to ret_dst = (routes received from earlier sources) + its return
// index.  recv_counts [world][2] are the (rows, routes) received per source.
__global__ void ep_unpack_kernel(const uint8_t* __restrict__ recv, int R, int T_own, int k, int H,
                                 long long row_bytes, int e_begin, int e_count,
                                 const int* __restrict__ recv_counts, int world,
                                 int64_t* __restrict__ idx_local, float* __restrict__ w_local,
                                 int* __restrict__ ret_dst) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T_own + R) return;
  if (t < T_own) {
    for (int j = 0; j < k; ++j) {
      idx_local[(size_t)t * k + j] = -1;
      w_local[(size_t)t * k + j] = 0.f;
      ret_dst[(size_t)t * k + j] = -1;
    }
    return;
  }
  const int i = t - T_own;
  int row_run = 0, route_run = 0, route_base = 0;
  for (int s = 0; s < world; ++s) {
    const int nr = recv_counts[2 * s], nrt = recv_counts[2 * s + 1];
    if (i >= row_run && i < row_run + nr) route_base = route_run;
    row_run += nr;
    route_run += nrt;
  }
  const uint8_t* meta = recv + (size_t)i * row_bytes + H + H / 128;
  for (int j = 0; j < k; ++j) {
    const int32_t e = reinterpret_cast<const int32_t*>(meta + kEpMetaEntry * j)[0];
    const float w = reinterpret_cast<const float*>(meta + kEpMetaEntry * j)[1];
    const int32_t ri = reinterpret_cast<const int32_t*>(meta + kEpMetaEntry * j)[2];
    int64_t le = -1;
    int rd = -1;
    if (e >= 0) {
      if (e >= e_begin && e < e_begin + e_count && ri >= 0 && route_base + ri < route_run) {
        le = e - e_begin;
        rd = route_base + ri;
      } else {
        record_error(DSV4_DEVERR_BAD_INDEX);
      }
    }
    idx_local[(size_t)t * k + j] = le;
    w_local[(size_t)t * k + j] = w;
    ret_dst[(size_t)t * k + j] = rd;
  }
}

// Receiver: every received route's output row (plan slot order in O) to its
// place in the return buffer.  One warp per route, 16-byte copies.
__global__ void __launch_bounds__(256) ep_return_gather_kernel(
    const __nv_bfloat16* __restrict__ O, int H, const int* __restrict__ route_slot,
    const int* __restrict__ ret_dst, int n_routes, long long ret_rows,
    __nv_bfloat16* __restrict__ ret) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n_routes; r += nwarps) {
    const int d = ret_dst[r];
    const int s = route_slot[r];
    if (d < 0 || s < 0 || d >= ret_rows) continue;
    const uint4* src = reinterpret_cast<const uint4*>(O + (size_t)s * H);
    uint4* dst = reinterpret_cast<uint4*>(ret + (size_t)d * H);
    for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
  }
}

// ---------------------------------------------------------------------------
// peer-memory exchange: signals, bounded waits, unpack and return over NVLink
// ---------------------------------------------------------------------------
// Owner: every route row is in its source's return region (previous launch);
// raise ret_flag[rank] in every rank's buffer.
__global__ void ep_signal_return_kernel(const uint64_t* __restrict__ bases, int rank, int world,
                                        int epoch) {
  const int d = threadIdx.x;
  if (d >= world) return;
  if (epoch <= 0) epoch = *ep_counter(bases, rank);
  __threadfence_system();
  st_release_sys(reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bases[d]) + kEpRetFlagOff) + rank,
                 epoch);
}

// Bounded wait until the flags at own + flag_off, one per rank, all equal
// epoch (epoch <= 0: the own call counter).  On timeout the lane records
// err_code and returns: the kernels that follow then read whatever the buffer
// holds, the host sees the error.
__global__ void ep_wait_kernel(const uint8_t* __restrict__ own, int flag_off, int world, int epoch,
                               int err_code) {
  const int s = threadIdx.x;
  if (s >= world) return;
  if (epoch <= 0) epoch = *reinterpret_cast<const int*>(own + kEpEpochOff);
  const int* flags = reinterpret_cast<const int*>(own + flag_off);
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flags + s) != epoch) {
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      record_error(err_code);
      return;
    }
    __nanosleep(200);
  }
}

// Owner, peer-memory form of ep_unpack_kernel: received row i sits in source
// s = i / cap's region, valid when i % cap < info[s].rows.  A route's return
// destination is encoded as (s << 24) | row in s's return region.
__global__ void ep_unpack_p2p_kernel(const uint8_t* __restrict__ exch, int cap, int T_own, int k,
                                     int H, long long row_bytes, int e_begin, int e_count,
                                     int world, int ret_cap, int64_t* __restrict__ idx_local,
                                     float* __restrict__ w_local, int* __restrict__ ret_dst) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = T_own + world * cap;
  if (t >= n) return;
  int s = -1, ii = 0;
  if (t >= T_own) {
    s = (t - T_own) / cap;
    ii = (t - T_own) - s * cap;
  }
  const int* info = reinterpret_cast<const int*>(exch + kEpInfoOff);
  const bool valid = s >= 0 && ii < info[4 * s];
  if (!valid) {
    for (int j = 0; j < k; ++j) {
      idx_local[(size_t)t * k + j] = -1;
      w_local[(size_t)t * k + j] = 0.f;
      ret_dst[(size_t)t * k + j] = -1;
    }
    return;
  }
  const int routes = info[4 * s + 1], ret_off = info[4 * s + 2];
  const uint8_t* meta = exch + kEpHeaderBytes + (size_t)(t - T_own) * row_bytes + H + H / 128;
  for (int j = 0; j < k; ++j) {
    const int32_t e = reinterpret_cast<const int32_t*>(meta + kEpMetaEntry * j)[0];
    const float w = reinterpret_cast<const float*>(meta + kEpMetaEntry * j)[1];
    const int32_t ri = reinterpret_cast<const int32_t*>(meta + kEpMetaEntry * j)[2];
    int64_t le = -1;
    int rd = -1;
    if (e >= 0) {
      const int dst = ret_off + ri;
      if (e >= e_begin && e < e_begin + e_count && ri >= 0 && ri < routes && ret_off >= 0 &&
          dst < ret_cap) {
        le = e - e_begin;
        rd = (s << 24) | dst;
      } else {
        record_error(DSV4_DEVERR_BAD_INDEX);
      }
    }
    idx_local[(size_t)t * k + j] = le;
    w_local[(size_t)t * k + j] = w;
    ret_dst[(size_t)t * k + j] = rd;
  }
}

// Owner: every received route's output row straight into its source's return
// region over peer memory (one warp per route, 16-byte stores).
__global__ void __launch_bounds__(256) ep_return_p2p_kernel(
    const __nv_bfloat16* __restrict__ O, int H, const int* __restrict__ route_slot,
    const int* __restrict__ ret_dst, int n_routes, const uint64_t* __restrict__ bases, int world,
    long long ret_region_off, int ret_cap) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n_routes; r += nwarps) {
    const int d = ret_dst[r];
    const int sl = route_slot[r];
    if (d < 0 || sl < 0) continue;
    const int s = d >> 24, row = d & 0xFFFFFF;
    if (s >= world || row >= ret_cap) continue;
    const uint4* src = reinterpret_cast<const uint4*>(O + (size_t)sl * H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(bases[s]) + ret_region_off +
                                          (size_t)row * H * 2);
    for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
long long ep_dispatch_workspace(int T, int world) {
  const long long nchunks = (T + kEpChunk - 1) / kEpChunk;
  const long long series = (2LL * world * nchunks * 4 + 255) / 256 * 256;
  return 256 + 2 * series + 256 + ((long long)T * world * 4 + 255) / 256 * 256;
}

long long ep_exchange_bytes(int H, int k, int world, int cap) {
  const long long recv = ((long long)world * cap * ep_row_bytes(H, k) + 255) / 256 * 256;
  const long long ret = ((long long)cap * k * H * 2 + 255) / 256 * 256;
  return kEpHeaderBytes + recv + ret;
}

long long ep_return_region_off(int H, int k, int world, int cap) {
  return kEpHeaderBytes + ((long long)world * cap * ep_row_bytes(H, k) + 255) / 256 * 256;
}

int launch_ep_dispatch(const void* x, const int64_t* indices, const float* weights, int T, int H,
                       int k, int E, int world, uint8_t* send, int* send_counts, int* ret_pos,
                       uint8_t* ws, int num_sms, cudaStream_t st, const uint64_t* peer_bases,
                       int rank, int cap, int epoch) {
  const int nchunks = (T + kEpChunk - 1) / kEpChunk;
  const long long series = (2LL * world * nchunks * 4 + 255) / 256 * 256;
  int* ctrl = reinterpret_cast<int*>(ws);
  int* cc = reinterpret_cast<int*>(ws + 256);
  int* cb = reinterpret_cast<int*>(ws + 256 + series);
  int* dst_base = reinterpret_cast<int*>(ws + 256 + 2 * series);
  int* row_pos = reinterpret_cast<int*>(ws + 256 + 2 * series + 256);
  const long long rb = ep_row_bytes(H, k);
  if (cudaMemsetAsync(ctrl, 0, 16, st) != cudaSuccess) return DSV4_ERR_CUDA;
  launch_k(ep_count_kernel, nchunks, kEpChunk, 0, st,
           indices, T, k, E, world, nchunks, cc, cb,
                                               send_counts, dst_base, ctrl);
  EpPeerRows peer{peer_bases, rank, (long long)cap * rb};
  launch_k(ep_plan_kernel, nchunks, kEpChunk, 0, st, indices, weights, T, k, E, world, H, rb,
           nchunks, cb, dst_base, row_pos, send, ret_pos, ctrl, peer);
  const int KQ = H / 512;
  int qsplit = (int)((8LL * num_sms * 8 + T - 1) / T);  // about 8 warps per SM slot
  qsplit = qsplit < 1 ? 1 : (qsplit > KQ ? KQ : qsplit);
  const long long warps = (long long)T * qsplit;
  // over peer memory the pack kernel's last CTA also raises the owners' flags
  launch_k(ep_pack_kernel, (unsigned)((warps + 7) / 8), 256, 0, st,
           static_cast<const __nv_bfloat16*>(x), T, H, world, rb, row_pos, qsplit, send,
           (const int*)dst_base, peer, ctrl + 2, (const int*)send_counts, epoch);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

// A source with no tokens: zero counts and offsets, then the dispatch signal.
int launch_ep_signal_empty(const uint64_t* peer_bases, int rank, int world, int* send_counts,
                           uint8_t* ws, int epoch, cudaStream_t st) {
  int* zero_base = reinterpret_cast<int*>(ws);  // [world][2] zeros (dst_base of no rows)
  if (cudaMemsetAsync(send_counts, 0, 2 * world * sizeof(int), st) != cudaSuccess ||
      cudaMemsetAsync(zero_base, 0, 2 * world * sizeof(int), st) != cudaSuccess)
    return DSV4_ERR_CUDA;
  launch_k(ep_signal_dispatch_kernel, 1, 32, 0, st, peer_bases, rank, world,
           (const int*)send_counts, (const int*)zero_base, epoch);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_ep_wait(const uint8_t* own, int flag_off, int world, int epoch, int err_code,
                   cudaStream_t st) {
  launch_k(ep_wait_kernel, 1, 32, 0, st, own, flag_off, world, epoch, err_code);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_ep_unpack_p2p(const uint8_t* exch, int cap, int T_own, int k, int H, int e_begin,
                         int e_count, int world, int64_t* idx_local, float* w_local, int* ret_dst,
                         cudaStream_t st) {
  const int n = T_own + world * cap;
  if (n <= 0) return DSV4_OK;
  launch_k(ep_unpack_p2p_kernel, (n + 255) / 256, 256, 0, st, exch, cap, T_own, k, H,
           ep_row_bytes(H, k), e_begin, e_count, world, cap * k, idx_local, w_local, ret_dst);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_ep_return_p2p(const void* O, int H, int k, const int* route_slot, const int* ret_dst,
                         int n_routes, const uint64_t* bases, int rank, int world, int cap,
                         int epoch, int num_sms, cudaStream_t st) {
  if (n_routes > 0) {
    int grid = (n_routes + 7) / 8;
    grid = grid < num_sms * 8 ? grid : num_sms * 8;
    launch_k(ep_return_p2p_kernel, grid, 256, 0, st, static_cast<const __nv_bfloat16*>(O), H,
             route_slot, ret_dst, n_routes, bases, world, ep_return_region_off(H, k, world, cap),
             cap * k);
  }
  launch_k(ep_signal_return_kernel, 1, 32, 0, st, bases, rank, world, epoch);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_ep_unpack(const uint8_t* recv, int R, int T_own, int k, int H, int e_begin, int e_count,
                     const int* recv_counts, int world, int64_t* idx_local, float* w_local,
                     int* ret_dst, cudaStream_t st) {
  const int n = T_own + R;
  if (n <= 0) return DSV4_OK;
  launch_k(ep_unpack_kernel, (n + 255) / 256, 256, 0, st,
           recv, R, T_own, k, H, ep_row_bytes(H, k), e_begin,
                                                    e_count, recv_counts, world, idx_local,
                                                    w_local, ret_dst);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_ep_return_gather(const void* O, int H, const int* route_slot, const int* ret_dst,
                            int n_routes, long long ret_rows, void* ret, int num_sms,
                            cudaStream_t st) {
  if (n_routes <= 0) return DSV4_OK;
  int grid = (n_routes + 7) / 8;
  grid = grid < num_sms * 8 ? grid : num_sms * 8;
  launch_k(ep_return_gather_kernel, grid, 256, 0, st,
           static_cast<const __nv_bfloat16*>(O), H, route_slot,
                                                ret_dst, n_routes, ret_rows,
                                                static_cast<__nv_bfloat16*>(ret));
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

}  // namespace dsv4
