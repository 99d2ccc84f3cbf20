// L2 prefetch of a decode layer's expert weights, overlapped with the routing.
//
// At decode sizes the layer's kernels before the expert GEMMs (route plan,
// permutation + act_quant) are latency-bound and leave HBM idle, while each
// GEMM then pays its first wave's memory latency (page walks, first DRAM
// round trips) before it streams.  Once the gate has chosen the experts this
// kernel, launched on a side stream next to the routing kernels, asks L2 for
// the touched experts' GEMM1 weights (w1, w3 and their scale atoms; the shared
// expert's after the routed ones) and then their GEMM2 weights (w2), in the
// order the GEMMs visit them, up to a byte budget below the L2 capacity.  The
// requests are bulk prefetches (cp.async.bulk.prefetch.L2: no data returns to
// the SM, no multicast), so every CTA only issues them and exits.
#include "kernels.cuh"

namespace dsv4 {

constexpr int kPrefetchChunk = 64 * 1024;  // bytes per bulk prefetch
constexpr int kPrefetchMaxExperts = 512;

__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)),
               "r"(bytes)
               : "memory");
}

struct PrefetchArgs {
  const int64_t* indices;  // [n_idx] routed expert ids of the batch (out of range: ignored)
  int n_idx;
  int n_routed;
  const int* expert_slot;
  int n_slots;
  const uint8_t* arena;
  long long slot_stride;
  const uint8_t* arena_sf;
  long long sf_slot_stride;
  long long w1_off, w3_off, w2_off;  // weight offsets inside a slot
  long long wg_bytes;                // bytes of one routed weight matrix
  long long sf_bytes;                // bytes of one matrix's scale atoms
  const uint8_t* shared_w1;
  const uint8_t* shared_w3;
  const uint8_t* shared_w2;
  const uint8_t* shared_sf;
  long long shared_bytes;            // bytes of one shared-expert matrix
  long long budget;                  // total bytes to prefetch
};

// Parts (address, bytes) of expert e's region in pass 0 (GEMM1: w1, w3, their
// atoms) or pass 1 (GEMM2: w2 and its atoms); e == n_routed is the shared expert.
__device__ __forceinline__ int prefetch_parts(const PrefetchArgs& a, int pass, int e,
                                              const uint8_t** ptr, long long* len) {
  if (e == a.n_routed) {
    if (!a.shared_w1) return 0;
    if (pass == 0) {
      ptr[0] = a.shared_w1; len[0] = a.shared_bytes;
      ptr[1] = a.shared_w3; len[1] = a.shared_bytes;
      ptr[2] = a.shared_sf; len[2] = 2 * a.sf_bytes;
      return 3;
    }
    ptr[0] = a.shared_w2; len[0] = a.shared_bytes;
    ptr[1] = a.shared_sf + 2 * a.sf_bytes; len[1] = a.sf_bytes;
    return 2;
  }
  const int slot = a.expert_slot[e];
  if (slot < 0 || slot >= a.n_slots) return 0;  // the GEMM skips such an expert too
  const uint8_t* w = a.arena + (size_t)slot * a.slot_stride;
  const uint8_t* sf = a.arena_sf + (size_t)slot * a.sf_slot_stride;
  if (pass == 0) {
    ptr[0] = w + a.w1_off; len[0] = a.wg_bytes;
    ptr[1] = w + a.w3_off; len[1] = a.wg_bytes;
    ptr[2] = sf; len[2] = 2 * a.sf_bytes;
    return 3;
  }
  ptr[0] = w + a.w2_off; len[0] = a.wg_bytes;
  ptr[1] = sf + 2 * a.sf_bytes; len[1] = a.sf_bytes;
  return 2;
}

// Every CTA finds the touched experts from the indices, walks the parts in the
// GEMMs' order and issues the 64 KB chunks whose order index is congruent to
// its own index (round robin over the grid), stopping at the budget.
__global__ void __launch_bounds__(128) weight_prefetch_kernel(const PrefetchArgs a) {
  __shared__ uint32_t touched[kPrefetchMaxExperts / 32];
  for (int i = threadIdx.x; i < kPrefetchMaxExperts / 32; i += blockDim.x) touched[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < a.n_idx; i += blockDim.x) {
    const int64_t e = a.indices[i];
    if (e >= 0 && e < a.n_routed) atomicOr(&touched[e >> 5], 1u << (e & 31));
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  const long long G = gridDim.x;
  long long pos = 0;    // bytes of the order before the current part
  long long chunk = 0;  // order index of the current part's first chunk
  for (int pass = 0; pass < 2 && pos < a.budget; ++pass) {
    for (int e = 0; e <= a.n_routed && pos < a.budget; ++e) {
      if (e < a.n_routed && !(touched[e >> 5] >> (e & 31) & 1)) continue;
      const uint8_t* ptr[3];
      long long len[3];
      const int n = prefetch_parts(a, pass, e, ptr, len);
      for (int p = 0; p < n && pos < a.budget; ++p) {
        const long long nch = (len[p] + kPrefetchChunk - 1) / kPrefetchChunk;
        for (long long j = ((long long)blockIdx.x - chunk % G + G) % G; j < nch; j += G) {
          const long long o = j * kPrefetchChunk;
          if (pos + o >= a.budget) break;
          const long long b = len[p] - o < kPrefetchChunk ? len[p] - o : kPrefetchChunk;
          l2_prefetch_bulk(ptr[p] + o, (uint32_t)b);
        }
        chunk += nch;
        pos += len[p];
      }
    }
  }
}

// A library-owned side stream per device, forked from and joined back into the
// caller's stream with events (also inside stream capture).
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

static SideStream* side_stream() {
  static SideStream s[64];
  static std::mutex mu;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  SideStream& ss = s[dev];
  if (!ss.stream) {
    if (cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      ss = SideStream();
      return nullptr;
    }
  }
  return &ss;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Fork: the prefetch kernel runs on the side stream after everything the
// caller's stream has enqueued so far (the gate's indices).  Returns the side
// stream to join later, or nullptr when nothing was launched (the layout does
// not allow 16-byte bulk requests, or the budget is 0).
cudaStream_t launch_weight_prefetch(const dsv4_moe_layer* L, const int64_t* indices, int n_idx,
                                    long long budget, int num_sms, cudaStream_t st) {
  if (budget <= 0 || n_idx <= 0 || L->n_routed > kPrefetchMaxExperts || !L->arena || !L->arena_sf ||
      !L->expert_slot)
    return nullptr;
  const long long H = L->hidden, I = L->inter, sc = I * H / 32;
  PrefetchArgs a{};
  a.indices = indices;
  a.n_idx = n_idx;
  a.n_routed = L->n_routed;
  a.expert_slot = L->expert_slot;
  a.n_slots = L->n_slots;
  a.arena = L->arena;
  a.slot_stride = L->slot_stride;
  a.arena_sf = L->arena_sf;
  a.sf_slot_stride = L->sf_slot_stride;
  a.w1_off = 3 * sc;
  a.w2_off = 3 * sc + I * H / 2;
  a.w3_off = 3 * sc + I * H;
  a.wg_bytes = I * H / 2;
  a.sf_bytes = sc;
  a.shared_w1 = L->shared_w1;
  a.shared_w3 = L->shared_w3;
  a.shared_w2 = L->shared_w2;
  a.shared_sf = L->shared_sf;
  a.shared_bytes = I * H;
  a.budget = budget;
  // every request stays inside a slot's block / atoms, 16-byte aligned
  if (!aligned16(L->arena) || !aligned16(L->arena_sf) || (L->slot_stride & 15) ||
      (L->sf_slot_stride & 15) || (sc & 15) || L->slot_stride < 3 * sc + 3 * I * H / 2 ||
      L->sf_slot_stride < 3 * sc || L->n_slots <= 0)
    return nullptr;
  if (L->shared_w1 && (!aligned16(L->shared_w1) || !aligned16(L->shared_w2) ||
                       !aligned16(L->shared_w3) || !aligned16(L->shared_sf)))
    return nullptr;
  SideStream* ss = side_stream();
  if (!ss) return nullptr;
  if (cudaEventRecord(ss->fork, st) != cudaSuccess ||
      cudaStreamWaitEvent(ss->stream, ss->fork, 0) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  launch_k(weight_prefetch_kernel, num_sms, 128, 0, ss->stream, a);
  cudaGetLastError();
  return ss->stream;
}

// Join: the caller's stream waits for the side stream (a stream capture must
// not end with it unjoined; the prefetch kernel is long finished by then).
int join_side_stream(cudaStream_t side, cudaStream_t st) {
  if (!side) return DSV4_OK;
  SideStream* ss = side_stream();
  if (!ss || ss->stream != side) return DSV4_ERR_CUDA;
  if (cudaEventRecord(ss->join, side) != cudaSuccess || cudaStreamWaitEvent(st, ss->join, 0) != cudaSuccess)
    return DSV4_ERR_CUDA;
  return DSV4_OK;
}

}  // namespace dsv4
