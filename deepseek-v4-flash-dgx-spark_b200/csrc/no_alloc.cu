// Allocation-free variant of the single-expert forward.
//
// Some callers cannot hand this library a workspace and may not let it call
// cudaMalloc either: a host runtime that owns every device allocation and only
// passes in input and output buffers, a serving loop that must not touch the
// allocator once it is running (an allocation can synchronise the device or
// fail under memory pressure at the worst moment), or a plugin host that
// forbids allocation inside its operator calls.  dsv4_expert_forward_static
// serves them: it takes only the inputs and the output, and its scratch lives
// in a fixed array in device memory that belongs to this library.
//
// The array is a file-scope __device__ variable, so every GPU on which the
// library's kernels are loaded holds kStaticScratchBytes of it until the
// process exits.  Its contents persist from call to call, and all calls share
// it: two calls that can run at the same time on the GPU (different streams,
// or different host threads without ordering) race on it and give undefined
// results.  Each call writes every part of the scratch its output depends on
// before reading it (the routing plan, the quantized activations and their
// scales, the intermediate activations); bytes left over from an earlier call
// reach only accumulator lanes and padding rows that are never stored, so
// nothing needs clearing.
#include <mutex>

#include "kernels.cuh"

namespace dsv4 {

constexpr size_t kStaticScratchBytes = 4u << 20;  // 4 MiB

// Device storage of the scratch.  In host code this name is only a handle for
// the runtime; the kernels get its device address from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
static void* g_static_scratch_ptr[kMaxDevices];
static std::mutex g_static_scratch_mu;

// Device address of the scratch on the current device, looked up once per
// device (the first call on a device does the lookup).  The address belongs
// to the device's primary context: after cudaDeviceReset the module is loaded
// again and the cached address is stale, so the entry point must not be used
// in a process that resets a device it has already called it on.
static int static_scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSV4_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (!g_static_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return DSV4_ERR_CUDA;
    }
    g_static_scratch_ptr[dev] = p;
  }
  *out = g_static_scratch_ptr[dev];
  return DSV4_OK;
}

}  // namespace dsv4

extern "C" long long dsv4_expert_static_scratch_bytes(void) {
  return static_cast<long long>(dsv4::kStaticScratchBytes);
}

extern "C" int dsv4_expert_forward_static(const dsv4_moe_layer* L, int expert, const void* x, int T,
                                          const float* row_weights, void* y, void* stream) {
  using namespace dsv4;
  if (!L || !x || !y || T < 0) return DSV4_ERR_ARG;
  const long long need = dsv4_expert_workspace_bytes(L, T);
  if (need < 0) return DSV4_ERR_ARG;
  if (need > static_cast<long long>(kStaticScratchBytes)) return DSV4_ERR_WORKSPACE;
  if (T == 0) return DSV4_OK;
  // Run on the device that owns the output when it is plain device memory;
  // managed or host-registered outputs run on the current device, as in
  // dsv4_expert_forward.
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, y) == cudaSuccess && a.type == cudaMemoryTypeDevice) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != a.device) {
      if (cudaSetDevice(a.device) != cudaSuccess) return DSV4_ERR_CUDA;
    }
  }
  cudaGetLastError();
  void* scratch = nullptr;
  int rc = static_scratch_address(&scratch);
  if (rc) return rc;
  return dsv4_expert_forward(L, expert, x, T, row_weights, y, scratch,
                             static_cast<long long>(kStaticScratchBytes), stream);
}
