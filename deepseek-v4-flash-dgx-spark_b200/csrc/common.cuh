// Shared device helpers for the dsv4moe sm_100a kernels: error reporting,
// bounded mbarrier waits, TMA / bulk copies and tcgen05 (TMEM + UMMA) wrappers.
//
// Every wait in this library is bounded: a wait that does not complete within
// kWaitTimeoutNs records an error code in g_dsv4_device_error and returns
// false, and the caller unwinds instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "dsv4moe.h"

namespace dsv4 {

// First device-side error of the process (0 = none).  Read and cleared by
// dsv4_device_error().  The library is one CUDA translation unit
// (dsv4moe.cu), so this is the single definition.
__device__ int g_dsv4_device_error = 0;

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

// Kernels enqueued by the library (host side; a captured graph counts each of
// its kernels once), read by dsv4_kernel_launches().
inline std::atomic<long long> g_kernel_launches{0};
inline void count_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }

// The one launch point of the library's kernels (counted for
// dsv4_kernel_launches()).
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  count_launch();
  kernel<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
}

// Raise a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device.  The attribute belongs to the device, so a process that
// drives several GPUs must set it on each of them; the largest size set so
// far is remembered per (kernel, device), and a larger request sets it again.
inline int ensure_smem_attr(const void* kernel, int bytes) {
  constexpr int kMaxDev = 64, kMaxKernels = 64;
  static std::mutex mu;
  static const void* fns[kMaxKernels];
  static int set_to[kMaxKernels][kMaxDev];  // bytes set on each device (0: never)
  static int n_fns = 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return DSV4_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  int i = 0;
  while (i < n_fns && fns[i] != kernel) ++i;
  if (i < n_fns && set_to[i][dev] >= bytes) return DSV4_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return DSV4_ERR_CUDA;
  }
  if (i == n_fns) {
    if (n_fns == kMaxKernels) return DSV4_OK;  // set, just not remembered
    fns[n_fns++] = kernel;
  }
  set_to[i][dev] = bytes;
  return DSV4_OK;
}

__device__ __forceinline__ void record_error(int code) {
  atomicCAS(&g_dsv4_device_error, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with cluster-scope acquire: for barriers another CTA of the
// cluster arrives on with release.cluster.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int err_code) {
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      record_error(err_code);
      return false;
    }
  }
}

// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int err_code) {
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      record_error(err_code);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA / bulk copies (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Pull the 128-byte line holding p into L2 (load/store unit path).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}

// Untiled bulk copy global -> shared; both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation tensor core
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive on an mbarrier once every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row groups of
// 128-byte rows (SBO = 1024 B), LBO unused (1), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Descriptor of a no-swizzle K-major 32-row x 16-byte block (tcgen05.cp source).
__device__ __forceinline__ uint64_t sdesc_sf(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)0 << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Copy a 32-lane x 128-bit scale block from shared memory into 4 TMEM columns,
// replicated into all four 32-lane sub-partitions.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// D(tmem) (+)= A(smem) x B(smem)^T with per-32 ue8m0 block scales from TMEM.
__device__ __forceinline__ void tc_mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t sfa_tmem,
                                                uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::
          "r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// D(tmem) (+)= A(smem) x B(smem)^T, both e2m1 packed two per byte (K = 64 per
// instruction, 32 bytes of each row), two ue8m0 scales per row per instruction
// (scale_vec::2X: the scale-factor id 0 or 2 picks bytes {id, id+1} of the
// 32-bit TMEM word, the first for k 0..31 of the instruction).
__device__ __forceinline__ void tc_mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::
          "r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Instruction descriptor for kind::mxf4: A and B e2m1 (format 1 in this kind),
// K-major, fp32 accumulate, ue8m0 scales (bit 23), dense K = 64 (bit 31 = 0),
// M = 128; sf ids 0 or 2 (bits 29-30 for A, 4-5 for B).
__host__ __device__ constexpr uint32_t idesc_mxf4(uint32_t n, uint32_t a_sf_id, uint32_t b_sf_id) {
  return (b_sf_id << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
         (a_sf_id << 29);
}

// D(tmem) (+)= A(smem) x B(smem)^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2) for cta_group::2 tensor-core work.  Every load of
// a pair fills the issuing CTA's own shared memory; only its completion is
// reported to the leader CTA's mbarrier.  The one cluster-wide broadcast is
// the MMA completion signal (tcgen05.commit to both CTAs' barriers).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the variable at local shared address `p` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}

// All threads of both CTAs of the cluster (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// Arrive once on an mbarrier given by its shared::cluster address (may be the peer CTA's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Tile loads into this CTA's shared memory whose completion is counted on the
// mbarrier at `bar_cluster` (a shared::cluster address in either CTA of the pair).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m,
                                                 uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m,
                                                 uint32_t bar_cluster, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Arrive on the mbarrier at the same shared offset in every CTA of `cta_mask`
// once every tcgen05 op this thread issued for the pair is done.
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Scale block copy for a pair: each CTA's shared memory to its own TMEM.
__device__ __forceinline__ void tc_cp_sf_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// D (+)= A x B^T for a CTA pair (M = 256: 128 rows per CTA; B's N rows split
// in halves over the two CTAs' shared memory).
__device__ __forceinline__ void tc_mma_mxf8f6f4_pair(uint32_t d_tmem, uint64_t adesc,
                                                     uint64_t bdesc, uint32_t idesc,
                                                     uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::
          "r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Load 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%"
      "15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Issue a load of 32 consecutive 32-bit columns of this thread's TMEM lane
// without waiting; the registers are valid only after tmem_wait_ld2().
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Wait for every TMEM load this thread issued.  The two register sets pass
// through the wait as read-write operands, so no use of them can be
// scheduled ahead of it.
__device__ __forceinline__ void tmem_wait_ld2(uint32_t (&a)[32], uint32_t (&b)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]), "+r"(a[16]), "+r"(a[17]), "+r"(a[18]), "+r"(a[19]), "+r"(a[20]), "+r"(a[21]), "+r"(a[22]), "+r"(a[23]), "+r"(a[24]), "+r"(a[25]), "+r"(a[26]), "+r"(a[27]), "+r"(a[28]), "+r"(a[29]), "+r"(a[30]), "+r"(a[31])
               :
               : "memory");
  asm volatile(""
               : "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15]), "+r"(b[16]), "+r"(b[17]), "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]), "+r"(b[22]), "+r"(b[23]), "+r"(b[24]), "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]), "+r"(b[29]), "+r"(b[30]), "+r"(b[31]));
}

// Instruction descriptor for kind::mxf8f6f4 block-scaled MMA, K-major A and B,
// fp32 accumulate, ue8m0 scales, M = 128 (256 for a CTA pair).
//   a_fmt / b_fmt: 0 = e4m3, 5 = e2m1.  sf ids select the byte of the 32-bit
//   TMEM scale word (the 32-wide K block inside a 128-wide K tile).
__host__ __device__ constexpr uint32_t idesc_mxf8f6f4(uint32_t a_fmt, uint32_t b_fmt, uint32_t n,
                                                      uint32_t a_sf_id, uint32_t b_sf_id,
                                                      uint32_t m = 128) {
  return (b_sf_id << 4) | (a_fmt << 7) | (b_fmt << 10) | ((n >> 3) << 17) | (1u << 23) |
         ((m >> 4) << 24) | (a_sf_id << 29);
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t n) {
  return (1u << 4) /*D fp32*/ | (1u << 7) /*A bf16*/ | (1u << 10) /*B bf16*/ | ((n >> 3) << 17) |
         ((128u >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Number formats
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// fp32 -> e4m3fn code, round to nearest even, saturate to +-448.
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

// Four fp32 -> e4m3fn codes (RNE, saturating), a in the low byte.  One
// cvt.rn.satfinite.e4m3x2.f32 converts a pair: its first source goes to the
// upper byte.
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// ceil(log2(v)) for a positive normal fp32 v, exact (from the bit pattern).
__device__ __forceinline__ int ceil_log2_exact(float v) {
  const uint32_t u = __float_as_uint(v);
  const int e = static_cast<int>((u >> 23) & 0xFF) - 127;
  return (u & 0x7FFFFF) ? e + 1 : e;
}

// Power-of-two per-128 activation scale exponent (ue8m0): amax -> e with
// 2^e = 2^ceil(log2(max(amax, 1e-4) * (1/448))).
__device__ __forceinline__ int act_scale_exp(float amax) {
  amax = fmaxf(amax, 1e-4f);
  const float v = __fmul_rn(amax, 1.0f / 448.0f);
  return ceil_log2_exact(v);
}

__device__ __forceinline__ float exp2i(int e) {  // exact 2^e for e in [-126, 127]
  return __int_as_float((e + 127) << 23);
}

// FP4 activations (the official fp4_act_quant(x, 32)): per block of 32 values
// amax = max(|x|, 1e-4), s = 2^ceil(log2(amax * fp32(1/6))), codes =
// e2m1(x / s) rounded to nearest even and saturated (cvt.rn.satfinite), two
// per byte with element 2i in the low nibble.  Returns s's exponent; `packed`
// gets the 16 code bytes of the 32 values v (already in fp32).
__device__ __forceinline__ int fp4_block_quant(const float (&v)[32], uint4& packed) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, 1e-4f);
  const int e = ceil_log2_exact(__fmul_rn(amax, 1.0f / 6.0f));
  const float inv = exp2i(-e);
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = 8 * j + 2 * b;
      const uint32_t byte = __nv_cvt_float2_to_fp4x2(make_float2(v[i] * inv, v[i + 1] * inv), __NV_E2M1,
                                                     cudaRoundNearest);
      word |= (byte & 0xFFu) << (8 * b);
    }
    w[j] = word;
  }
  packed = make_uint4(w[0], w[1], w[2], w[3]);
  return e;
}

// 32 bf16 values (64 bytes, 16-byte aligned) -> fp32
__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 r = *reinterpret_cast<const uint4*>(src + 8 * q);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[8 * q + i] = __bfloat162float(b[i]);
  }
}

}  // namespace dsv4
