// Cycles per 128-wide k tile of the grouped expert GEMM's MMA loop, measured
// on every SM at once with operands resident in shared memory (zero-filled;
// no global traffic): block-scaled tcgen05.mma (kind::mxf8f6f4, e4m3 x e2m1)
// by N, the cost of the loop's mbarrier poll / fence / commit, and of the
// scale-factor copies (tcgen05.cp) by shape.  These figures bound what the
// expert GEMM's single MMA-issuing thread can reach once its data is staged.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 --expt-relaxed-constexpr \
//        -I include -I deepseek-v4-flash-dgx-spark_b200/csrc \
//        deepseek-v4-flash-dgx-spark_b200/microbench/tcgen05_issue.cu -o tcgen05_issue -lcuda
//
// One CTA of 128 threads per SM; warp 1 allocates 512 TMEM columns and one of
// its threads issues.  Every descriptor stays inside the 56 KB of shared
// memory the CTA allocates; every wait is bounded (common.cuh).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "common.cuh"

using namespace dsv4;

namespace {

__device__ __forceinline__ void cp_128x256b(uint32_t t, uint64_t d) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(t), "l"(d) : "memory");
}

// no-swizzle K-major shared-memory descriptor with explicit LBO / SBO (bytes)
__device__ __forceinline__ uint64_t sdesc_ns(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

constexpr int kA = 16384, kB = 32768, kSF = 8192;  // smem: A | B | scale blocks
constexpr int kSmem = 1024 + kA + kB + kSF;

// EXTRA: 0 none; 1 ready mbarrier poll + fence + commit per k tile; 2 = 1 + two
// 32x128b.warpx4 copies per k tile; 3 = 2 + one more per 4 k tiles (the expert
// GEMM's copy pattern); 4 = 1 + one 128x256b copy per k tile.
template <int N, int EXTRA>
__global__ void __launch_bounds__(128, 1) kloop(unsigned long long* out, int iters) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
  for (int i = threadIdx.x; i < (kA + kB + kSF) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(sm)[i] = make_uint4(0, 0, 0, 0);
  __shared__ uint32_t tslot;
  __shared__ uint64_t bar, ready, sink;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_init(&ready, 1);
    mbar_init(&sink, 1);
    fence_barrier_init();
  }
  fence_proxy_async_shared();
  if (warp == 1) {
    tmem_alloc(&tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (threadIdx.x == 0) mbar_arrive(&ready);  // phase 0 of `ready` completes
  __syncthreads();
  if (warp == 1 && lane == 0) {
    const uint64_t ad = sdesc_k_sw128(smem_u32(sm));
    const uint64_t bd = sdesc_k_sw128(smem_u32(sm + kA));
    const uint32_t sf = smem_u32(sm + kA + kB);
    const uint32_t sfa = tmem + 256, sfb = tmem + 264;
    tc_cp_sf(sfa, sdesc_sf(sf));
    tc_cp_sf(sfb, sdesc_sf(sf + 512));
    tc_cp_sf(sfb + 4, sdesc_sf(sf + 1024));
    tc_commit(&bar);
    bool ok = mbar_wait(&bar, 0, 1);
    tc_fence_after();
    const uint64_t g0 = globaltimer();
    const unsigned long long c0 = clock64();
    for (int i = 0; i < iters && ok; ++i) {
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        if (EXTRA >= 1) {
          ok = mbar_wait(&ready, 0, 1);
          tc_fence_after();
        }
        if (EXTRA == 2 || EXTRA == 3) {
          tc_cp_sf(tmem + 320 + 8 * kt, sdesc_sf(sf + 2048));
          tc_cp_sf(tmem + 324 + 8 * kt, sdesc_sf(sf + 2560));
        }
        if (EXTRA == 3 && kt == 0) tc_cp_sf(tmem + 360, sdesc_sf(sf + 3072));
        if (EXTRA == 4) cp_128x256b(tmem + 320 + 8 * kt, sdesc_ns(sf + 2048, 2048, 128));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          constexpr uint32_t id0 = idesc_mxf8f6f4(0u, 5u, N, 0, 0);
          tc_mma_mxf8f6f4(tmem, ad + 2 * kk, bd + 2 * kk, id0 | ((uint32_t)kk << 4), sfa, sfb, 1u);
        }
        if (EXTRA >= 1) tc_commit(&sink);
      }
    }
    tc_commit(&bar);
    ok = mbar_wait(&bar, 1, 1) && ok;
    const unsigned long long c1 = clock64();
    const uint64_t g1 = globaltimer();
    out[blockIdx.x * 2] = ok ? c1 - c0 : 0;
    out[blockIdx.x * 2 + 1] = g1 - g0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int N, int EXTRA>
void run(const char* name, unsigned long long* d, int grid) {
  cudaFuncSetAttribute(kloop<N, EXTRA>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  const int iters = 1000;
  kloop<N, EXTRA><<<grid, 128, kSmem>>>(d, 20);
  kloop<N, EXTRA><<<grid, 128, kSmem>>>(d, iters);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    printf("%s: CUDA error\n", name);
    exit(1);
  }
  std::vector<unsigned long long> h(grid * 2);
  cudaMemcpy(h.data(), d, grid * 2 * 8, cudaMemcpyDeviceToHost);
  std::vector<double> cyc, mhz;
  for (int i = 0; i < grid; ++i) {
    if (h[2 * i] == 0) {
      printf("%s: a wait timed out\n", name);
      exit(1);
    }
    cyc.push_back((double)h[2 * i]);
    mhz.push_back((double)h[2 * i] / (double)h[2 * i + 1] * 1000.0);
  }
  std::sort(cyc.begin(), cyc.end());
  std::sort(mhz.begin(), mhz.end());
  const double per_kt = cyc[cyc.size() / 2] / (iters * 4.0);
  const double flop = 2.0 * 128 * N * 128;  // one k tile: 4 MMAs of K = 32
  printf("%-48s %7.1f cycles/k-tile  %6.0f FLOP/clk/SM  %5.0f MHz  %6.0f TFLOP/s on %d SMs\n", name,
         per_kt, flop / per_kt, mhz[mhz.size() / 2],
         flop / per_kt * mhz[mhz.size() / 2] * 1e6 * grid / 1e12, grid);
}

}  // namespace

int main() {
  int nsm = 0;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, 0);
  unsigned long long* d = nullptr;
  cudaMalloc(&d, nsm * 2 * 8);
  run<256, 0>("4 MMA N=256", d, nsm);
  run<128, 0>("4 MMA N=128", d, nsm);
  run<64, 0>("4 MMA N=64", d, nsm);
  run<32, 0>("4 MMA N=32", d, nsm);
  run<256, 1>("N=256 + mbarrier poll, fence, commit", d, nsm);
  run<256, 2>("N=256 + 2 cp 32x128b.warpx4 per k tile", d, nsm);
  run<256, 3>("N=256 + expert GEMM copy pattern (9 per 4 k tiles)", d, nsm);
  run<256, 4>("N=256 + 1 cp 128x256b per k tile", d, nsm);
  cudaFree(d);
  return 0;
}
