// Expert materializer: packed-slab blocks -> expert arena slots on the device.
//
// Replaces LazyRoutedExpert.materialize (spark_runtime/lazy_official_runtime.py:
// 761-917) and the per-tensor cudaMemcpyAsync plan of ExpertCopyPlan::
// read_into_and_copy_cuda (spark_runtime/native/native_packed_loader.cpp:
// 122-174,281-316).  A slot keeps the packed block's bytes unchanged (tensor
// order w1.scale, w2.scale, w3.scale, w1.weight, w2.weight, w3.weight,
// scripts/build_packed_expert_layout.py:76-86), so the arena's parameter
// views are bit-exact copies of the checkpoint tensors.  The same pass also
// writes the derived tensor-memory scale atoms the grouped GEMM reads and,
// optionally, an exact e2m1 x ue8m0 -> bf16 decode of the three weights.
#include "kernels.cuh"

namespace dsv4 {

// 16-byte vector copy of n blocks, block i from slab + src_off[i] to
// arena + dst_slot[i] * slot_stride.  HBM-bound: grid-stride over 16-byte
// chunks of the concatenated blocks.  A block whose source offset is not
// 16-byte aligned is skipped and latches DSV4_DEVERR_MISALIGNED.
__global__ void __launch_bounds__(256) materialize_copy_kernel(
    const uint8_t* __restrict__ slab, const long long* __restrict__ src_off,
    const int* __restrict__ dst_slot, int n, long long block_bytes, uint8_t* __restrict__ arena,
    long long slot_stride) {
  const long long chunks_per_block = block_bytes >> 4;
  const long long total = chunks_per_block * n;
  for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < total;
       c += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(c / chunks_per_block);
    const long long o = (c - (long long)b * chunks_per_block) << 4;
    const long long so = src_off[b];
    if (so & 15) {
      if (o == 0) record_error(DSV4_DEVERR_MISALIGNED);
      continue;
    }
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(slab + so + o));
    __stcs(reinterpret_cast<uint4*>(arena + (long long)dst_slot[b] * slot_stride + o), v);
  }
}

// Scale atoms of the three fp4 weights of n experts.  Source: the raw [rows,
// K/32] ue8m0 matrices at src + src_off[i] (or dst_slot[i] * src_stride when
// src_off is NULL: the arena itself) + {w1, w2, w3 scale offsets};
// destination: sf + dst_slot[i] * sf_slot_stride + {w1, w3, w2 atom offsets}.
// One thread writes one 16-byte atom row (m0): 4 rows x 4 scales.
__global__ void __launch_bounds__(256) build_sf_fp4_kernel(
    const uint8_t* __restrict__ src, const long long* __restrict__ src_off, long long src_stride,
    const int* __restrict__ dst_slot, int n, int hidden, int inter, uint8_t* __restrict__ sf,
    long long sf_slot_stride) {
  const long long w13_bytes = (long long)inter * hidden / 32;  // per weight
  // atoms: w1 -> (inter/128) x (hidden/128); w3 same; w2 -> (hidden/128) x (inter/128)
  const long long rows_per_expert = 3 * w13_bytes / 16;  // 16-byte atom rows
  const long long total = rows_per_expert * n;
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < total;
       r += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(r / rows_per_expert);
    long long ar = r - (long long)b * rows_per_expert;  // atom-row index within the expert
    const int wsel = (int)(ar / (w13_bytes / 16));      // 0 = w1, 1 = w3, 2 = w2
    ar -= (long long)wsel * (w13_bytes / 16);
    const int K = wsel == 2 ? inter : hidden;
    const int KT = K / 128;
    const long long atom = ar >> 5;  // 32 rows per atom
    const int m0 = (int)(ar & 31);
    const int nb = (int)(atom / KT), kt = (int)(atom % KT);
    // raw scale offsets inside the packed block: w1.scale, w2.scale, w3.scale
    const long long raw_off = wsel == 0 ? 0 : (wsel == 1 ? 2 * w13_bytes : w13_bytes);
    const long long base = src_off ? src_off[b] : (long long)dst_slot[b] * src_stride;
    const uint8_t* s = src + base + raw_off;
    const int ks = K / 32;
    uint32_t words[4];
#pragma unroll
    for (int m1 = 0; m1 < 4; ++m1) {
      const int row = nb * 128 + m1 * 32 + m0;
      words[m1] = *reinterpret_cast<const uint32_t*>(s + (long long)row * ks + kt * 4);
    }
    *reinterpret_cast<uint4*>(sf + (long long)dst_slot[b] * sf_slot_stride +
                              (long long)wsel * w13_bytes + (atom << 9) + (m0 << 4)) =
        make_uint4(words[0], words[1], words[2], words[3]);
  }
}

// Scale atoms of one fp8 weight [rows, K] with [rows/128, K/128] ue8m0 block
// scales: every per-32 scale of row r is its block's scale.
__global__ void __launch_bounds__(256) build_sf_fp8_kernel(const uint8_t* __restrict__ scale,
                                                           int rows, int K,
                                                           uint8_t* __restrict__ atoms) {
  const int KT = K / 128;
  const long long total = (long long)(rows / 128) * KT * 32;  // atom rows
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < total;
       r += (long long)gridDim.x * blockDim.x) {
    const long long atom = r >> 5;
    const int nb = (int)(atom / KT), kt = (int)(atom % KT);
    const uint32_t w = (uint32_t)scale[(long long)nb * KT + kt] * 0x01010101u;
    *reinterpret_cast<uint4*>(atoms + (r << 4)) = make_uint4(w, w, w, w);
  }
}

constexpr int kDecodeWordsPerThread = 8;

// bf16 bits of the two e2m1 codes of byte v (low nibble first) at scale 1.
__device__ __forceinline__ uint32_t e2m1_pair_bf16_bits(uint32_t v) {
  uint32_t out = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t c = (v >> (4 * h)) & 0xF, mag = c & 7, e2 = mag >> 1;
    // 0.5 = 2^-1 (exponent field 126); otherwise (1 + m/2) * 2^(e2-1)
    const uint32_t bits = mag == 0 ? 0u : (e2 == 0 ? (126u << 7) : (((126u + e2) << 7) | ((mag & 1) << 6)));
    out |= (bits | ((c & 8) << 12)) << (16 * h);
  }
  return out;
}

// 8 e2m1 codes (one 32-bit word) at ue8m0 scale byte s -> 8 bf16 (16 bytes).
__device__ __forceinline__ uint4 decode_word(uint32_t cw, int s, const uint32_t* lut) {
  uint32_t pk[4];
  if (s >= 16 && s <= 239) {
    const uint32_t d = (uint32_t)((s - 127) << 7) & 0xFFFFu;
    const uint32_t dpair = d | (d << 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t x = lut[(cw >> (8 * i)) & 0xFF];
      const uint32_t nz = __vcmpne2(x & 0x7FFF7FFFu, 0u);  // +-0 keeps its exponent
      pk[i] = __vadd2(x, dpair & nz);
    }
  } else {
    const float sc = exp2i(s - 127);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t c = (cw >> (8 * i + 4 * h)) & 0xF;
        // e2m1: exponent bits 2..1, mantissa bit 0; subnormal when exponent = 0
        const uint32_t ex = (c >> 1) & 3, m = c & 1;
        const float mag = ex == 0 ? 0.5f * (float)m : exp2i((int)ex - 1) * (1.0f + 0.5f * (float)m);
        v[h] = (c & 8) ? -mag * sc : mag * sc;
      }
      const __nv_bfloat162 p = __floats2bfloat162_rn(v[0], v[1]);
      pk[i] = *reinterpret_cast<const uint32_t*>(&p);
    }
  }
  return make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// Exact bf16 decode of the three fp4 weights of n experts:
// out + dst_slot[i] * out_slot_stride + {w1, w2, w3} as [rows, K] bf16.
// blockIdx.y = expert * 3 + weight (packed order w1, w2, w3).  One thread
// decodes one 32-bit code word (8 codes, a quarter of a ue8m0 scale group)
// into 16 bytes of bf16: a warp reads 128 contiguous bytes and writes 512, so
// every store instruction fills whole sectors; each thread keeps
// kDecodeWordsPerThread words in flight.  e2m1 x 2^(s-127) is exact in bf16;
// for 16 <= s <= 239 every nonzero result is a normal bf16, so the product is
// the scale-1 bit pattern (a 256-entry byte -> bf16x2 table) with s - 127
// added to both exponent fields; other scale bytes take the float path.
__global__ void __launch_bounds__(256) decode_bf16_kernel(
    const uint8_t* __restrict__ src, const long long* __restrict__ src_off,
    const int* __restrict__ dst_slot, int hidden, int inter, __nv_bfloat16* __restrict__ out,
    long long out_slot_stride) {
  __shared__ uint32_t lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = e2m1_pair_bf16_bits(i);
  __syncthreads();
  const int b = blockIdx.y / 3, wsel = blockIdx.y % 3;
  const long long w_elems = (long long)inter * hidden;
  const long long groups = w_elems / 32;  // scale groups of one weight (= its scale bytes)
  const long long words = w_elems / 8;    // 32-bit code words of one weight
  if (src_off[b] & 15) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_error(DSV4_DEVERR_MISALIGNED);
    return;
  }
  const uint8_t* blk = src + src_off[b];
  const uint8_t* scale = blk + (long long)wsel * groups;
  const uint32_t* codes = reinterpret_cast<const uint32_t*>(blk + 3 * groups + (long long)wsel * (w_elems / 2));
  uint4* o = reinterpret_cast<uint4*>(out + (long long)dst_slot[b] * out_slot_stride + (long long)wsel * w_elems);
  const long long w0 = (long long)blockIdx.x * kDecodeWordsPerThread * blockDim.x + threadIdx.x;
  uint32_t cw[kDecodeWordsPerThread];
  int sc[kDecodeWordsPerThread];
#pragma unroll
  for (int u = 0; u < kDecodeWordsPerThread; ++u) {
    const long long w = w0 + (long long)u * blockDim.x;
    cw[u] = 0;
    sc[u] = 127;
    if (w < words) {
      cw[u] = __ldcs(codes + w);
      sc[u] = scale[w >> 2];
    }
  }
#pragma unroll
  for (int u = 0; u < kDecodeWordsPerThread; ++u) {
    const long long w = w0 + (long long)u * blockDim.x;
    if (w < words) __stcs(o + w, decode_word(cw[u], sc[u], lut));
  }
}

static int grid_for(long long work, int num_sms) {
  long long g = (work + 255) / 256;
  const long long cap = (long long)num_sms * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

int launch_materialize(const uint8_t* slab, const long long* src_off, const int* dst_slot, int n,
                       long long block_bytes, uint8_t* arena, long long slot_stride, int hidden,
                       int inter, uint8_t* sf, long long sf_slot_stride, void* bf16_out,
                       long long bf16_slot_stride, int num_sms, cudaStream_t st) {
  if (n <= 0) return DSV4_OK;
  if (arena) {
    count_launch();
    materialize_copy_kernel<<<grid_for((block_bytes >> 4) * n, num_sms), 256, 0, st>>>(
        slab, src_off, dst_slot, n, block_bytes, arena, slot_stride);
  }
  if (sf) {
    const long long rows = 3LL * inter * hidden / 32 / 16 * n;
    count_launch();
    build_sf_fp4_kernel<<<grid_for(rows, num_sms), 256, 0, st>>>(slab, src_off, 0, dst_slot, n,
                                                                 hidden, inter, sf,
                                                                 sf_slot_stride);
  }
  if (bf16_out) {
    if (3LL * n > 65535) return DSV4_ERR_UNSUPPORTED;
    const long long per_cta = 256LL * kDecodeWordsPerThread;
    const dim3 grid((unsigned)(((long long)inter * hidden / 8 + per_cta - 1) / per_cta), 3 * n);
    count_launch();
    decode_bf16_kernel<<<grid, 256, 0, st>>>(slab, src_off, dst_slot, hidden, inter,
                                             static_cast<__nv_bfloat16*>(bf16_out),
                                             bf16_slot_stride);
  }
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_build_sf_fp4_arena(const uint8_t* arena, long long slot_stride, const int* slots,
                              int n, int hidden, int inter, uint8_t* sf, long long sf_slot_stride,
                              int num_sms, cudaStream_t st) {
  if (n <= 0) return DSV4_OK;
  const long long rows = 3LL * inter * hidden / 32 / 16 * n;
  count_launch();
  build_sf_fp4_kernel<<<grid_for(rows, num_sms), 256, 0, st>>>(arena, nullptr, slot_stride, slots,
                                                               n, hidden, inter, sf,
                                                               sf_slot_stride);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int launch_build_sf_fp8(const uint8_t* scale, int rows, int K, uint8_t* atoms, int num_sms,
                        cudaStream_t st) {
  const long long work = (long long)(rows / 128) * (K / 128) * 32;
  count_launch();
  build_sf_fp8_kernel<<<grid_for(work, num_sms), 256, 0, st>>>(scale, rows, K, atoms);
  return cudaGetLastError() == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

}  // namespace dsv4
