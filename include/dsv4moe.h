/*
 * dsv4moe — B200 (sm_100a) routed-expert MoE hot path of DeepSeek-V4-Flash.
 *
 * C ABI of libdsv4moe.so.  Plain pointers and sizes only; every function
 * returns DSV4_OK (0) or a negative DSV4_ERR_* code and never aborts.  Device
 * pointers are CUDA global memory of the current device; `stream` is a
 * cudaStream_t (NULL = legacy default stream).  Kernels are enqueued
 * asynchronously; errors raised inside a kernel (bounded waits that expired,
 * out-of-range expert ids) are latched in a device flag read by
 * dsv4_device_error().
 *
 * Reference interfaces replaced (paths inside bigs/deepseek-v4-flash-dgx-spark):
 *   spark_runtime/lazy_official_runtime.py:946-1002   LazyMoE / official Gate, Expert
 *   spark_runtime/lazy_official_runtime.py:49-338     PackedExpertStore
 *   spark_runtime/lazy_official_runtime.py:641-667    ExpertArena
 *   spark_runtime/native/native_packed_loader.cpp:1-359  read_into, copy plans
 */
#ifndef DSV4MOE_H_
#define DSV4MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSV4_API __attribute__((visibility("default")))
#else
#define DSV4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define DSV4_OK 0
#define DSV4_ERR_ARG (-1)         /* invalid argument (TORCH_CHECK failures in the reference) */
#define DSV4_ERR_CUDA (-2)        /* CUDA runtime / launch error */
#define DSV4_ERR_UNSUPPORTED (-3) /* shape or option this build does not implement */
#define DSV4_ERR_IO (-4)          /* pread failed (errno kept in *err_no) */
#define DSV4_ERR_SHORT_READ (-5)  /* "short packed expert read" */
#define DSV4_ERR_BOUNDS (-6)      /* "source slice exceeds storage tensor" */
#define DSV4_ERR_SIZE (-7)        /* "target size does not match expert copy plan" */
#define DSV4_ERR_WORKSPACE (-8)   /* workspace smaller than dsv4_moe_workspace_bytes() */

/* device-side error codes latched by kernels (read with dsv4_device_error) */
#define DSV4_DEVERR_TIMEOUT_PRODUCER 101
#define DSV4_DEVERR_TIMEOUT_MMA 102
#define DSV4_DEVERR_TIMEOUT_EPILOGUE 103
#define DSV4_DEVERR_BAD_INDEX 104
#define DSV4_DEVERR_PLAN_OVERFLOW 105
#define DSV4_DEVERR_MISALIGNED 106  /* a materializer source offset is not 16-byte aligned */
#define DSV4_DEVERR_TIMEOUT_PEER 107  /* a peer rank's exchange flag did not arrive within 2 s */

DSV4_API int dsv4_version(void);
/* Number of kernels the library has enqueued in this process (every launch
 * counts once, including launches captured into a CUDA graph; graph replays
 * do not pass through the library and are not counted).  No counterpart in
 * the reference: it backs the launch count a benchmark reports. */
DSV4_API long long dsv4_kernel_launches(void);
DSV4_API const char* dsv4_status_string(int status);
/* Split-K control of the expert GEMMs (no counterpart in the reference; a
 * tuning and testing control).  1 (the default, or the DSV4_KSPLIT environment
 * variable at the first call) keeps every GEMM item on one CTA; 0 lets small
 * decode batches split each item's k range over several CTAs automatically;
 * n > 1 asks for up to n slices (at most 8).  Measured on B200 the split was
 * no faster at 1-16 tokens.  The split changes only the fp32 summation order of the expert
 * GEMMs.  It also changes dsv4_moe_workspace_bytes and the EP workspace
 * sizes: set it before sizing workspaces, not while calls are in flight. */
DSV4_API int dsv4_set_k_split(int slices);
/* Opt-in FP4 activations for the routed experts' GEMM1 (no counterpart in the
 * reference, whose layer quantizes activations to e4m3 per 128): on = 1 makes
 * dsv4_moe_forward quantize each routed row with the official fp4_act_quant
 * semantics (dsv4_fp4_act_quant) and run w1 | w3 as kind::mxf4 products
 * (e2m1 x e2m1, per-32 ue8m0 scales: the FP4 tensor rate, twice the FP8 one).
 * The shared expert, GEMM2 and the expert-parallel entry points keep e4m3
 * activations.  This changes the layer's numerics (FP4 activations); 0 (the
 * default, or DSV4_FP4_ACT=0) is the reference's arithmetic.  It changes
 * dsv4_moe_workspace_bytes: set it before sizing workspaces.
 * dsv4_moe_workspace_layout's out[20] says whether a layout uses it. */
DSV4_API int dsv4_set_fp4_activations(int on);
/* Decode batches of at most 8 tokens with the tensor-core gate: run the
 * gate's top-k, the route plan and the scatter as one kernel (1) instead of
 * three (0, the default).  Bit-identical results; measured no faster inside a
 * CUDA graph.  No counterpart in the reference. */
DSV4_API int dsv4_set_fused_routing(int on);
/* A counter that every call of dsv4_set_k_split / dsv4_set_fp4_activations /
 * dsv4_set_fused_routing
 * advances: a caller that captured CUDA graphs of the layer recaptures when it
 * changes (the settings choose the kernels a graph holds). */
DSV4_API long long dsv4_settings_generation(void);
/* Synchronises the device, returns the first device-side error code (0 if
 * none) in *code, and clears it when clear != 0. */
DSV4_API int dsv4_device_error(int clear, int* code);
/* Enqueues on `stream` a copy of the device-side error word of the current
 * device into *dst (pinned host or device memory) and returns at once; the
 * value is valid once the stream has reached that point.  Lets a caller check
 * for a latched error (for example a peer wait that ran out) without
 * synchronising the device.  No counterpart in the reference. */
DSV4_API int dsv4_device_error_async(int* dst, void* stream);

/* ---- MoE layer description ---------------------------------------------
 * Routed experts live in an expert arena: one device buffer of n_slots slots
 * of slot_stride bytes; a slot holds one packed expert block, bytes unchanged
 * from the packed slab (w1.scale, w2.scale, w3.scale, w1.weight, w2.weight,
 * w3.weight; scripts/build_packed_expert_layout.py:76-86): e2m1x2 weights
 * [I,H/2], [H,I/2], [I,H/2] and ue8m0 scales per 32 along K.  arena_sf holds
 * the tensor-memory scale atoms derived from those scales (written by
 * dsv4_materialize or dsv4_build_scale_atoms), sf_slot_stride = 3*I*H/32.
 * The shared expert is fp8 e4m3 [I,H], [H,I], [I,H] with 128x128 ue8m0 block
 * scales; shared_sf holds its atoms (dsv4_build_shared_scale_atoms). */
typedef struct dsv4_moe_layer {
  int hidden;          /* H (args.dim) */
  int inter;           /* I (args.moe_inter_dim) */
  int n_routed;        /* E (args.n_routed_experts) */
  int topk;            /* k (args.n_activated_experts) */
  int n_shared;        /* 0 or 1 (args.n_shared_experts) */
  float route_scale;   /* routed scaling factor */
  float swiglu_limit;  /* args.swiglu_limit; <= 0 disables the clamp */
  const void* gate_w;  /* [E,H] bf16 or fp32 */
  int gate_w_fp32;     /* 1 if gate_w is fp32 */
  const float* gate_bias;      /* [E] score-correction bias, or NULL */
  const uint8_t* arena;        /* routed expert slots */
  long long slot_stride;       /* bytes per slot (>= packed block bytes, % 32 == 0) */
  int n_slots;
  const uint8_t* arena_sf;     /* scale atoms per slot */
  long long sf_slot_stride;
  const int* expert_slot;      /* [E] expert id -> slot (device) */
  const uint8_t* shared_w1;    /* fp8 [I,H] */
  const uint8_t* shared_w2;    /* fp8 [H,I] */
  const uint8_t* shared_w3;    /* fp8 [I,H] */
  const uint8_t* shared_sf;    /* atoms: w1 | w3 | w2, each I*H/32 bytes */
} dsv4_moe_layer;

/* Bytes of scratch dsv4_moe_forward needs for T tokens (caller allocates). */
DSV4_API long long dsv4_moe_workspace_bytes(const dsv4_moe_layer* L, int T);

/* Byte offsets inside the workspace of the intermediate buffers, for
 * inspection: out[0..] = logits, weights, indices, counts, seg_start,
 * n_tiles, route_slot, slot_token, slot_weight, tiles, xq, xsf, hq, hsf, O.
 * Also returns max_rows in out[15] and block_n in out[16]. n_out >= 17.
 * With n_out > 17: out[17] = gate partial logits; with n_out > 19: out[18],
 * out[19] = split-K slices of the two expert GEMMs (1 = no split; small
 * batches split each GEMM item's k range so that every SM streams weights). */
DSV4_API int dsv4_moe_workspace_layout(const dsv4_moe_layer* L, int T, long long* out, int n_out);

/* LazyMoE.forward(x, input_ids) (spark_runtime/lazy_official_runtime.py:980-1002)
 * for one layer on one GPU: gate -> route plan -> permute+act_quant ->
 * grouped GEMM1 (w1|w3, SwiGLU, x routing weight, fp8 re-quant) -> grouped
 * GEMM2 (w2) -> ordered combine + shared expert -> bf16 y [T,H].
 * x: bf16 [T,H].  If routing_weights/routing_indices are non-NULL they
 * replace the gate (fp32 [T,k], int64 [T,k]).  No host synchronisation. */
DSV4_API int dsv4_moe_forward(const dsv4_moe_layer* L, const void* x, int T, void* y,
                     const float* routing_weights, const int64_t* routing_indices,
                     void* workspace, long long workspace_bytes, void* stream);

/* Official Expert.forward(x, weights) (constructed at
 * lazy_official_runtime.py:769-774 routed, :976-978 shared; called at :998,
 * :1001) for one expert over T rows: act_quant -> w1|w3 -> SwiGLU (clamp at
 * swiglu_limit) -> x row_weights[r] (if non-NULL) -> bf16 -> act_quant -> w2
 * -> bf16 y [T,H].  expert >= 0 selects routed expert `expert` of the arena
 * (via expert_slot); expert < 0 selects the fp8 shared expert. */
DSV4_API long long dsv4_expert_workspace_bytes(const dsv4_moe_layer* L, int T);
DSV4_API int dsv4_expert_forward(const dsv4_moe_layer* L, int expert, const void* x, int T,
                                 const float* row_weights, void* y, void* workspace,
                                 long long workspace_bytes, void* stream);

/* Stage timing of dsv4_moe_forward (no counterpart in the reference; its
 * telemetry timer is spark_runtime/telemetry.py:98-117): while enabled, every
 * forward records library-owned CUDA events between its kernels (as graph
 * nodes when the stream is being captured).  dsv4_profile_read waits for the
 * last forward and returns 6 durations in ms: gate, plan, permute, GEMM1,
 * GEMM2, combine.  The events are created on first enable and live until
 * the process exits, so graphs captured while profiling stay valid after
 * profiling is disabled. */
DSV4_API int dsv4_profile_enable(int enable);
DSV4_API int dsv4_profile_read(float* stage_ms, int n);

/* Allocation-free dsv4_expert_forward (no counterpart in the reference).
 * For callers that may not allocate device memory and cannot pass a
 * workspace: a host runtime that owns every allocation and passes only the
 * input and output buffers, or a serving loop that must not touch the
 * allocator while it runs.  Same arguments and results as
 * dsv4_expert_forward minus the workspace; the scratch is a fixed
 * dsv4_expert_static_scratch_bytes() (4 MiB) array of device memory that the
 * library holds on every GPU it runs on until the process exits.  Calls whose
 * dsv4_expert_workspace_bytes(L, T) exceeds it return DSV4_ERR_WORKSPACE
 * (up to 640 tokens at H=4096, I=2048).  The first call on a device looks up
 * the array's device address; make it before any stream capture.  The
 * address is cached for the life of the process, so the entry point is not
 * valid after cudaDeviceReset on a device it was called on.  All calls share
 * the array: calls that may overlap on the GPU race and must not be issued.
 * Nothing is allocated, freed or cleared.  y may be device, managed or
 * host-registered memory, as for dsv4_expert_forward. */
DSV4_API long long dsv4_expert_static_scratch_bytes(void);
DSV4_API int dsv4_expert_forward_static(const dsv4_moe_layer* L, int expert, const void* x, int T,
                                        const float* row_weights, void* y, void* stream);

/* ---- individual stages (same kernels as dsv4_moe_forward) --------------- */

/* Official Gate logits: logits[T,E] = x[T,H] . Wg[E,H]^T in fp32. */
DSV4_API int dsv4_gate_logits(const void* x, const void* w, int w_is_fp32, int T, int H, int E,
                     float* logits, void* stream);

/* Official Gate scoring (lazy_official_runtime.py:966,983): sigmoid scores,
 * + bias for selection, top-k (ties -> lower id), weights = scores at the
 * chosen ids renormalised to sum 1, x route_scale.  Bit-exact fp32. */
DSV4_API int dsv4_gate_topk(const float* logits, const float* bias, int T, int E, int topk,
                   float route_scale, float* weights, int64_t* indices, void* stream);

/* Official Gate.forward(x, input_ids) -> (weights, indices) (called at
 * lazy_official_runtime.py:983) in one call.  bf16 gate weights over 256
 * experts run on the tensor core: large batches with the routing fused into
 * the GEMM epilogue, small ones as split GEMM partials in `workspace`
 * (dsv4_gate_workspace_bytes() bytes; with less, the fused form is used).
 * Other gates run dsv4_gate_logits + dsv4_gate_topk.  Writes the fp32 logits
 * [T,E] too; routing is bit-exact on those logits on every path. */
DSV4_API long long dsv4_gate_workspace_bytes(const void* w, int w_is_fp32, int T, int H, int E);
DSV4_API int dsv4_gate_route(const void* x, const void* w, int w_is_fp32, const float* bias, int T,
                             int H, int E, int topk, float route_scale, float* logits,
                             float* weights, int64_t* indices, void* workspace,
                             long long workspace_bytes, void* stream);

/* Hash-routed layers (the official Gate with gate.tid2eid, layers 0-2 of the
 * checkpoint, weight-manifest.csv:3): the experts of token t are the row
 * tid2eid[input_ids[t]] ([vocab][topk] int64, in row order); the weights are
 * their sigmoid scores renormalised to sum 1 in row order, times route_scale.
 * logits [T][E] fp32 are written as for dsv4_gate_route.  Invalid ids or
 * table entries latch DSV4_DEVERR_BAD_INDEX and give index -1, weight 0. */
DSV4_API long long dsv4_gate_hash_workspace_bytes(const void* w, int w_is_fp32, int T, int H, int E);
DSV4_API int dsv4_gate_route_hash(const void* x, const void* w, int w_is_fp32, const int64_t* tid2eid,
                                  long long vocab, const int64_t* input_ids, int T, int H, int E,
                                  int topk, float route_scale, float* logits, float* weights,
                                  int64_t* indices, void* workspace, long long workspace_bytes,
                                  void* stream);

/* Official kernel.act_quant(x, 128, "ue8m0") (scripts/smoke_official_kernels.py:
 * 44-49): bf16 [M,K] -> e4m3 codes [M,K] + ue8m0 scales [M,K/128]. */
DSV4_API int dsv4_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* scale, void* stream);

/* Official kernel.fp4_act_quant(x, 32) (scripts/smoke_official_kernels.py:
 * 32-34; results float4_e2m1fn_x2 codes + float8_e8m0fnu scales,
 * docs/experiments/016-native-kernel-smoke.md:50): bf16 [M,K] -> packed e2m1
 * codes [M,K/2] (element 2i in the low nibble) + ue8m0 scales [M,K/32].  Per
 * 32 values: amax = max(|x|, 1e-4), s = 2^ceil(log2(amax * fp32(1/6))),
 * codes = e2m1(x / s) rounded to nearest even.  K % 32 == 0; x and q 16-byte
 * aligned. */
DSV4_API int dsv4_fp4_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* scale, void* stream);

/* ---- attention block: dense FP8 linear layers ---------------------------
 * The official linear(x, W) for an FP8 weight (act_quant(x, 128, "ue8m0") ->
 * fp8_gemm -> bf16; kernel API scripts/smoke_official_kernels.py:36-43), as the
 * attention projections wq_a [1024,4096], wq_b [32768,1024], wkv [512,4096],
 * wo_a [8192,4096], wo_b [4096,8192] use it (e4m3 weights with 128x128 ue8m0
 * block scales, results/spark-66c9/checkpoint-tensors.csv layers.L.attn.*).
 * y[M,N] bf16 = act_quant(x[M,K] bf16) . W[N,K]^T on the tensor core
 * (kind::mxf8f6f4, fp32 accumulate).  N % 256 == 0 and K % 512 == 0
 * (DSV4_ERR_UNSUPPORTED otherwise); x, W and y 16-byte aligned.
 * w_atoms: the weight's scales expanded once by dsv4_build_fp8_weight_atoms
 * (dsv4_fp8_weight_atoms_bytes(N, K) bytes) from scale [N/128][K/128].
 * With the split-K setting on (dsv4_set_k_split; off by default) and M <= 64,
 * the k range is split into 2-8 slices of whole 512-wide groups whose fp32
 * sums are added in slice order (deterministic); the workspace size follows
 * the setting in force when it is asked for. */
DSV4_API long long dsv4_fp8_weight_atoms_bytes(int N, int K);
DSV4_API int dsv4_build_fp8_weight_atoms(const uint8_t* scale, int N, int K, uint8_t* atoms, void* stream);
DSV4_API long long dsv4_fp8_linear_workspace_bytes(int M, int N, int K);
DSV4_API int dsv4_fp8_linear(const void* x, int M, int K, const uint8_t* w, const uint8_t* w_atoms, int N,
                             void* y, void* workspace, long long workspace_bytes, void* stream);

/* Official kernel.sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale)
 * (scripts/smoke_official_kernels.py:53-57), which the reference replaces by
 * its per-token fallback spark_runtime/lazy_official_runtime.py:1024-1049
 * because the official kernel fails at h=64, d=512 on GB10 (LOG.md:134-135).
 * q [B,S,H,D] bf16, kv [B,N,D] bf16 (one KV row for every head), attn_sink
 * [H] fp32, topk_idxs [B,S,K] int32 (-1 = no row), out [B,S,H,D] bf16:
 * out[b,s,h] = sum_j p[h,j] kv[b,idx_j] over the valid indices, p = softmax of
 * softmax_scale * q.kv with the sink's exp in the denominator; zeros when no
 * index is valid.  H = 64 and D = 512 (DSV4_ERR_UNSUPPORTED otherwise); q and
 * kv 16-byte aligned.  Indices >= N count as invalid and latch
 * DSV4_DEVERR_BAD_INDEX.  Workspace: dsv4_sparse_attn_workspace_bytes(B, S,
 * K) bytes (0 when every token fits one CTA's pass over its indices). */
DSV4_API long long dsv4_sparse_attn_workspace_bytes(int B, int S, int K);
DSV4_API int dsv4_sparse_attn(const void* q, const void* kv, const float* attn_sink, const int* topk_idxs,
                              int B, int S, int H, int N, int D, int K, float softmax_scale, void* out,
                              void* workspace, long long workspace_bytes, void* stream);

/* ---- expert arena / materializer ---------------------------------------
 * LazyRoutedExpert.materialize + ExpertCopyPlan::read_into_and_copy_cuda
 * (lazy_official_runtime.py:761-917; native_packed_loader.cpp:122-174,281-316),
 * device side: blocks already in device memory (slab + src_off[i]) are copied
 * into arena slots dst_slot[i] (bit-exact), their scale atoms written to
 * arena_sf, and (if bf16_out != NULL) their weights decoded exactly to bf16
 * ([I,H], [H,I], [I,H] in packed order w1, w2, w3 per slot).  Any of arena,
 * arena_sf, bf16_out may be NULL to skip that output.  src_off (int64) and
 * dst_slot (int32) are device arrays of length n; src_off % 16 == 0 (a block
 * whose offset is not is skipped and latches DSV4_DEVERR_MISALIGNED). */
DSV4_API int dsv4_materialize(const uint8_t* slab, const long long* src_off, const int* dst_slot, int n,
                     int hidden, int inter, uint8_t* arena, long long slot_stride,
                     uint8_t* arena_sf, long long sf_slot_stride, void* bf16_out,
                     long long bf16_slot_stride, void* stream);

/* Scale atoms for arena slots whose bytes are already in place
 * (slots[i] of n, device int32 array). */
DSV4_API int dsv4_build_scale_atoms(const uint8_t* arena, long long slot_stride, const int* slots, int n,
                           int hidden, int inter, uint8_t* arena_sf, long long sf_slot_stride,
                           void* stream);

/* Scale atoms for the fp8 shared expert (128x128 block scales w1/w3 [I/128,H/128],
 * w2 [H/128,I/128]) into shared_sf (3*I*H/32 bytes: w1 | w3 | w2). */
DSV4_API int dsv4_build_shared_scale_atoms(const uint8_t* w1_scale, const uint8_t* w2_scale,
                                  const uint8_t* w3_scale, int hidden, int inter,
                                  uint8_t* shared_sf, void* stream);

/* ---- packed-slab loader (host) -------------------------------------------
 * native_packed_loader.cpp:26-68 read_into: EINTR-safe pread loop of up to
 * `size` bytes at `offset` into dst (host memory).  Returns the byte count
 * (short at EOF) in *read_bytes.  errno of a failed pread in *err_no. */
DSV4_API int dsv4_read_into(int fd, void* dst, long long dst_capacity, long long size, long long offset,
                   long long* read_bytes, int* err_no);

/* native_packed_loader.cpp:70-190 copy_storage_to_tensors[_cuda] and
 * ExpertCopyPlan::copy_storage_to_tensors[_cuda]: copies slices
 * storage[offsets[i] : offsets[i]+target_bytes[i]] to targets[i].
 * expected_sizes (plan sizes) may be NULL.  to_device: 0 = host memcpy,
 * 1 = cudaMemcpyAsync host->device on `stream`, one per target.
 * The sum of copied bytes is returned in *copied. */
DSV4_API int dsv4_copy_slices(const void* storage, long long storage_bytes, void* const* targets,
                     const long long* target_bytes, const long long* offsets,
                     const long long* expected_sizes, int n, int to_device, void* stream,
                     long long* copied);

/* ExpertCopyPlan::read_into_and_copy[_cuda] (native_packed_loader.cpp:232-316):
 * read `size` bytes at `offset` into staging, fail with DSV4_ERR_SHORT_READ
 * on a short read, then copy the planned slices.  Timings in seconds. */
DSV4_API int dsv4_read_into_and_copy(int fd, void* staging, long long staging_capacity, long long size,
                            long long offset, void* const* targets, const long long* target_bytes,
                            const long long* offsets, const long long* expected_sizes, int n,
                            int to_device, void* stream, long long* read_bytes,
                            long long* copied_bytes, double* read_seconds, double* copy_seconds,
                            int* err_no);

/* ------------------------------------------------------------------------
 * Expert parallelism over W ranks (W <= 8; rank r owns experts
 * [r*E/W, (r+1)*E/W), spark_runtime/lazy_official_runtime.py:956-965).
 * Replaces the reference's replicated tokens + dist.all_reduce(y) (:999-1000)
 * with a dispatch of FP8 rows to the owning ranks and a return of every
 * route's bf16 output row; the host moves the buffers (NCCL all-to-all):
 *
 *   1 dsv4_ep_dispatch       (source)  send rows + send_counts [W][2] (rows,
 *                                      routes per destination) + ret_pos
 *   2 exchange send_counts -> recv_counts; rows: send -> recv (row_bytes each)
 *   3 dsv4_ep_expert_forward (owner)   recv rows + own tokens' shared expert
 *                                      -> ret_send [sum recv routes][H] bf16
 *   4 exchange ret_send -> ret_recv (bf16 rows, H each; split by routes)
 *   5 dsv4_ep_combine        (source)  y [T_own][H] bf16
 *
 * Steps 3 and 5 share one workspace of dsv4_ep_expert_workspace_bytes(L, W,
 * T_own, R), R = rows received.  The result is bit-identical to
 * dsv4_moe_forward on the same tokens and routing.
 * ---------------------------------------------------------------------- */
/* Bytes of one send row: H e4m3 codes, H/128 ue8m0 scales, topk route
 * entries {int32 expert (-1: another rank's), f32 weight, int32 return
 * index}, padded to 16. */
DSV4_API long long dsv4_ep_row_bytes(int hidden, int topk);
DSV4_API long long dsv4_ep_dispatch_workspace_bytes(int T, int world);
/* send: >= T*min(world, topk) rows of dsv4_ep_row_bytes; rows for rank d
 * start at the sum of earlier ranks' row counts, tokens in order.
 * send_counts: device int32 [world][2].  ret_pos: device int32 [T][topk],
 * the row of the return buffer (blocks in rank order) holding each route. */
DSV4_API int dsv4_ep_dispatch(const void* x, const int64_t* indices, const float* weights, int T,
                              int hidden, int topk, int n_routed, int world, void* send,
                              long long send_rows, int* send_counts, int* ret_pos,
                              void* workspace, long long workspace_bytes, void* stream);
DSV4_API long long dsv4_ep_expert_workspace_bytes(const dsv4_moe_layer* L, int world, int T_own,
                                                  int R);
/* x_own: this rank's T_own tokens (bf16, for the shared expert); recv: R
 * received rows in source-rank order; recv_counts: device int32 [world][2]
 * as received.  ret_send: >= ret_rows bf16 rows of H, filled for every
 * received route (blocks by source rank). */
DSV4_API int dsv4_ep_expert_forward(const dsv4_moe_layer* L, int rank, int world,
                                    const void* x_own, int T_own, const void* recv, int R,
                                    const int* recv_counts, void* ret_send, long long ret_rows,
                                    void* workspace, long long workspace_bytes, void* stream);
/* y[t] = bf16( sum over t's routes in ascending expert id of ret_recv[ret_pos]
 * + t's shared row ), as the single GPU combine. */
DSV4_API int dsv4_ep_combine(const dsv4_moe_layer* L, int rank, int world, const void* ret_recv,
                             const int* ret_pos, const int64_t* indices, int T_own, int R,
                             const void* workspace, long long workspace_bytes, void* y,
                             void* stream);

/* ------------------------------------------------------------------------
 * Expert parallelism over peer memory (one process per GPU of one NVLink /
 * NVSwitch node).  The same five steps as above, with the two exchanges done
 * by the kernels themselves instead of host collectives and with no host
 * synchronisation: the source's pack kernel quantizes each token once and
 * stores its FP8 row straight into the owning rank's exchange buffer over
 * NVLink, and the owner's return kernel stores every route's bf16 output row
 * straight into the source's buffer.  Each side raises an epoch flag in the
 * other's buffer after a system-scope fence; the waiting side spins on it for
 * at most 2 s (DSV4_DEVERR_TIMEOUT_PEER on expiry, never a hang).  Plain
 * peer loads and stores only: no multicast object, no NVLS.
 *
 * Set-up, once per rank: an exchange buffer of dsv4_ep_exchange_bytes(H,
 * topk, W, cap_tokens) from dsv4_ep_exchange_alloc (zeroed), its IPC handle
 * (dsv4_ipc_handle) sent to every other rank, their buffers mapped with
 * dsv4_ipc_open, and a device array uint64 peer_bases[W] of every rank's
 * buffer as seen from this GPU (this rank's own at index rank).  cap_tokens
 * bounds the tokens any rank passes per call.  Per layer call, every rank
 * uses the same epoch, a positive value that differs from the previous
 * call's; or every call of the buffer's life passes epoch 0, and the library
 * counts calls in the buffer itself (dispatch increments, the other steps
 * read), which is what a CUDA graph of the three steps needs (every rank
 * replays it the same number of times):
 *
 *   dsv4_ep_dispatch_p2p       (source)  rows into every owner's buffer, ret_pos
 *   dsv4_ep_expert_forward_p2p (owner)   waits for all W sources, computes,
 *                                        stores return rows into their buffers
 *   dsv4_ep_combine_p2p        (source)  waits for all W owners, y [T_own][H]
 *
 * Buffers are reused across calls without further synchronisation: a source
 * starts call e+1 only after its call-e combine has received every owner's
 * returns, so no owner is still reading call e's rows.  The result is
 * bit-identical to dsv4_moe_forward.  Replaces the same reference exchange as
 * above (spark_runtime/lazy_official_runtime.py:999-1000).
 * ---------------------------------------------------------------------- */
#define DSV4_IPC_HANDLE_BYTES 64
DSV4_API long long dsv4_ep_exchange_bytes(int hidden, int topk, int world, int cap_tokens);
DSV4_API int dsv4_ep_exchange_alloc(int device, long long bytes, void** out);
DSV4_API int dsv4_ep_exchange_free(void* buffer);
/* 64-byte CUDA IPC handle of an allocation from dsv4_ep_exchange_alloc. */
DSV4_API int dsv4_ipc_handle(const void* buffer, uint8_t* handle);
/* Map another process's buffer into GPU `device`'s address space (peer access). */
DSV4_API int dsv4_ipc_open(int device, const uint8_t* handle, void** out);
DSV4_API int dsv4_ipc_close(void* mapped);
DSV4_API long long dsv4_ep_p2p_dispatch_workspace_bytes(int T, int world);
/* ret_pos: device int32 [T][topk], the row of this rank's return region that
 * will hold each route (blocks in owner-rank order). */
DSV4_API int dsv4_ep_dispatch_p2p(const void* x, const int64_t* indices, const float* weights,
                                  int T, int hidden, int topk, int n_routed, int world, int rank,
                                  const uint64_t* peer_bases, int cap_tokens, int epoch,
                                  int* ret_pos, void* workspace, long long workspace_bytes,
                                  void* stream);
DSV4_API long long dsv4_ep_p2p_expert_workspace_bytes(const dsv4_moe_layer* L, int world,
                                                      int T_own, int cap_tokens);
/* exchange: this rank's own buffer. Steps 3 and 5 share one workspace. */
DSV4_API int dsv4_ep_expert_forward_p2p(const dsv4_moe_layer* L, int rank, int world,
                                        const void* x_own, int T_own, void* exchange,
                                        const uint64_t* peer_bases, int cap_tokens, int epoch,
                                        void* workspace, long long workspace_bytes, void* stream);
DSV4_API int dsv4_ep_combine_p2p(const dsv4_moe_layer* L, int rank, int world,
                                 const void* exchange, const int* ret_pos, const int64_t* indices,
                                 int T_own, int cap_tokens, int epoch, const void* workspace,
                                 long long workspace_bytes, void* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSV4MOE_H_ */
