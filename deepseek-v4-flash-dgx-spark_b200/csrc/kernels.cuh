// Internal declarations shared by the dsv4moe translation units.
#pragma once

#include "common.cuh"

namespace dsv4 {

// Arguments of the grouped expert GEMM kernel (see expert_gemm.cu).
struct GemmArgs {
  const int4* tiles;      // [n_tiles] {segment, row0, nrows, compact index of row0}
  const int* n_tiles;     // device scalar written by the route plan
  const int* expert_slot; // [n_routed] routed expert -> arena slot
  int n_routed;           // segment id n_routed is the shared expert
  int kt_count;           // K / 128
  int nb_count;           // weight blocks per tile: GEMM1 inter/128 (w1|w3 pairs), GEMM2 hidden/256
  const uint8_t* sf_routed;
  long long sf_slot_stride;
  long long sf_off0, sf_off1;  // byte offsets of the A0 / A1 atoms inside a slot
  const uint8_t* sf_shared0;
  const uint8_t* sf_shared1;
  const uint8_t* sfb;          // activation atoms, sliding k-packed layout [row/32][kt_count/4][512]
  const float* slot_weight;    // GEMM1: routing weight of each segment row
  uint8_t* out_q;              // GEMM1: H codes [rows][out_ld]
  uint8_t* out_sf;             // GEMM1: H scale atoms, same layout [row/32][out_ld/512][512]
  __nv_bfloat16* out_bf16;     // GEMM2: O [rows][out_ld]
  int out_ld;
  float swiglu_limit;
  // split-K (k_split > 1): every item's k tiles are cut into k_split slices
  // of whole scale groups; a slice stores its fp32 sums of the item's valid
  // rows in partial[slice][compact row][part_ld], and the CTA that finishes
  // the item's last slice adds the slices in order and runs the epilogue.
  int k_split;
  float* partial;
  int part_rows;          // compact rows per slice (>= every valid route row)
  int part_ld;            // floats per compact row: nb_count * 256
  int* item_done;         // [n_tiles * nb_count] slices finished, zeroed by the route plan
  // 0: every segment; 1: routed segments only; 2: the shared segment only
  // (an item of another segment is skipped by all warps alike)
  int seg_filter;
};

int launch_gate_logits(const void* x, const void* w, int w_is_fp32, int T, int H, int E,
                       float* logits, cudaStream_t st);
int launch_gate_topk(const float* logits, const float* bias, int T, int E, int k,
                     float route_scale, float* weights, int64_t* indices, cudaStream_t st,
                     int nsplit = 1, float* logits_out = nullptr,
                     const int64_t* hash_table = nullptr, const int64_t* input_ids = nullptr,
                     long long vocab = 0);
int launch_gate_gemm_partials(const void* x, const void* w, int T, int H, int E, float* partials,
                              int num_sms, cudaStream_t st);
void gate_gemm_split_shape(int T, int H, int E, int num_sms, int* bm, int* ksplit);
int launch_gate_gemm_topk(const void* x, const void* w, int T, int H, const float* bias, int k,
                          float route_scale, float* logits, float* weights, int64_t* indices,
                          int num_sms, cudaStream_t st);
int route_chunk_tokens(int T);
int launch_route_plan(const int64_t* indices, int T, int k, int E, int allow_skip,
                      int shared_rows, int block_n, int max_rows, int max_tiles, int* chunk_cnt,
                      int* chunk_base, int* ctrl, int* counts, int* seg_start, int4* tiles,
                      int* n_tiles, int* slot_token, float* slot_weight, cudaStream_t st,
                      int* zero_ptr = nullptr, int n_zero = 0);
int launch_route_scatter(const void* x, int n_x_rows, const uint8_t* rows_in,
                         long long rows_in_stride, const int64_t* indices, const float* weights,
                         int T, int k, int E, int H, int shared_rows, const int* seg_start,
                         const int* chunk_base, const int* ctrl, int* route_slot, int* slot_token,
                         float* slot_weight, uint8_t* xq, uint8_t* sfb, int num_sms,
                         cudaStream_t st);
int launch_permute_quant(const void* x, int H, const int* slot_token, const int* total_rows_ptr,
                         int max_rows, uint8_t* xq, uint8_t* sfb, int num_sms, cudaStream_t st);
int launch_single_segment_plan(int T, int seg, int block_n, int rows_pad, const float* w,
                               int* slot_token, float* slot_weight, int4* tiles, int* n_tiles,
                               int* total_rows, cudaStream_t st);
int launch_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* s, int num_sms,
                     cudaStream_t st);
// Decode batches (T <= 8): gate top-k from split-K partial logits + route plan
// + scatter/act_quant in one launch.
int launch_route_small_fused(const float* partials, int nsplit, float* logits_out, const float* bias, int T, int E,
                             int k, float route_scale, float* weights, int64_t* indices, const void* x, int H,
                             int shared_rows, int block_n, int max_rows, int max_tiles, int* chunk_base, int* counts,
                             int* seg_start, int4* tiles, int* n_tiles, int* slot_token, float* slot_weight,
                             int* ctrl, int* zero_ptr, int n_zero, int* route_slot, uint8_t* xq, uint8_t* sfb,
                             cudaStream_t st);
int launch_fp4_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* s, int num_sms, cudaStream_t st);
int launch_fp4_scatter_quant(const void* x, int T, int H, int k, const int* route_slot, int max_rows, uint8_t* xq4,
                             uint8_t* atoms, int num_sms, cudaStream_t st);
// expert parallelism (ep.cu)
long long ep_row_bytes(int H, int k);
long long ep_dispatch_workspace(int T, int world);
int launch_ep_dispatch(const void* x, const int64_t* indices, const float* weights, int T, int H,
                       int k, int E, int world, uint8_t* send, int* send_counts, int* ret_pos,
                       uint8_t* ws, int num_sms, cudaStream_t st,
                       const uint64_t* peer_bases = nullptr, int rank = 0, int cap = 0,
                       int epoch = 0);
long long ep_exchange_bytes(int H, int k, int world, int cap);
long long ep_return_region_off(int H, int k, int world, int cap);
int launch_ep_signal_empty(const uint64_t* peer_bases, int rank, int world, int* send_counts,
                           uint8_t* ws, int epoch, cudaStream_t st);
int launch_ep_wait(const uint8_t* own, int flag_off, int world, int epoch, int err_code,
                   cudaStream_t st);
int launch_ep_unpack_p2p(const uint8_t* exch, int cap, int T_own, int k, int H, int e_begin,
                         int e_count, int world, int64_t* idx_local, float* w_local, int* ret_dst,
                         cudaStream_t st);
int launch_ep_return_p2p(const void* O, int H, int k, const int* route_slot, const int* ret_dst,
                         int n_routes, const uint64_t* bases, int rank, int world, int cap,
                         int epoch, int num_sms, cudaStream_t st);
int launch_ep_unpack(const uint8_t* recv, int R, int T_own, int k, int H, int e_begin, int e_count,
                     const int* recv_counts, int world, int64_t* idx_local, float* w_local,
                     int* ret_dst, cudaStream_t st);
int launch_ep_return_gather(const void* O, int H, const int* route_slot, const int* ret_dst,
                            int n_routes, long long ret_rows, void* ret, int num_sms,
                            cudaStream_t st);
long long sparse_attn_workspace(int tokens, int K, int num_sms, int* splits_out, int* cps_out);
int launch_sparse_attn(const void* q, const void* kv, const float* sink, const int* idx, int B, int S,
                       int N, int K, float scale, void* out, void* ws, long long ws_bytes, int num_sms,
                       cudaStream_t st);
int launch_combine(const void* O, int H, const int* route_slot, const int64_t* indices, int T,
                   int k, const int* shared_base, void* y, cudaStream_t st,
                   const void* O_shared = nullptr);
int launch_materialize(const uint8_t* slab, const long long* src_off, const int* dst_slot, int n,
                       long long block_bytes, uint8_t* arena, long long slot_stride, int hidden,
                       int inter, uint8_t* sf, long long sf_slot_stride, void* bf16_out,
                       long long bf16_slot_stride, int num_sms, cudaStream_t st);
int launch_build_sf_fp4_arena(const uint8_t* arena, long long slot_stride, const int* slots,
                              int n, int hidden, int inter, uint8_t* sf, long long sf_slot_stride,
                              int num_sms, cudaStream_t st);
int launch_build_sf_fp8(const uint8_t* scale, int rows, int K, uint8_t* atoms, int num_sms,
                        cudaStream_t st);
int make_tmap_fp4_arena(CUtensorMap* m, const void* base, int K, int rows, int slots,
                        long long slot_stride, int l2_promotion);
int make_tmap_u8(CUtensorMap* m, const void* base, int K, int rows, int box_rows);
int make_tmap_fp4_packed_arena(CUtensorMap* m, const void* base, int K, int rows, int slots,
                               long long slot_stride, int l2_promotion);
struct PairMaps;
int make_tmap_atoms(CUtensorMap* m, const void* base, long long bytes, int box_rows);
int pair_clusters_resident(bool gated);
int launch_expert_gemm_pair(bool gated, const PairMaps& maps, const GemmArgs& args,
                            long long sfs_row_off0, long long sfs_row_off1,
                            long long sfw_row_off0, long long sfw_row_off1, int clusters,
                            cudaStream_t st);
int launch_expert_gemm(bool gated, int block_n, const CUtensorMap& a0, const CUtensorMap& a1,
                       const CUtensorMap& s0, const CUtensorMap& s1, const CUtensorMap& b,
                       const GemmArgs& args, int grid, cudaStream_t st);
// The routed experts' GEMMs on FP4 activations (kind::mxf4): gated = GEMM1
// (a0 / a1 packed w1 / w3 arena maps; its epilogue writes FP4 h: packed codes
// [rows][out_ld/2] + per-32 atoms), else GEMM2 (a0 the packed w2 map);
// b the packed activation rows, args.kt_count = K / 256, args.sfb the per-32
// activation atoms.
int launch_expert_gemm_fp4(bool gated, int block_n, const CUtensorMap& a0, const CUtensorMap& a1,
                           const CUtensorMap& b, const GemmArgs& args, int grid, cudaStream_t st);

}  // namespace dsv4
