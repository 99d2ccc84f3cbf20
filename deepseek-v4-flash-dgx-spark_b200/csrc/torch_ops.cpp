// torch custom-op layer over the C ABI of libdsv4moe.so: TORCH_LIBRARY(dsv4moe).
//
// Each op unpacks its tensors into the plain pointers and sizes of the C ABI
// (include/dsv4moe.h), runs on torch's current CUDA stream of the input's
// device, takes scratch from torch's caching allocator, and turns a non-zero
// status into a RuntimeError (TORCH_CHECK) with the reference's message where
// the reference has one (spark_runtime/native/native_packed_loader.cpp:27-33,
// 47-56,77-108,128-160,203-207,265,299).  Nothing here computes: every op is
// one C ABI call.  Fake (meta) kernels are registered from Python
// (spark_b200/ops.py), so the ops trace under torch.compile / FakeTensor.
//
// A MoE layer is passed as three lists, in this order:
//   layer   : Tensor?[9]  gate_w, gate_bias, arena, arena_sf, expert_slot,
//                         shared_w1, shared_w2, shared_w3, shared_sf
//   dims    : int[8]      hidden, inter, n_routed, topk, n_shared, n_slots,
//                         slot_stride, sf_slot_stride
//   scalars : float[2]    route_scale, swiglu_limit
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cerrno>
#include <cstring>
#include <optional>
#include <string>
#include <vector>

#include "dsv4moe.h"

namespace {

using OptT = std::optional<at::Tensor>;
using TList = c10::List<std::optional<at::Tensor>>;

void* stream_of(const at::Tensor& t) {
  return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

const void* ptr_or_null(const OptT& t) { return t.has_value() ? t->data_ptr() : nullptr; }

void check_status(int rc, const char* what) {
  if (rc == DSV4_OK) return;
  switch (rc) {
    case DSV4_ERR_SHORT_READ: TORCH_CHECK(false, "short packed expert read");
    case DSV4_ERR_BOUNDS: TORCH_CHECK(false, "source slice exceeds storage tensor");
    case DSV4_ERR_SIZE: TORCH_CHECK(false, "target size does not match expert copy plan");
    default: TORCH_CHECK(false, what, ": ", dsv4_status_string(rc), " (status ", rc, ")");
  }
}

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

// The C ABI's layer description from the three lists.
dsv4_moe_layer make_layer(const TList& layer, at::IntArrayRef dims, at::ArrayRef<double> scalars) {
  TORCH_CHECK(layer.size() == 9, "layer must list 9 tensors (gate_w, gate_bias, arena, arena_sf, "
              "expert_slot, shared_w1, shared_w2, shared_w3, shared_sf)");
  TORCH_CHECK(dims.size() == 8, "dims must hold hidden, inter, n_routed, topk, n_shared, n_slots, "
              "slot_stride, sf_slot_stride");
  TORCH_CHECK(scalars.size() == 2, "scalars must hold route_scale, swiglu_limit");
  auto get = [&](size_t i) -> OptT { return layer.get(i); };
  for (size_t i = 0; i < 9; ++i) {
    const OptT t = get(i);
    if (t.has_value()) check_cuda(*t, "layer tensor");
  }
  dsv4_moe_layer L{};
  L.hidden = static_cast<int>(dims[0]);
  L.inter = static_cast<int>(dims[1]);
  L.n_routed = static_cast<int>(dims[2]);
  L.topk = static_cast<int>(dims[3]);
  L.n_shared = static_cast<int>(dims[4]);
  L.n_slots = static_cast<int>(dims[5]);
  L.slot_stride = dims[6];
  L.sf_slot_stride = dims[7];
  L.route_scale = static_cast<float>(scalars[0]);
  L.swiglu_limit = static_cast<float>(scalars[1]);
  const OptT gw = get(0);
  L.gate_w = ptr_or_null(gw);
  L.gate_w_fp32 = gw.has_value() && gw->scalar_type() == at::kFloat;
  L.gate_bias = static_cast<const float*>(ptr_or_null(get(1)));
  L.arena = static_cast<const uint8_t*>(ptr_or_null(get(2)));
  L.arena_sf = static_cast<const uint8_t*>(ptr_or_null(get(3)));
  L.expert_slot = static_cast<const int*>(ptr_or_null(get(4)));
  L.shared_w1 = static_cast<const uint8_t*>(ptr_or_null(get(5)));
  L.shared_w2 = static_cast<const uint8_t*>(ptr_or_null(get(6)));
  L.shared_w3 = static_cast<const uint8_t*>(ptr_or_null(get(7)));
  L.shared_sf = static_cast<const uint8_t*>(ptr_or_null(get(8)));
  return L;
}

at::Tensor workspace_for(const OptT& given, long long need, const at::Tensor& like) {
  TORCH_CHECK(need >= 0, "invalid layer description");
  if (given.has_value()) {
    check_cuda(*given, "workspace");
    TORCH_CHECK(given->scalar_type() == at::kByte, "workspace must be uint8");
    TORCH_CHECK(given->numel() >= need, "workspace too small");
    return *given;
  }
  return at::empty({std::max<long long>(need, 1)}, like.options().dtype(at::kByte));
}

at::Tensor bf16_rows(const at::Tensor& x, int64_t hidden) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must be bfloat16");
  TORCH_CHECK(x.size(-1) == hidden, "x's last dimension must be the hidden size");
  return x.reshape({-1, hidden});
}

// ---------------------------------------------------------------- layer ops
void moe_forward_out(const at::Tensor& x, const TList& layer, at::IntArrayRef dims,
                     at::ArrayRef<double> scalars, const OptT& routing_weights,
                     const OptT& routing_indices, const OptT& workspace, at::Tensor& out) {
  const dsv4_moe_layer L = make_layer(layer, dims, scalars);
  const at::Tensor x2 = bf16_rows(x, L.hidden);
  c10::cuda::CUDAGuard guard(x2.device());
  check_cuda(out, "out");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.numel() == x2.numel(), "out must match x");
  const int T = static_cast<int>(x2.size(0));
  TORCH_CHECK(routing_weights.has_value() == routing_indices.has_value(),
              "routing_weights and routing_indices go together");
  at::Tensor rw, ri;
  if (routing_weights.has_value()) {
    rw = routing_weights->to(at::kFloat).contiguous();
    ri = routing_indices->to(at::kLong).contiguous();
    TORCH_CHECK(rw.numel() == (int64_t)T * L.topk && ri.numel() == rw.numel(), "routing must be [T, topk]");
  }
  const long long need = dsv4_moe_workspace_bytes(&L, T);
  at::Tensor ws = workspace_for(workspace, need, x2);
  check_status(dsv4_moe_forward(&L, x2.data_ptr(), T, out.data_ptr(),
                                rw.defined() ? rw.data_ptr<float>() : nullptr,
                                ri.defined() ? ri.data_ptr<int64_t>() : nullptr, ws.data_ptr(),
                                ws.numel(), stream_of(x2)),
               "dsv4_moe_forward");
}

at::Tensor moe_forward(const at::Tensor& x, const TList& layer, at::IntArrayRef dims,
                       at::ArrayRef<double> scalars, const OptT& routing_weights,
                       const OptT& routing_indices, const OptT& workspace) {
  at::Tensor out = at::empty_like(x, x.options().memory_format(at::MemoryFormat::Contiguous));
  moe_forward_out(x, layer, dims, scalars, routing_weights, routing_indices, workspace, out);
  return out;
}

int64_t moe_workspace_bytes(const TList& layer, at::IntArrayRef dims, at::ArrayRef<double> scalars,
                            int64_t T) {
  const dsv4_moe_layer L = make_layer(layer, dims, scalars);
  return dsv4_moe_workspace_bytes(&L, static_cast<int>(T));
}

at::Tensor expert_forward(const at::Tensor& x, int64_t expert, const OptT& row_weights,
                          const TList& layer, at::IntArrayRef dims, at::ArrayRef<double> scalars) {
  const dsv4_moe_layer L = make_layer(layer, dims, scalars);
  const at::Tensor x2 = bf16_rows(x, L.hidden);
  c10::cuda::CUDAGuard guard(x2.device());
  const int T = static_cast<int>(x2.size(0));
  at::Tensor w;
  if (row_weights.has_value()) {
    w = row_weights->to(at::kFloat).contiguous();
    TORCH_CHECK(w.numel() == T, "routing weights must have one entry per row");
  }
  at::Tensor y = at::empty_like(x2);
  at::Tensor ws = workspace_for(std::nullopt, dsv4_expert_workspace_bytes(&L, T), x2);
  check_status(dsv4_expert_forward(&L, static_cast<int>(expert), x2.data_ptr(), T,
                                   w.defined() ? w.data_ptr<float>() : nullptr, y.data_ptr(),
                                   ws.data_ptr(), ws.numel(), stream_of(x2)),
               "dsv4_expert_forward");
  return y.view(x.sizes());
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> gate_route(const at::Tensor& x, const at::Tensor& w,
                                                          const OptT& bias, int64_t topk,
                                                          double route_scale, const OptT& tid2eid,
                                                          const OptT& input_ids) {
  check_cuda(w, "gate weight");
  const int64_t H = w.size(1), E = w.size(0);
  const at::Tensor x2 = bf16_rows(x, H);
  c10::cuda::CUDAGuard guard(x2.device());
  const int T = static_cast<int>(x2.size(0));
  const int fp32 = w.scalar_type() == at::kFloat;
  auto opts = x2.options();
  at::Tensor logits = at::empty({T, E}, opts.dtype(at::kFloat));
  at::Tensor weights = at::empty({T, topk}, opts.dtype(at::kFloat));
  at::Tensor indices = at::empty({T, topk}, opts.dtype(at::kLong));
  TORCH_CHECK(tid2eid.has_value() == input_ids.has_value(), "tid2eid and input_ids go together");
  if (tid2eid.has_value()) {
    check_cuda(*tid2eid, "tid2eid");
    at::Tensor ids = input_ids->to(x2.device(), at::kLong).contiguous().view(-1);
    TORCH_CHECK(ids.numel() == T, "input_ids must hold one id per token");
    const long long need = dsv4_gate_hash_workspace_bytes(w.data_ptr(), fp32, T, H, E);
    at::Tensor ws = workspace_for(std::nullopt, need, x2);
    check_status(dsv4_gate_route_hash(x2.data_ptr(), w.data_ptr(), fp32, tid2eid->data_ptr<int64_t>(),
                                      tid2eid->size(0), ids.data_ptr<int64_t>(), T, H, E, topk,
                                      static_cast<float>(route_scale), logits.data_ptr<float>(),
                                      weights.data_ptr<float>(), indices.data_ptr<int64_t>(),
                                      ws.data_ptr(), need > 0 ? need : 0, stream_of(x2)),
                 "dsv4_gate_route_hash");
  } else {
    const long long need = dsv4_gate_workspace_bytes(w.data_ptr(), fp32, T, H, E);
    at::Tensor ws = workspace_for(std::nullopt, need, x2);
    check_status(dsv4_gate_route(x2.data_ptr(), w.data_ptr(), fp32,
                                 static_cast<const float*>(ptr_or_null(bias)), T, H, E, topk,
                                 static_cast<float>(route_scale), logits.data_ptr<float>(),
                                 weights.data_ptr<float>(), indices.data_ptr<int64_t>(), ws.data_ptr(),
                                 need > 0 ? need : 0, stream_of(x2)),
                 "dsv4_gate_route");
  }
  return {weights, indices, logits};
}

at::Tensor gate_logits(const at::Tensor& x, const at::Tensor& w) {
  check_cuda(w, "gate weight");
  const int64_t H = w.size(1), E = w.size(0);
  const at::Tensor x2 = bf16_rows(x, H);
  c10::cuda::CUDAGuard guard(x2.device());
  at::Tensor logits = at::empty({x2.size(0), E}, x2.options().dtype(at::kFloat));
  check_status(dsv4_gate_logits(x2.data_ptr(), w.data_ptr(), w.scalar_type() == at::kFloat,
                                static_cast<int>(x2.size(0)), static_cast<int>(H), static_cast<int>(E),
                                logits.data_ptr<float>(), stream_of(x2)),
               "dsv4_gate_logits");
  return logits;
}

std::tuple<at::Tensor, at::Tensor> gate_topk(const at::Tensor& logits, const OptT& bias, int64_t topk,
                                             double route_scale) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2, "logits must be fp32 [T, E]");
  c10::cuda::CUDAGuard guard(logits.device());
  const int T = static_cast<int>(logits.size(0)), E = static_cast<int>(logits.size(1));
  at::Tensor w = at::empty({T, topk}, logits.options());
  at::Tensor idx = at::empty({T, topk}, logits.options().dtype(at::kLong));
  check_status(dsv4_gate_topk(logits.data_ptr<float>(), static_cast<const float*>(ptr_or_null(bias)), T, E,
                              static_cast<int>(topk), static_cast<float>(route_scale), w.data_ptr<float>(),
                              idx.data_ptr<int64_t>(), stream_of(logits)),
               "dsv4_gate_topk");
  return {w, idx};
}

std::tuple<at::Tensor, at::Tensor> act_quant(const at::Tensor& x) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must be bfloat16");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t K = x.size(-1);
  const at::Tensor x2 = x.reshape({-1, K});
  at::Tensor q = at::empty(x2.sizes(), x2.options().dtype(at::kByte));
  at::Tensor s = at::empty({x2.size(0), K / 128}, x2.options().dtype(at::kByte));
  check_status(dsv4_act_quant(x2.data_ptr(), static_cast<int>(x2.size(0)), static_cast<int>(K),
                              q.data_ptr<uint8_t>(), s.data_ptr<uint8_t>(), stream_of(x2)),
               "dsv4_act_quant");
  return {q, s};
}

// The official kernel.fp4_act_quant(x, 32): packed e2m1 codes [M, K/2] (two
// per byte, element 2i in the low nibble) and ue8m0 scale bytes [M, K/32].
std::tuple<at::Tensor, at::Tensor> fp4_act_quant(const at::Tensor& x) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must be bfloat16");
  const int64_t K = x.size(-1);
  TORCH_CHECK(K % 32 == 0, "the last dimension must be a multiple of 32");
  c10::cuda::CUDAGuard guard(x.device());
  const at::Tensor x2 = x.reshape({-1, K});
  at::Tensor q = at::empty({x2.size(0), K / 2}, x2.options().dtype(at::kByte));
  at::Tensor s = at::empty({x2.size(0), K / 32}, x2.options().dtype(at::kByte));
  check_status(dsv4_fp4_act_quant(x2.data_ptr(), static_cast<int>(x2.size(0)), static_cast<int>(K),
                                  q.data_ptr<uint8_t>(), s.data_ptr<uint8_t>(), stream_of(x2)),
               "dsv4_fp4_act_quant");
  return {q, s};
}

// ---------------------------------------------------------- attention block
// The official kernel.sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale)
// (spark_runtime/lazy_official_runtime.py:1016-1049 swaps in a Python fallback).
at::Tensor sparse_attn(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& attn_sink,
                       const at::Tensor& topk_idxs, double softmax_scale) {
  check_cuda(q, "q");
  check_cuda(kv, "kv");
  TORCH_CHECK(q.dim() == 4 && kv.dim() == 3 && topk_idxs.dim() == 3, "q [B,S,H,D], kv [B,N,D], topk_idxs [B,S,K]");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && kv.scalar_type() == at::kBFloat16, "q and kv must be bfloat16");
  c10::cuda::CUDAGuard guard(q.device());
  const int B = static_cast<int>(q.size(0)), S = static_cast<int>(q.size(1));
  const int H = static_cast<int>(q.size(2)), D = static_cast<int>(q.size(3));
  const int N = static_cast<int>(kv.size(1)), K = static_cast<int>(topk_idxs.size(2));
  TORCH_CHECK(kv.size(0) == B && kv.size(2) == D && topk_idxs.size(0) == B && topk_idxs.size(1) == S,
              "q, kv and topk_idxs disagree on batch, positions or head dim");
  const at::Tensor sink = attn_sink.to(q.device(), at::kFloat).contiguous();
  const at::Tensor idx = topk_idxs.to(q.device(), at::kInt).contiguous();
  at::Tensor out = at::empty_like(q);
  const long long need = dsv4_sparse_attn_workspace_bytes(B, S, K);
  TORCH_CHECK(need >= 0, "sparse_attn: invalid shape");
  at::Tensor ws = at::empty({std::max<long long>(need, 1)}, q.options().dtype(at::kByte));
  check_status(dsv4_sparse_attn(q.data_ptr(), kv.data_ptr(), sink.data_ptr<float>(), idx.data_ptr<int>(), B, S, H,
                                N, D, K, static_cast<float>(softmax_scale), out.data_ptr(), ws.data_ptr(), need,
                                stream_of(q)),
               "dsv4_sparse_attn");
  return out;
}

// The official linear for an FP8 weight: act_quant(x) then fp8_gemm with the
// weight's 128x128 ue8m0 block scales, given here as the atoms
// build_fp8_weight_atoms lays out once per weight.
at::Tensor build_fp8_weight_atoms(const at::Tensor& scale, int64_t out_features, int64_t in_features) {
  check_cuda(scale, "scale");
  c10::cuda::CUDAGuard guard(scale.device());
  const long long n = dsv4_fp8_weight_atoms_bytes(static_cast<int>(out_features), static_cast<int>(in_features));
  TORCH_CHECK(n > 0, "in and out features must be multiples of 128");
  at::Tensor atoms = at::empty({n}, scale.options().dtype(at::kByte));
  check_status(dsv4_build_fp8_weight_atoms(static_cast<const uint8_t*>(scale.data_ptr()),
                                           static_cast<int>(out_features), static_cast<int>(in_features),
                                           atoms.data_ptr<uint8_t>(), stream_of(scale)),
               "dsv4_build_fp8_weight_atoms");
  return atoms;
}

at::Tensor fp8_linear(const at::Tensor& x, const at::Tensor& weight, const at::Tensor& weight_atoms) {
  check_cuda(weight, "weight");
  check_cuda(weight_atoms, "weight_atoms");
  TORCH_CHECK(weight.dim() == 2 && weight.element_size() == 1, "weight must be [out, in] e4m3");
  const int64_t N = weight.size(0), K = weight.size(1);
  const at::Tensor x2 = bf16_rows(x, K).contiguous();
  c10::cuda::CUDAGuard guard(x2.device());
  const int M = static_cast<int>(x2.size(0));
  const long long need = dsv4_fp8_linear_workspace_bytes(M, static_cast<int>(N), static_cast<int>(K));
  TORCH_CHECK(need >= 0, "fp8_linear: out_features must be a multiple of 256, in_features of 512");
  at::Tensor ws = at::empty({std::max<long long>(need, 1)}, x2.options().dtype(at::kByte));
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape.back() = N;
  at::Tensor y = at::empty(shape, x2.options());
  check_status(dsv4_fp8_linear(x2.data_ptr(), M, static_cast<int>(K), static_cast<const uint8_t*>(weight.data_ptr()),
                               weight_atoms.data_ptr<uint8_t>(), static_cast<int>(N), y.data_ptr(), ws.data_ptr(),
                               need, stream_of(x2)),
               "dsv4_fp8_linear");
  return y;
}

// ---------------------------------------------------------- arena / materializer
int64_t materialize(const at::Tensor& slab, const at::Tensor& src_off, const at::Tensor& dst_slot,
                    const OptT& arena, int64_t slot_stride, const OptT& arena_sf, int64_t sf_slot_stride,
                    const OptT& bf16_out, int64_t bf16_slot_stride, int64_t hidden, int64_t inter) {
  check_cuda(slab, "slab");
  c10::cuda::CUDAGuard guard(slab.device());
  const at::Tensor off = src_off.to(slab.device(), at::kLong).contiguous();
  const at::Tensor slots = dst_slot.to(slab.device(), at::kInt).contiguous();
  TORCH_CHECK(off.numel() == slots.numel(), "targets and offsets length mismatch");
  const int n = static_cast<int>(off.numel());
  check_status(dsv4_materialize(slab.data_ptr<uint8_t>(), reinterpret_cast<const long long*>(off.data_ptr<int64_t>()),
                                slots.data_ptr<int>(), n, static_cast<int>(hidden), static_cast<int>(inter),
                                arena.has_value() ? arena->data_ptr<uint8_t>() : nullptr, slot_stride,
                                arena_sf.has_value() ? arena_sf->data_ptr<uint8_t>() : nullptr,
                                sf_slot_stride,
                                bf16_out.has_value() ? bf16_out->data_ptr() : nullptr, bf16_slot_stride,
                                stream_of(slab)),
               "dsv4_materialize");
  return static_cast<int64_t>(n) * (3 * inter * hidden / 32 + 3 * inter * hidden / 2);
}

void build_scale_atoms(const at::Tensor& arena, int64_t slot_stride, const at::Tensor& slots,
                       int64_t hidden, int64_t inter, at::Tensor& arena_sf, int64_t sf_slot_stride) {
  check_cuda(arena, "arena");
  c10::cuda::CUDAGuard guard(arena.device());
  const at::Tensor s = slots.to(arena.device(), at::kInt).contiguous();
  check_status(dsv4_build_scale_atoms(arena.data_ptr<uint8_t>(), slot_stride, s.data_ptr<int>(),
                                      static_cast<int>(s.numel()), static_cast<int>(hidden),
                                      static_cast<int>(inter), arena_sf.data_ptr<uint8_t>(), sf_slot_stride,
                                      stream_of(arena)),
               "dsv4_build_scale_atoms");
}

void build_shared_scale_atoms(const at::Tensor& w1_scale, const at::Tensor& w2_scale,
                              const at::Tensor& w3_scale, int64_t hidden, int64_t inter,
                              at::Tensor& shared_sf) {
  check_cuda(shared_sf, "shared_sf");
  c10::cuda::CUDAGuard guard(shared_sf.device());
  check_status(dsv4_build_shared_scale_atoms(static_cast<const uint8_t*>(w1_scale.data_ptr()),
                                             static_cast<const uint8_t*>(w2_scale.data_ptr()),
                                             static_cast<const uint8_t*>(w3_scale.data_ptr()),
                                             static_cast<int>(hidden), static_cast<int>(inter),
                                             shared_sf.data_ptr<uint8_t>(), stream_of(shared_sf)),
               "dsv4_build_shared_scale_atoms");
}

// ------------------------------------------------------------- expert parallelism
std::tuple<at::Tensor, at::Tensor, at::Tensor> ep_dispatch(const at::Tensor& x, const at::Tensor& indices,
                                                           const at::Tensor& weights, int64_t n_routed,
                                                           int64_t world) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  const int T = static_cast<int>(x.size(0)), H = static_cast<int>(x.size(1));
  const int k = static_cast<int>(indices.size(1));
  const long long row = dsv4_ep_row_bytes(H, k);
  TORCH_CHECK(row > 0, "dsv4_ep_row_bytes: unsupported hidden size / top-k");
  const int64_t rows = std::max<int64_t>((int64_t)T * std::min<int64_t>(world, k), 1);
  auto opts = x.options();
  at::Tensor send = at::empty({rows, row}, opts.dtype(at::kByte));
  at::Tensor counts = at::empty({world, 2}, opts.dtype(at::kInt));
  at::Tensor ret_pos = at::empty({std::max(T, 1), k}, opts.dtype(at::kInt));
  at::Tensor ws = workspace_for(std::nullopt, dsv4_ep_dispatch_workspace_bytes(T, (int)world), x);
  const at::Tensor idx = indices.to(at::kLong).contiguous();
  const at::Tensor wts = weights.to(at::kFloat).contiguous();
  check_status(dsv4_ep_dispatch(x.data_ptr(), idx.data_ptr<int64_t>(), wts.data_ptr<float>(), T, H, k,
                                (int)n_routed, (int)world, send.data_ptr(), rows, counts.data_ptr<int>(),
                                ret_pos.data_ptr<int>(), ws.data_ptr(), ws.numel(), stream_of(x)),
               "dsv4_ep_dispatch");
  return {send, counts, ret_pos};
}

std::tuple<at::Tensor, at::Tensor> ep_expert_forward(const TList& layer, at::IntArrayRef dims,
                                                     at::ArrayRef<double> scalars, int64_t rank,
                                                     int64_t world, const at::Tensor& x_own,
                                                     const at::Tensor& recv, const at::Tensor& recv_counts,
                                                     int64_t n_ret) {
  const dsv4_moe_layer L = make_layer(layer, dims, scalars);
  c10::cuda::CUDAGuard guard(x_own.device());
  const int T = static_cast<int>(x_own.size(0)), R = static_cast<int>(recv.size(0));
  const long long need = dsv4_ep_expert_workspace_bytes(&L, (int)world, T, R);
  at::Tensor ws = workspace_for(std::nullopt, need, x_own);
  at::Tensor ret = at::empty({n_ret, L.hidden}, x_own.options().dtype(at::kBFloat16));
  check_status(dsv4_ep_expert_forward(&L, (int)rank, (int)world, x_own.data_ptr(), T, recv.data_ptr(), R,
                                      recv_counts.data_ptr<int>(), ret.data_ptr(), n_ret, ws.data_ptr(),
                                      ws.numel(), stream_of(x_own)),
               "dsv4_ep_expert_forward");
  return {ret, ws};
}

at::Tensor ep_combine(const TList& layer, at::IntArrayRef dims, at::ArrayRef<double> scalars, int64_t rank,
                      int64_t world, const at::Tensor& ret_recv, const at::Tensor& ret_pos,
                      const at::Tensor& indices, const at::Tensor& x_own, int64_t R,
                      const at::Tensor& workspace) {
  const dsv4_moe_layer L = make_layer(layer, dims, scalars);
  c10::cuda::CUDAGuard guard(x_own.device());
  at::Tensor y = at::empty_like(x_own);
  const at::Tensor idx = indices.to(at::kLong).contiguous();
  check_status(dsv4_ep_combine(&L, (int)rank, (int)world, ret_recv.data_ptr(), ret_pos.data_ptr<int>(),
                               idx.data_ptr<int64_t>(), (int)x_own.size(0), (int)R, workspace.data_ptr(),
                               workspace.numel(), y.data_ptr(), stream_of(x_own)),
               "dsv4_ep_combine");
  return y;
}

// Peer-memory forms: `exchange` is this rank's exchange buffer (a device
// address from dsv4_ep_exchange_alloc), `peer_bases` the int64 device array of
// every rank's buffer as seen from this GPU.
at::Tensor ep_dispatch_p2p(const at::Tensor& x, const at::Tensor& indices, const at::Tensor& weights,
                           int64_t n_routed, int64_t world, int64_t rank, const at::Tensor& peer_bases,
                           int64_t cap, int64_t epoch) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  const int T = static_cast<int>(x.size(0)), H = static_cast<int>(x.size(1));
  const int k = static_cast<int>(indices.size(1));
  at::Tensor ret_pos = at::empty({std::max(T, 1), k}, x.options().dtype(at::kInt));
  at::Tensor ws = workspace_for(std::nullopt, dsv4_ep_p2p_dispatch_workspace_bytes(T, (int)world), x);
  const at::Tensor idx = indices.to(at::kLong).contiguous();
  const at::Tensor wts = weights.to(at::kFloat).contiguous();
  check_status(dsv4_ep_dispatch_p2p(x.data_ptr(), idx.data_ptr<int64_t>(), wts.data_ptr<float>(), T, H, k,
                                    (int)n_routed, (int)world, (int)rank,
                                    reinterpret_cast<const uint64_t*>(peer_bases.data_ptr<int64_t>()),
                                    (int)cap, (int)epoch, ret_pos.data_ptr<int>(), ws.data_ptr(),
                                    ws.numel(), stream_of(x)),
               "dsv4_ep_dispatch_p2p");
  return ret_pos;
}

void ep_expert_forward_p2p(const TList& layer, at::IntArrayRef dims, at::ArrayRef<double> scalars,
                           int64_t rank, int64_t world, const at::Tensor& x_own, int64_t exchange,
                           const at::Tensor& peer_bases, int64_t cap, int64_t epoch, at::Tensor& workspace) {
  const dsv4_moe_layer L = make_layer(layer, dims, scalars);
  c10::cuda::CUDAGuard guard(x_own.device());
  check_status(dsv4_ep_expert_forward_p2p(&L, (int)rank, (int)world, x_own.data_ptr(), (int)x_own.size(0),
                                          reinterpret_cast<void*>(exchange),
                                          reinterpret_cast<const uint64_t*>(peer_bases.data_ptr<int64_t>()),
                                          (int)cap, (int)epoch, workspace.data_ptr(), workspace.numel(),
                                          stream_of(x_own)),
               "dsv4_ep_expert_forward_p2p");
}

at::Tensor ep_combine_p2p(const TList& layer, at::IntArrayRef dims, at::ArrayRef<double> scalars, int64_t rank,
                          int64_t world, int64_t exchange, const at::Tensor& ret_pos, const at::Tensor& indices,
                          const at::Tensor& x_own, int64_t cap, int64_t epoch, const at::Tensor& workspace) {
  const dsv4_moe_layer L = make_layer(layer, dims, scalars);
  c10::cuda::CUDAGuard guard(x_own.device());
  at::Tensor y = at::empty_like(x_own);
  const at::Tensor idx = indices.to(at::kLong).contiguous();
  check_status(dsv4_ep_combine_p2p(&L, (int)rank, (int)world, reinterpret_cast<const void*>(exchange),
                                   ret_pos.data_ptr<int>(), idx.data_ptr<int64_t>(), (int)x_own.size(0),
                                   (int)cap, (int)epoch, workspace.data_ptr(), workspace.numel(), y.data_ptr(),
                                   stream_of(x_own)),
               "dsv4_ep_combine_p2p");
  return y;
}

// ------------------------------------------------------------------ loader
// native_packed_loader.cpp:26-68: EINTR-safe pread of up to `size` bytes at
// `offset` into a CPU uint8 tensor; returns the byte count (short at EOF).
int64_t read_into(int64_t fd, at::Tensor& destination, int64_t size, int64_t offset) {
  TORCH_CHECK(fd >= 0, "fd must be non-negative");
  TORCH_CHECK(size >= 0, "size must be non-negative");
  TORCH_CHECK(offset >= 0, "offset must be non-negative");
  TORCH_CHECK(destination.device().is_cpu(), "destination must be a CPU tensor");
  TORCH_CHECK(destination.scalar_type() == at::kByte, "destination must be uint8");
  TORCH_CHECK(destination.is_contiguous(), "destination must be contiguous");
  TORCH_CHECK(destination.numel() >= size, "destination tensor is too small");
  long long got = 0;
  int err = 0;
  const int rc = dsv4_read_into(static_cast<int>(fd), destination.data_ptr(), destination.numel(), size, offset,
                                &got, &err);
  TORCH_CHECK(rc != DSV4_ERR_IO, "pread failed: ", std::strerror(err ? err : EIO));
  check_status(rc, "read_into");
  return got;
}

}  // namespace

#define DSV4_LAYER_ARGS "Tensor?[] layer, int[] dims, float[] scalars"

TORCH_LIBRARY(dsv4moe, m) {
  m.def("moe_forward(Tensor x, " DSV4_LAYER_ARGS
        ", Tensor? routing_weights=None, Tensor? routing_indices=None, Tensor? workspace=None) -> Tensor");
  m.def("moe_forward_out(Tensor x, " DSV4_LAYER_ARGS
        ", Tensor? routing_weights, Tensor? routing_indices, Tensor? workspace, Tensor(a!) out) -> ()");
  m.def("moe_workspace_bytes(" DSV4_LAYER_ARGS ", int T) -> int");
  m.def("expert_forward(Tensor x, int expert, Tensor? row_weights, " DSV4_LAYER_ARGS ") -> Tensor");
  m.def("gate_route(Tensor x, Tensor weight, Tensor? bias, int topk, float route_scale, Tensor? tid2eid=None, "
        "Tensor? input_ids=None) -> (Tensor, Tensor, Tensor)");
  m.def("gate_logits(Tensor x, Tensor weight) -> Tensor");
  m.def("gate_topk(Tensor logits, Tensor? bias, int topk, float route_scale) -> (Tensor, Tensor)");
  m.def("act_quant(Tensor x) -> (Tensor, Tensor)");
  m.def("fp4_act_quant(Tensor x) -> (Tensor, Tensor)");
  m.def("materialize(Tensor slab, Tensor src_off, Tensor dst_slot, Tensor(a!)? arena, int slot_stride, "
        "Tensor(b!)? arena_sf, int sf_slot_stride, Tensor(c!)? bf16_out, int bf16_slot_stride, int hidden, "
        "int inter) -> int");
  m.def("build_scale_atoms(Tensor arena, int slot_stride, Tensor slots, int hidden, int inter, "
        "Tensor(a!) arena_sf, int sf_slot_stride) -> ()");
  m.def("build_shared_scale_atoms(Tensor w1_scale, Tensor w2_scale, Tensor w3_scale, int hidden, int inter, "
        "Tensor(a!) shared_sf) -> ()");
  m.def("ep_dispatch(Tensor x, Tensor indices, Tensor weights, int n_routed, int world) -> (Tensor, Tensor, Tensor)");
  m.def("ep_expert_forward(" DSV4_LAYER_ARGS
        ", int rank, int world, Tensor x_own, Tensor recv, Tensor recv_counts, int n_ret) -> (Tensor, Tensor)");
  m.def("ep_combine(" DSV4_LAYER_ARGS
        ", int rank, int world, Tensor ret_recv, Tensor ret_pos, Tensor indices, Tensor x_own, int R, "
        "Tensor workspace) -> Tensor");
  m.def("ep_dispatch_p2p(Tensor x, Tensor indices, Tensor weights, int n_routed, int world, int rank, "
        "Tensor peer_bases, int cap, int epoch) -> Tensor");
  m.def("ep_expert_forward_p2p(" DSV4_LAYER_ARGS
        ", int rank, int world, Tensor x_own, int exchange, Tensor peer_bases, int cap, int epoch, "
        "Tensor(a!) workspace) -> ()");
  m.def("ep_combine_p2p(" DSV4_LAYER_ARGS
        ", int rank, int world, int exchange, Tensor ret_pos, Tensor indices, Tensor x_own, int cap, int epoch, "
        "Tensor workspace) -> Tensor");
  m.def("read_into(int fd, Tensor(a!) destination, int size, int offset) -> int");
  m.def("sparse_attn(Tensor q, Tensor kv, Tensor attn_sink, Tensor topk_idxs, float softmax_scale) -> Tensor");
  m.def("build_fp8_weight_atoms(Tensor scale, int out_features, int in_features) -> Tensor");
  m.def("fp8_linear(Tensor x, Tensor weight, Tensor weight_atoms) -> Tensor");
}

TORCH_LIBRARY_IMPL(dsv4moe, CUDA, m) {
  m.impl("moe_forward", &moe_forward);
  m.impl("moe_forward_out", &moe_forward_out);
  m.impl("expert_forward", &expert_forward);
  m.impl("gate_route", &gate_route);
  m.impl("gate_logits", &gate_logits);
  m.impl("gate_topk", &gate_topk);
  m.impl("act_quant", &act_quant);
  m.impl("fp4_act_quant", &fp4_act_quant);
  m.impl("materialize", &materialize);
  m.impl("build_scale_atoms", &build_scale_atoms);
  m.impl("build_shared_scale_atoms", &build_shared_scale_atoms);
  m.impl("ep_dispatch", &ep_dispatch);
  m.impl("ep_expert_forward", &ep_expert_forward);
  m.impl("ep_combine", &ep_combine);
  m.impl("ep_dispatch_p2p", &ep_dispatch_p2p);
  m.impl("ep_expert_forward_p2p", &ep_expert_forward_p2p);
  m.impl("ep_combine_p2p", &ep_combine_p2p);
  m.impl("sparse_attn", &sparse_attn);
  m.impl("build_fp8_weight_atoms", &build_fp8_weight_atoms);
  m.impl("fp8_linear", &fp8_linear);
}

// Ops without tensor inputs on a device (sizes, host reads) dispatch here.
TORCH_LIBRARY_IMPL(dsv4moe, CompositeExplicitAutograd, m) {
  m.impl("moe_workspace_bytes", &moe_workspace_bytes);
  m.impl("read_into", &read_into);
}
