"""``torch.ops.dsv4moe``: the torch custom-op layer over libdsv4moe.so.

``load()`` loads lib/libdsv4moe_torch.so (``TORCH_LIBRARY(dsv4moe)``, built
from csrc/torch_ops.cpp) and registers a fake kernel for every op that
returns tensors, so the ops run under FakeTensor / meta tracing with the right
output shapes.  The CUDA kernels of the ops are single calls into the C ABI of
libdsv4moe.so on torch's current stream; a non-zero status raises
RuntimeError.  There is no other implementation: on a machine where the op
library is missing, ``load()`` raises.

A MoE layer crosses the boundary as three lists (``layer_args``):

* ``layer``   - 9 optional tensors: gate_w, gate_bias, arena, arena_sf,
  expert_slot, shared_w1, shared_w2, shared_w3, shared_sf
* ``dims``    - hidden, inter, n_routed, topk, n_shared, n_slots,
  slot_stride, sf_slot_stride
* ``scalars`` - route_scale, swiglu_limit
"""

from __future__ import annotations

import threading

import torch

from . import _lib

OPS_LIB = _lib.PKG_ROOT / "lib" / "libdsv4moe_torch.so"
_lock = threading.Lock()
_loaded = False


def load():
    """Load the op library once and return the ``torch.ops.dsv4moe`` namespace."""
    global _loaded
    with _lock:
        if not _loaded:
            if not OPS_LIB.exists():
                raise RuntimeError(f"{OPS_LIB} is missing: build it with "
                                   "`python deepseek-v4-flash-dgx-spark_b200/build.py`")
            _lib.load()
            torch.ops.load_library(str(OPS_LIB))
            _register_fakes()
            _loaded = True
    return torch.ops.dsv4moe


def layer_args(d: "_lib.MoELayerDesc", tensors: list) -> tuple[list, list[int], list[float]]:
    """The op layer's three lists from a C ABI layer description and the
    tensors whose pointers it holds (same order as ``layer``)."""
    dims = [d.hidden, d.inter, d.n_routed, d.topk, d.n_shared, d.n_slots, d.slot_stride, d.sf_slot_stride]
    return tensors, [int(v) for v in dims], [float(d.route_scale), float(d.swiglu_limit)]


def _register_fakes() -> None:
    lib = "dsv4moe::"

    def fake(name):
        return torch.library.register_fake(lib + name)

    @fake("moe_forward")
    def _(x, layer, dims, scalars, routing_weights=None, routing_indices=None, workspace=None):
        return torch.empty_like(x)

    @fake("moe_forward_out")
    def _(x, layer, dims, scalars, routing_weights, routing_indices, workspace, out):
        return None

    @fake("expert_forward")
    def _(x, expert, row_weights, layer, dims, scalars):
        return torch.empty_like(x)

    @fake("gate_route")
    def _(x, weight, bias, topk, route_scale, tid2eid=None, input_ids=None):
        T = x.numel() // weight.shape[1]
        E = weight.shape[0]
        return (x.new_empty((T, topk), dtype=torch.float32), x.new_empty((T, topk), dtype=torch.int64),
                x.new_empty((T, E), dtype=torch.float32))

    @fake("gate_logits")
    def _(x, weight):
        return x.new_empty((x.numel() // weight.shape[1], weight.shape[0]), dtype=torch.float32)

    @fake("gate_topk")
    def _(logits, bias, topk, route_scale):
        T = logits.shape[0]
        return logits.new_empty((T, topk)), logits.new_empty((T, topk), dtype=torch.int64)

    @fake("act_quant")
    def _(x):
        K = x.shape[-1]
        M = x.numel() // K
        return x.new_empty((M, K), dtype=torch.uint8), x.new_empty((M, K // 128), dtype=torch.uint8)

    @fake("fp4_act_quant")
    def _(x):
        K = x.shape[-1]
        M = x.numel() // K
        return x.new_empty((M, K // 2), dtype=torch.uint8), x.new_empty((M, K // 32), dtype=torch.uint8)

    @fake("ep_dispatch_p2p")
    def _(x, indices, weights, n_routed, world, rank, peer_bases, cap, epoch):
        return x.new_empty((max(x.shape[0], 1), indices.shape[1]), dtype=torch.int32)

    @fake("ep_combine_p2p")
    def _(layer, dims, scalars, rank, world, exchange, ret_pos, indices, x_own, cap, epoch, workspace):
        return torch.empty_like(x_own)

    @fake("ep_combine")
    def _(layer, dims, scalars, rank, world, ret_recv, ret_pos, indices, x_own, R, workspace):
        return torch.empty_like(x_own)

    @fake("sparse_attn")
    def _(q, kv, attn_sink, topk_idxs, softmax_scale):
        return torch.empty_like(q)

    @fake("build_fp8_weight_atoms")
    def _(scale, out_features, in_features):
        n = int(_lib.load().dsv4_fp8_weight_atoms_bytes(out_features, in_features))
        return scale.new_empty((n,), dtype=torch.uint8)

    @fake("fp8_linear")
    def _(x, weight, weight_atoms):
        return x.new_empty((*x.shape[:-1], weight.shape[0]))
