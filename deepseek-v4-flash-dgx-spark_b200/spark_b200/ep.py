"""Expert-parallel MoE layer: dispatch / owning-rank forward / combine.

The reference shards experts by rank (rank r of W owns experts
[r*E/W, (r+1)*E/W), spark_runtime/lazy_official_runtime.py:956-965) but keeps
every token on every rank and all-reduces the fp32 partial outputs
(``dist.all_reduce(y)``, :999-1000).  Here each rank routes only its own tokens
and moves only what the routing needs, in five steps per layer:

1. ``dispatch`` (device): every token is act-quantized once and written once
   per rank that owns one of its experts (FP8 codes + ue8m0 scales + route
   entries), plus ``send_counts[W][2]`` (rows, routes) and ``ret_pos``.
2. all-to-all of the counts, one host read of both count tables (the only host
   synchronisation), all-to-all of the rows.
3. ``expert_forward`` (device, owning rank): received rows through the grouped
   expert GEMMs together with the rank's own tokens for the shared expert;
   every route's bf16 output row lands in the return buffer.
4. all-to-all of the return rows.
5. ``combine`` (device, source rank): the single-GPU combine over the returned
   rows, so the result is bit-identical to the single-GPU layer.

The device work sits behind an ``ops`` object; ``CudaEPOps`` drives
libdsv4moe.so, and the CPU tests substitute an implementation of the same
buffer formats to exercise this orchestration over ``gloo``.  Row exchanges
carry bf16 rows as their bytes so every backend moves them unchanged.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, ptr, stream_ptr


class CudaEPOps:
    """Device steps of one expert-parallel layer call through the C ABI."""

    def __init__(self, moe):
        self.moe = moe
        self.world, self.rank = moe.world, moe.rank
        self.hidden, self.topk = moe.dim, moe.n_activated_experts
        self.n_routed = moe.n_routed_experts
        self.lib = _lib.load()
        self.row_bytes = int(self.lib.dsv4_ep_row_bytes(self.hidden, self.topk))
        if self.row_bytes <= 0:
            raise RuntimeError("dsv4_ep_row_bytes: unsupported hidden size / top-k")
        self._ws = None
        self._desc = None

    def empty(self, shape, dtype, like):
        return torch.empty(shape, dtype=dtype, device=like.device)

    def gate(self, x):
        return self.moe.gate(x)

    def dispatch(self, x, weights, indices):
        T, W, k = x.shape[0], self.world, self.topk
        send = torch.empty((max(T * min(W, k), 1), self.row_bytes), dtype=torch.uint8, device=x.device)
        counts = torch.empty((W, 2), dtype=torch.int32, device=x.device)
        ret_pos = torch.empty((max(T, 1), k), dtype=torch.int32, device=x.device)
        ws = torch.empty(max(int(self.lib.dsv4_ep_dispatch_workspace_bytes(T, W)), 1), dtype=torch.uint8,
                         device=x.device)
        weights = weights.to(torch.float32).contiguous()
        indices = indices.to(torch.int64).contiguous()
        check(self.lib.dsv4_ep_dispatch(ptr(x), ptr(indices), ptr(weights), T, self.hidden, k, self.n_routed, W,
                                        ptr(send), send.shape[0], ptr(counts), ptr(ret_pos), ptr(ws), ws.numel(),
                                        stream_ptr()), "dsv4_ep_dispatch")
        return send, counts, ret_pos

    def expert_forward(self, x, recv, recv_counts, n_ret):
        T, R = x.shape[0], recv.shape[0]
        self._desc = self.moe.layer_desc()
        need = int(self.lib.dsv4_ep_expert_workspace_bytes(ctypes.byref(self._desc), self.world, T, R))
        if need < 0:
            raise RuntimeError("dsv4_ep_expert_workspace_bytes: invalid layer")
        ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        ret_send = torch.empty((n_ret, self.hidden), dtype=torch.bfloat16, device=x.device)
        check(self.lib.dsv4_ep_expert_forward(ctypes.byref(self._desc), self.rank, self.world, ptr(x), T,
                                              ptr(recv), R, ptr(recv_counts), ptr(ret_send), n_ret, ptr(ws),
                                              ws.numel(), stream_ptr()), "dsv4_ep_expert_forward")
        return ret_send, ws

    def combine(self, ret_recv, ret_pos, indices, x, R, state):
        ws = state
        y = torch.empty_like(x)
        indices = indices.to(torch.int64).contiguous()
        check(self.lib.dsv4_ep_combine(ctypes.byref(self._desc), self.rank, self.world, ptr(ret_recv), ptr(ret_pos),
                                       ptr(indices), x.shape[0], R, ptr(ws), ws.numel(), ptr(y), stream_ptr()),
              "dsv4_ep_combine")
        return y


def _a2a_rows(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group) -> None:
    """all-to-all of whole rows (splits in rows); bf16 rows travel as their bytes."""
    def as_bytes(t: torch.Tensor) -> torch.Tensor:
        if t.numel() == 0:  # an empty tensor may carry strides a byte view rejects
            return torch.empty((t.shape[0], t.shape[1] * t.element_size()), dtype=torch.uint8, device=t.device)
        return t.contiguous().view(torch.uint8)

    if out.dtype == torch.bfloat16:
        out_b = as_bytes(out)
        dist.all_to_all_single(out_b, as_bytes(inp), list(out_splits), list(in_splits), group=group)
        if out.numel() and out_b.data_ptr() != out.data_ptr():
            out.view(torch.uint8).copy_(out_b)
        return
    dist.all_to_all_single(out, inp, list(out_splits), list(in_splits), group=group)


def ep_forward(ops, x: torch.Tensor, group=None, routing=None) -> torch.Tensor:
    """One expert-parallel layer call over this rank's tokens x [T, H] bf16.

    Every rank of ``group`` must call it (with its own T, possibly 0); the
    collectives run in the same order on every rank."""
    W = ops.world
    if routing is None:
        weights, indices = ops.gate(x)
    else:
        weights, indices = routing
    send, send_counts, ret_pos = ops.dispatch(x, weights, indices)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    both = torch.stack([send_counts, recv_counts]).cpu()  # the one host synchronisation
    s_rows, s_routes = both[0, :, 0].tolist(), both[0, :, 1].tolist()
    r_rows, r_routes = both[1, :, 0].tolist(), both[1, :, 1].tolist()
    R = sum(r_rows)
    recv = ops.empty((R, send.shape[1]), send.dtype, send)
    _a2a_rows(recv, send[: sum(s_rows)], r_rows, s_rows, group)
    ret_send, state = ops.expert_forward(x, recv, recv_counts, sum(r_routes))
    ret_recv = ops.empty((sum(s_routes), ret_send.shape[1]), ret_send.dtype, ret_send)
    _a2a_rows(ret_recv, ret_send, s_routes, r_routes, group)
    return ops.combine(ret_recv, ret_pos, indices, x, R, state)


def ep_moe_forward(moe, x: torch.Tensor, routing=None) -> torch.Tensor:
    """``MoE.forward`` body for world > 1 (x [T, H] bf16 on this rank's GPU)."""
    return ep_forward(CudaEPOps(moe), x, group=moe.group, routing=routing)
