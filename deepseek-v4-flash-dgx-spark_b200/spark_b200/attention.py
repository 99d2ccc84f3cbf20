"""The attention block's hot ops of DeepSeek-V4-Flash on B200.

* ``sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale)``: drop-in for the
  official ``kernel.sparse_attn`` and for the reference's replacement of it,
  ``sparse_attn_fallback`` (spark_runtime/lazy_official_runtime.py:1016-1049,
  installed by ``import_official_model`` at :1020).  Same arguments and
  result; the work is one tcgen05 kernel (csrc/sparse_attn.cu) instead of a
  Python loop over tokens.
* ``FP8Linear(in_features, out_features)``: the official linear layer with an
  FP8 e4m3 weight and 128x128 ue8m0 block scales (parameters ``weight`` and
  ``scale``, as the checkpoint's ``layers.L.attn.{wq_a, wq_b, wkv, wo_a,
  wo_b}``); forward = act_quant + FP8 GEMM on the tensor core.

To use them in the reference runtime: ``official_model.sparse_attn =
spark_b200.attention.sparse_attn`` where ``import_official_model`` installs
its fallback.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib
from ._lib import check, ptr, stream_ptr

E4M3 = torch.float8_e4m3fn
E8M0 = torch.float8_e8m0fnu


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor, topk_idxs: torch.Tensor,
                softmax_scale: float) -> torch.Tensor:
    """q [B,S,H,D] bf16, kv [B,N,D] bf16, attn_sink [H], topk_idxs [B,S,K]
    (-1 = no row) -> [B,S,H,D] in q's dtype.  H = 64, D = 512."""
    B, S, H, D = q.shape
    N, K = kv.shape[1], topk_idxs.shape[-1]
    qb = q.to(torch.bfloat16).contiguous()
    kvb = kv.to(torch.bfloat16).contiguous()
    sink = attn_sink.to(device=q.device, dtype=torch.float32).contiguous()
    idx = topk_idxs.to(device=q.device, dtype=torch.int32).contiguous()
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=q.device)
    lib = _lib.load()
    need = int(lib.dsv4_sparse_attn_workspace_bytes(B, S, K))
    if need < 0:
        raise RuntimeError("dsv4_sparse_attn_workspace_bytes: invalid shape")
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device) if need else None
    check(lib.dsv4_sparse_attn(ptr(qb), ptr(kvb), ptr(sink), ptr(idx), B, S, H, N, D, K, float(softmax_scale),
                               ptr(out), ptr(ws), need, stream_ptr()), "dsv4_sparse_attn")
    return out.to(q.dtype)


class FP8Linear(nn.Module):
    """Official ``Linear(in_features, out_features)`` with an FP8 weight:
    ``weight`` e4m3 [out, in], ``scale`` ue8m0 [out/128, in/128].  Call
    ``refresh_scale_atoms()`` after writing them (``load_state_dict`` does)."""

    def __init__(self, in_features: int, out_features: int, *, device=None):
        super().__init__()
        device = torch.device(device) if device is not None else torch.device("cuda")
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.zeros(out_features, in_features, dtype=torch.uint8, device=device).view(E4M3),
                                   requires_grad=False)
        self.scale = nn.Parameter(torch.full((out_features // 128, in_features // 128), 127, dtype=torch.uint8,
                                             device=device).view(E8M0), requires_grad=False)
        n = int(_lib.load().dsv4_fp8_weight_atoms_bytes(out_features, in_features))
        if n <= 0:
            raise RuntimeError("FP8Linear needs in and out features that are multiples of 128")
        self.register_buffer("scale_atoms", torch.zeros(n, dtype=torch.uint8, device=device), persistent=False)
        self.register_load_state_dict_post_hook(lambda m, _keys: m.refresh_scale_atoms())
        self.refresh_scale_atoms()

    def refresh_scale_atoms(self) -> None:
        check(_lib.load().dsv4_build_fp8_weight_atoms(ptr(self.scale), self.out_features, self.in_features,
                                                      ptr(self.scale_atoms), stream_ptr()),
              "dsv4_build_fp8_weight_atoms")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.in_features).to(torch.bfloat16).contiguous()
        M = x2.shape[0]
        y = torch.empty((M, self.out_features), dtype=torch.bfloat16, device=x2.device)
        lib = _lib.load()
        need = int(lib.dsv4_fp8_linear_workspace_bytes(M, self.out_features, self.in_features))
        if need < 0:
            raise RuntimeError("FP8Linear: out_features must be a multiple of 256, in_features of 512")
        ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x2.device)
        check(lib.dsv4_fp8_linear(ptr(x2), M, self.in_features, ptr(self.weight), ptr(self.scale_atoms),
                                  self.out_features, ptr(y), ptr(ws), need, stream_ptr()), "dsv4_fp8_linear")
        return y.view(*shape[:-1], self.out_features).to(x.dtype)
