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

from . import _lib, ops

E4M3 = torch.float8_e4m3fn
E8M0 = torch.float8_e8m0fnu


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor, topk_idxs: torch.Tensor,
                softmax_scale: float) -> torch.Tensor:
    """q [B,S,H,D] bf16, kv [B,N,D] bf16, attn_sink [H], topk_idxs [B,S,K]
    (-1 = no row) -> [B,S,H,D] in q's dtype.  H = 64, D = 512.  Runs
    ``torch.ops.dsv4moe.sparse_attn`` (one call into ``dsv4_sparse_attn``)."""
    out = ops.load().sparse_attn(q.to(torch.bfloat16).contiguous(), kv.to(torch.bfloat16).contiguous(),
                                 attn_sink, topk_idxs, float(softmax_scale))
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
        if int(_lib.load().dsv4_fp8_weight_atoms_bytes(out_features, in_features)) <= 0:
            raise RuntimeError("FP8Linear needs in and out features that are multiples of 128")
        self.register_buffer("scale_atoms", torch.zeros(0, dtype=torch.uint8, device=device), persistent=False)
        self.register_load_state_dict_post_hook(lambda m, _keys: m.refresh_scale_atoms())
        self.refresh_scale_atoms()

    def refresh_scale_atoms(self) -> None:
        self.scale_atoms = ops.load().build_fp8_weight_atoms(self.scale, self.out_features, self.in_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """``torch.ops.dsv4moe.fp8_linear`` (act_quant + the FP8 GEMM) in bf16, cast to x's dtype."""
        y = ops.load().fp8_linear(x.to(torch.bfloat16).contiguous(), self.weight, self.scale_atoms)
        return y.to(x.dtype)
