"""CPU restatement of the attention block's two hot ops, for the tests only.

* ``sparse_attn``: the reference's correctness fallback for the official
  sparse attention (spark_runtime/lazy_official_runtime.py:1024-1049),
  restated in float64: for every (batch, query position) the valid (>= 0)
  indices select kv rows; scores = scale * q.kv per head; the max includes the
  head's sink logit; probabilities are exp(score - max) / (sum exp(score - max)
  + exp(sink - max)); the output is the probability-weighted sum of the rows,
  zeros when no index is valid.
* ``fp8_linear``: the official ``linear`` for an FP8 weight (act_quant(x, 128,
  "ue8m0") then fp8_gemm with 128x128 ue8m0 weight scales, kernel API at
  scripts/smoke_official_kernels.py:36-43), built from the MoE oracle's exact
  act_quant and FP8 dequantization.
"""

from __future__ import annotations

import numpy as np

from . import moe_oracle as O


def sparse_attn(q: np.ndarray, kv: np.ndarray, attn_sink: np.ndarray, topk_idxs: np.ndarray,
                softmax_scale: float) -> np.ndarray:
    """q [B,S,H,D], kv [B,N,D] (float values of the bf16 inputs), attn_sink [H],
    topk_idxs [B,S,K] -> float64 [B,S,H,D] (the device rounds it to bf16)."""
    B, S, H, D = q.shape
    out = np.zeros((B, S, H, D), np.float64)
    sink = np.asarray(attn_sink, np.float64)
    for b in range(B):
        for s in range(S):
            idx = np.asarray(topk_idxs[b, s])
            idx = idx[idx >= 0]
            if idx.size == 0:
                continue
            rows = kv[b, idx].astype(np.float64)                        # [k, D]
            scores = (q[b, s].astype(np.float64) @ rows.T) * softmax_scale  # [H, k]
            m = np.maximum(scores.max(axis=1), sink)
            e = np.exp(scores - m[:, None])
            den = e.sum(axis=1) + np.exp(sink - m)
            out[b, s] = (e / den[:, None]) @ rows
    return out


def fp8_linear(x_bf16: np.ndarray, w_codes: np.ndarray, w_scale: np.ndarray) -> np.ndarray:
    """y [M,N] (bf16 values as float32) = act_quant(x) . dequant(W)^T."""
    return O.quantized_linear(np.asarray(x_bf16, np.float32), O.dequant_fp8_weight(w_codes, w_scale))
