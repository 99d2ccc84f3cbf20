"""The attention oracle pinned to the reference: oracle/attention_oracle.py's
sparse attention against the output bits of the reference's own
sparse_attn_fallback (tests/golden/make_attention_golden.py), and its FP8
linear against the MoE oracle's exact pieces.  CPU only."""

from pathlib import Path

import numpy as np
import torch

from oracle import attention_oracle as A
from oracle import moe_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "sparse_attn_ref.npz"


def _bf16(a):
    return torch.from_numpy(a).view(torch.bfloat16).float().numpy()


def test_sparse_attn_oracle_reproduces_the_reference_fallback():
    z = np.load(GOLDEN)
    got = A.sparse_attn(_bf16(z["q"]), _bf16(z["kv"]), z["sink"], z["idx"], float(z["scale"]))
    ref = _bf16(z["out"])
    # the reference rounds to bf16 once at the end; the oracle keeps float64
    assert np.array_equal(O.round_bf16(got.astype(np.float32)), ref)
    assert np.all(ref[1, 2] == 0)  # a query with no valid index gives zeros


def test_fp8_linear_oracle_is_act_quant_then_exact_fp8_gemm():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 512, generator=g).to(torch.bfloat16).float().numpy()
    w = torch.randn(256, 512, generator=g).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    s = torch.randint(119, 124, (2, 4), generator=g, dtype=torch.uint8).numpy()
    y = A.fp8_linear(x, w, s)
    q, qs = O.act_quant(x)
    ref = O.round_bf16((O.act_dequant(q, qs).astype(np.float64) @ O.dequant_fp8_weight(w, s).astype(np.float64).T)
                       .astype(np.float32))
    assert np.array_equal(y, ref)
