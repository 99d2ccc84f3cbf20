"""Golden vectors of the reference's sparse attention fallback.

    python tests/golden/make_attention_golden.py --reference <checkout of the reference> (or $REFERENCE_DIR)

Runs the reference's own ``sparse_attn_fallback``
(spark_runtime/lazy_official_runtime.py:1024-1049) on the CPU on small seeded
inputs (some indices -1, one query with no valid index, a nonzero sink) and
stores inputs and output bits in tests/golden/sparse_attn_ref.npz; the
oracle's restatement (oracle/attention_oracle.py) is pinned to them.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_DIR"), required="REFERENCE_DIR" not in os.environ)
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference)))
    from spark_runtime.lazy_official_runtime import sparse_attn_fallback

    g = torch.Generator().manual_seed(7)
    B, S, H, D, N, K = 2, 3, 4, 64, 20, 8
    q = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    kv = torch.randn(B, N, D, generator=g).to(torch.bfloat16)
    sink = torch.randn(H, generator=g)
    idx = torch.randint(0, N, (B, S, K), generator=g, dtype=torch.int32)
    idx[0, 1, ::3] = -1
    idx[1, 2, :] = -1  # no valid index: zeros
    scale = D ** -0.5
    out = sparse_attn_fallback(q, kv, sink, idx, scale)
    np.savez_compressed(HERE / "sparse_attn_ref.npz", q=q.view(torch.int16).numpy(), kv=kv.view(torch.int16).numpy(),
                        sink=sink.numpy(), idx=idx.numpy(), scale=np.float64(scale),
                        out=out.view(torch.int16).numpy())
    print("wrote", HERE / "sparse_attn_ref.npz")


if __name__ == "__main__":
    main()
