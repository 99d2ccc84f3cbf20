"""GPU results against the reference's own outputs (tests/golden/)."""

import hashlib
import json
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
FIX = json.loads((GOLDEN / "cpu_ref_seed0.json").read_text())
NPZ = np.load(GOLDEN / "cpu_ref_seed0.npz")
TOL = 2e-2


def _sha(t) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()


def test_device_materializer_reproduces_reference_bytes(cuda_device):
    """Slab written in the reference format -> pinned read -> one H2D copy ->
    device materializer into arena slots (reversed order): every parameter's
    bytes equal what the reference store + loader materialized."""
    from spark_b200.moe import ExpertArena
    from spark_b200.packed_store import PackedExpertStore, write_packed_layout
    from spark_b200.synthetic import CONFIGS, make_layer

    cfg = CONFIGS["cpu_ref"]
    layer = make_layer(cfg, seed=0, device="cpu")
    with tempfile.TemporaryDirectory() as tmp:
        write_packed_layout(Path(tmp), {3: {e: layer["blocks"][e].numpy() for e in range(cfg.n_routed)}},
                            cfg.dim, cfg.inter)
        store = PackedExpertStore(Path(tmp) / "layout.json")
        arena = ExpertArena(cfg.n_routed, cfg.dim, cfg.inter, device=cuda_device)
        experts = list(range(cfg.n_routed))
        slots = experts[::-1]
        stats = store.upload_experts(3, experts, arena, slots)
        store.close()
    assert stats["copied_bytes"] == FIX["slab_bytes"]
    for e, s in zip(experts, slots):
        ex = arena.expert_for_slot(s)
        got = {n: _sha(p.data) for n, p in ex.named_parameters()}
        assert got == FIX["materialized_sha256"][str(e)], e


def test_layer_output_matches_reference_lazymoe(cuda_device):
    """The B200 layer (gate, routing, grouped FP4/FP8 GEMMs, combine) against
    the output of the reference's LazyMoE.forward on the same inputs."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["cpu_ref"]
    layer = make_layer(cfg, seed=0, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].view(1, cfg.tokens, cfg.dim).to(cuda_device)
    w, idx = moe.gate(x.view(-1, cfg.dim))
    assert np.array_equal(idx.cpu().numpy(), NPZ["indices"])
    y = moe(x, torch.arange(cfg.tokens, device=cuda_device).view(1, -1))
    torch.cuda.synchronize()
    ref = O.bf16_bits_to_f32(NPZ["y_bits"])
    got = y.float().cpu().numpy().reshape(cfg.tokens, -1)
    err = float(np.max(np.abs(got - ref)) / np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    assert err <= TOL, err
