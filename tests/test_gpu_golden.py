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


@pytest.mark.parametrize("chunk", [1, 3, 16])
def test_pipelined_upload_reproduces_reference_bytes(cuda_device, chunk):
    """The chunked upload (pread of chunk i+1, H2D of chunk i on a copy stream,
    materializer of chunk i-1) with ragged chunks and a permuted slot order:
    every parameter's bytes equal what the reference store + loader
    materialized, and the copies and the materializer really overlap in
    order (no chunk read before its copy landed)."""
    from spark_b200.moe import ExpertArena
    from spark_b200.packed_store import PackedExpertStore, write_packed_layout
    from spark_b200.synthetic import CONFIGS, make_layer

    cfg = CONFIGS["cpu_ref"]
    layer = make_layer(cfg, seed=0, device="cpu")
    perm = np.random.default_rng(chunk).permutation(cfg.n_routed).tolist()
    with tempfile.TemporaryDirectory() as tmp:
        write_packed_layout(Path(tmp), {3: {e: layer["blocks"][e].numpy() for e in range(cfg.n_routed)}},
                            cfg.dim, cfg.inter)
        store = PackedExpertStore(Path(tmp) / "layout.json")
        arena = ExpertArena(cfg.n_routed, cfg.dim, cfg.inter, device=cuda_device)
        experts = list(range(cfg.n_routed))
        stats = store.upload_experts(3, experts, arena, perm, chunk_experts=chunk)
        store.close()
    assert stats["copied_bytes"] == FIX["slab_bytes"] and stats["packed_read_bytes"] == FIX["slab_bytes"]
    for e, s in zip(experts, perm):
        got = {n: _sha(p.data) for n, p in arena.expert_for_slot(s).named_parameters()}
        assert got == FIX["materialized_sha256"][str(e)], e


def test_loader_cuda_variants_reproduce_reference_bytes(cuda_device):
    """ExpertCopyPlan.read_into_and_copy_cuda and copy_storage_to_tensors_cuda
    (native_packed_loader.cpp:121-174,281-316: one cudaMemcpyAsync per target
    on the current stream) fill device parameters with the bytes the
    reference's own store + loader produced."""
    from spark_b200 import native_packed_loader as npl
    from spark_b200.moe import packed_block_layout
    from spark_b200.packed_store import PackedExpertStore, write_packed_layout
    from spark_b200.synthetic import CONFIGS, make_layer

    cfg = CONFIGS["cpu_ref"]
    layer = make_layer(cfg, seed=0, device="cpu")
    lay = packed_block_layout(cfg.dim, cfg.inter)
    names = ["w1.weight", "w1.scale", "w2.weight", "w2.scale", "w3.weight", "w3.scale"]
    with tempfile.TemporaryDirectory() as tmp:
        write_packed_layout(Path(tmp), {3: {e: layer["blocks"][e].numpy() for e in range(cfg.n_routed)}},
                            cfg.dim, cfg.inter)
        store = PackedExpertStore(Path(tmp) / "layout.json")
        store.native_cuda_memcpy = True  # DEEPSEEK_SPARK_NATIVE_CUDA_MEMCPY=1
        for e in range(cfg.n_routed):
            params = [(n, torch.nn.Parameter(torch.zeros(lay[n][3], dtype=torch.uint8, device=cuda_device),
                                             requires_grad=False)) for n in names]
            plan = store.native_plan_for_expert(3, e, f"layers.3.ffn.experts.{e}", params)
            if e % 2 == 0:  # fused pread + per-tensor device copies
                rb, cb, rs, cs = store.read_and_copy_with_plan(3, e, plan.plan, [p.data for _, p in params],
                                                               non_blocking=True)
                assert rb == cb == FIX["layout"]["layers"]["3"]["experts"][str(e)]["bytes"] and rs >= 0 and cs >= 0
            else:           # host block first, then the planned device copies
                batch = store.tensors_for_expert(3, e)
                n = store.copy_storage_with_plan(plan.plan, batch._storage, [p.data for _, p in params],
                                                 non_blocking=True)
                assert n == batch.read_bytes
            torch.cuda.current_stream().synchronize()
            assert {n: _sha(p.data) for n, p in params} == FIX["materialized_sha256"][str(e)], e
        # the CUDA variants reject host targets with the reference's message
        with pytest.raises(RuntimeError, match="CUDA memcpy target must be a CUDA tensor"):
            npl.ExpertCopyPlan([0], [8]).copy_storage_to_tensors_cuda(torch.zeros(8, dtype=torch.uint8),
                                                                     [torch.zeros(8, dtype=torch.uint8)])
        store.close()


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
