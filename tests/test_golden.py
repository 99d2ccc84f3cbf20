"""Pins against the reference's own outputs (tests/golden/, made by
tests/golden/make_golden.py from the reference's layout builder, packed store,
C++ loader and LazyMoE.forward).  CPU only."""

import hashlib
import json
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
FIX = json.loads((GOLDEN / "cpu_ref_seed0.json").read_text())
NPZ = np.load(GOLDEN / "cpu_ref_seed0.npz")


def _sha(t) -> str:
    if isinstance(t, torch.Tensor):
        t = t.contiguous().view(torch.uint8).numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def layer():
    from spark_b200.synthetic import CONFIGS, make_layer

    return make_layer(CONFIGS["cpu_ref"], seed=0, device="cpu")


def test_seeded_inputs_match_the_fixture(layer):
    got = {"x": _sha(layer["x"]), "gate_w": _sha(layer["gate_w"]), "gate_bias": _sha(layer["gate_bias"]),
           "blocks": _sha(layer["blocks"]), **{f"shared.{k}": _sha(v) for k, v in layer["shared"].items()}}
    assert got == FIX["inputs"]


def _mw(layer):
    cfg = layer["cfg"]
    return O.MoEWeights(
        gate_w=layer["gate_w"].float().numpy(), gate_bias=layer["gate_bias"].numpy(),
        experts={e: O.expert_from_block(layer["blocks"][e].numpy(), cfg.dim, cfg.inter) for e in range(cfg.n_routed)},
        shared=O.shared_from_tensors({k: v.numpy() for k, v in layer["shared"].items()}),
        topk=cfg.topk, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)


def test_oracle_gate_matches_reference_run(layer):
    w, idx, logits = O.gate_forward(layer["x"].float().numpy(), layer["gate_w"].float().numpy(),
                                    layer["gate_bias"].numpy(), 4, 2.5)
    assert np.array_equal(idx, NPZ["indices"])
    assert np.array_equal(w.view(np.uint32), NPZ["weights"].view(np.uint32))


def test_oracle_layer_is_bit_identical_to_reference_lazymoe(layer):
    """The reference's LazyMoE.forward (dispatch by torch.where, fp32 y[idx] +=
    in expert order, + shared, cast) run with the oracle's Gate/Expert; the
    oracle's own combine must reproduce its bits exactly."""
    y = O.moe_forward(layer["x"].float().numpy(), _mw(layer))[0]
    assert np.array_equal(O.f32_to_bf16_bits(y), NPZ["y_bits"])


def test_layout_writer_matches_reference_builder(layer):
    from spark_b200.packed_store import write_packed_layout

    cfg = layer["cfg"]
    with tempfile.TemporaryDirectory() as tmp:
        lay = write_packed_layout(Path(tmp), {3: {e: layer["blocks"][e].numpy() for e in range(cfg.n_routed)}},
                                  cfg.dim, cfg.inter)
        slab = (Path(tmp) / "layer_03.bin").read_bytes()
    assert hashlib.sha256(slab).hexdigest() == FIX["slab_sha256"]
    assert {k: v for k, v in lay.items() if k not in ("created_at_unix", "model_dir", "manifest_csv")} == FIX["layout"]


def test_loader_mirror_materializes_reference_bytes(layer):
    """PackedExpertStore + ExpertCopyPlan.read_into_and_copy of the drop-in
    loader fill CPU parameters with the bytes the reference loader produced."""
    from spark_b200.packed_store import PackedExpertStore, write_packed_layout

    cfg = layer["cfg"]
    with tempfile.TemporaryDirectory() as tmp:
        write_packed_layout(Path(tmp), {3: {e: layer["blocks"][e].numpy() for e in range(cfg.n_routed)}},
                            cfg.dim, cfg.inter)
        store = PackedExpertStore(Path(tmp) / "layout.json")
        names = ["w1.weight", "w1.scale", "w2.weight", "w2.scale", "w3.weight", "w3.scale"]
        from spark_b200.moe import packed_block_layout

        lay = packed_block_layout(cfg.dim, cfg.inter)
        for e in range(cfg.n_routed):
            params = [(n, torch.nn.Parameter(torch.zeros(lay[n][3], dtype=torch.uint8), requires_grad=False))
                      for n in names]
            plan = store.native_plan_for_expert(3, e, f"layers.3.ffn.experts.{e}", params)
            assert plan.fallback_indices == ()
            rb, cb, _, _ = store.read_and_copy_with_plan(3, e, plan.plan, [p.data for _, p in params],
                                                         non_blocking=False)
            assert rb == cb == FIX["layout"]["layers"]["3"]["experts"][str(e)]["bytes"]
            assert {n: _sha(p.data) for n, p in params} == FIX["materialized_sha256"][str(e)]
        store.close()


def test_threaded_block_reads_give_the_same_bytes(layer):
    """read_blocks preads up to read_threads blocks at once; the buffer equals
    a one-thread read byte for byte, and a short read still raises."""
    from spark_b200.packed_store import PackedExpertStore, write_packed_layout

    cfg = layer["cfg"]
    with tempfile.TemporaryDirectory() as tmp:
        write_packed_layout(Path(tmp), {3: {e: layer["blocks"][e].numpy() for e in range(cfg.n_routed)}},
                            cfg.dim, cfg.inter)
        experts = list(range(cfg.n_routed))[::-1]
        bufs = []
        for threads in (1, 4):
            store = PackedExpertStore(Path(tmp) / "layout.json")
            store.read_threads = threads
            buf, offs, _ = store.read_blocks(3, experts)
            bufs.append((buf.clone(), offs))
            store.close()
        assert bufs[0][1] == bufs[1][1] and torch.equal(bufs[0][0], bufs[1][0])
        for e, o in zip(experts, bufs[1][1]):
            blk = layer["blocks"][e].numpy().reshape(-1)
            assert np.array_equal(bufs[1][0][o:o + blk.size].numpy(), blk)
        # truncate the slab: the threaded read reports the short read
        slab = next(Path(tmp).glob("*.bin"))
        with open(slab, "r+b") as f:
            f.truncate(slab.stat().st_size // 2)
        store = PackedExpertStore(Path(tmp) / "layout.json")
        store.read_threads = 4
        with pytest.raises(RuntimeError, match="short packed expert read"):
            store.read_blocks(3, experts)
        store.close()


def test_loader_mirror_error_messages():
    from spark_b200 import native_packed_loader as npl

    plan = npl.ExpertCopyPlan([0, 8], [8, 8])
    storage = torch.zeros(12, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="source slice exceeds storage tensor"):
        plan.copy_storage_to_tensors(storage, [torch.zeros(8, dtype=torch.uint8)] * 2, False)
    with pytest.raises(RuntimeError, match="target size does not match expert copy plan"):
        plan.copy_storage_to_tensors(torch.zeros(32, dtype=torch.uint8), [torch.zeros(4, dtype=torch.uint8)] * 2,
                                     False)
    with pytest.raises(RuntimeError, match="copy-plan offset must be non-negative"):
        npl.ExpertCopyPlan([-1], [1])
    with tempfile.NamedTemporaryFile() as f:
        f.write(b"x" * 10)
        f.flush()
        fd = os.open(f.name, os.O_RDONLY)
        try:
            with pytest.raises(RuntimeError, match="short packed expert read"):
                plan.read_into_and_copy(fd, torch.zeros(16, dtype=torch.uint8), 16, 0,
                                        [torch.zeros(8, dtype=torch.uint8)] * 2, False)
            assert npl.read_into(fd, torch.zeros(16, dtype=torch.uint8), 16, 4) == 6
        finally:
            os.close(fd)


def _ref_loader():
    so = sorted((Path(__file__).resolve().parent.parent / "oracle" / "_ref").glob("native_packed_loader_ref*.so"))
    if not so:
        pytest.skip("reference loader not built (make -C oracle)")
    import importlib.util

    spec = importlib.util.spec_from_file_location("native_packed_loader_ref", so[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_pread_failure_raises_like_the_reference_loader():
    """A failed pread (a bad descriptor) raises RuntimeError with the same
    message in the drop-in loader and in the reference loader compiled from
    its own source."""
    from spark_b200 import native_packed_loader as npl

    ref = _ref_loader()
    msgs = []
    for mod in (ref, npl):
        with pytest.raises(RuntimeError) as info:
            mod.read_into(987654, torch.zeros(16, dtype=torch.uint8), 8, 0)
        msgs.append(str(info.value))
    assert msgs[0] == msgs[1] == "pread failed: Bad file descriptor"


def test_loader_mirror_agrees_with_compiled_reference_loader():
    """Same return values and copies as the reference C++ loader compiled from
    its own source (oracle/_ref), on a random block and plan."""
    ref = _ref_loader()
    from spark_b200 import native_packed_loader as npl

    rng = np.random.default_rng(3)
    data = rng.integers(0, 256, 4096, dtype=np.uint8)
    offsets, sizes = [0, 100, 1000, 3000], [100, 900, 2000, 1096]
    with tempfile.NamedTemporaryFile() as f:
        f.write(b"\0" * 512 + data.tobytes())
        f.flush()
        fd = os.open(f.name, os.O_RDONLY)
        try:
            outs = []
            for mod in (ref, npl):
                plan = mod.ExpertCopyPlan(offsets, sizes)
                tg = [torch.zeros(s, dtype=torch.uint8) for s in sizes]
                rb, cb, _, _ = plan.read_into_and_copy(fd, torch.zeros(4096, dtype=torch.uint8), 4096, 512, tg, False)
                outs.append((rb, cb, [t.numpy().tobytes() for t in tg], plan.count))
                assert mod.read_into(fd, torch.zeros(64, dtype=torch.uint8), 64, 4096 + 512 - 10) == 10
            assert outs[0] == outs[1]
        finally:
            os.close(fd)
