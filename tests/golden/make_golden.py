"""Generate the golden fixtures of the MoE hot path from the reference itself.

    make -C oracle REFERENCE_DIR=<checkout>   # the reference loader, built from its source
    python tests/golden/make_golden.py  --reference <checkout of the reference> (or $REFERENCE_DIR)

Runs, on the CPU of the build container, the reference's own code for the
layer configuration "4 tokens, H=1024, 16 routed experts top-4 + 1 shared,
I=512, seed 0":

1. its packed-layout builder (scripts/build_packed_expert_layout.py
   ``load_manifest`` + ``build_layout``) over a synthetic safetensors
   checkpoint and manifest holding the seeded expert tensors;
2. its ``PackedExpertStore`` + compiled ``native_packed_loader.cpp``
   (``ExpertCopyPlan.read_into_and_copy``) to materialize every expert;
3. its ``LazyMoE.forward`` (spark_runtime/lazy_official_runtime.py:980-1002)
   with the official ``Gate`` / ``Expert`` - absent from the reference - stood
   in by the oracle's restatement.

It writes cpu_ref_seed0.npz (inputs' hashes, routing, layer output) and
cpu_ref_seed0.json (slab / layout / materialized-bytes hashes).  The tests
regenerate the seeded inputs, check their hashes, and compare.
"""

from __future__ import annotations

import argparse
import csv
import hashlib
import importlib.util
import json
import os
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "deepseek-v4-flash-dgx-spark_b200"))

from oracle import moe_oracle as O  # noqa: E402
from spark_b200.moe import PACKED_ORDER, packed_block_layout  # noqa: E402
from spark_b200.packed_store import write_packed_layout  # noqa: E402
from spark_b200.synthetic import CONFIGS, make_layer  # noqa: E402

LAYER = 3
VOLATILE = ("created_at_unix", "model_dir", "manifest_csv")


def sha(b) -> str:
    if isinstance(b, torch.Tensor):
        b = b.contiguous().view(torch.uint8).numpy().tobytes()
    elif isinstance(b, np.ndarray):
        b = np.ascontiguousarray(b).tobytes()
    return hashlib.sha256(b).hexdigest()


def load_ref_loader():
    so = sorted((REPO / "oracle" / "_ref").glob("native_packed_loader_ref*.so"))
    if not so:
        raise SystemExit("build the reference loader first: make -C oracle")
    spec = importlib.util.spec_from_file_location("native_packed_loader_ref", so[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def write_checkpoint(model_dir: Path, blocks: torch.Tensor, dim: int, inter: int) -> Path:
    """safetensors shard with the routed-expert tensors + manifest CSV in the
    reference's column layout (results/spark-66c9/weight-manifest.csv:1)."""
    from safetensors.torch import save_file

    lay = packed_block_layout(dim, inter)
    tensors = {}
    meta = {}
    for e in range(blocks.shape[0]):
        blk = blocks[e]
        for name in PACKED_ORDER:
            off, n, _, shape = lay[name]
            t = blk[off:off + n].clone().view(*shape)
            tname = f"layers.{LAYER}.ffn.experts.{e}.{name}"
            tensors[tname] = t.view(torch.int8) if name.endswith("weight") else t
            meta[tname] = ("I8" if name.endswith("weight") else "F8_E8M0", shape, n)
    shard = "model-00001-of-00001.safetensors"
    save_file(tensors, str(model_dir / shard))
    raw = (model_dir / shard).read_bytes()
    hlen = int.from_bytes(raw[:8], "little")
    header = json.loads(raw[8:8 + hlen])
    manifest = model_dir / "weight-manifest.csv"
    cols = ["source_name", "target_name", "status", "role", "transform", "source_dtype", "source_shape",
            "source_bytes", "source_shard", "source_offset", "target_known", "target_dtype", "target_shape",
            "target_bytes"]
    with manifest.open("w", newline="") as f:
        w = csv.writer(f)
        w.writerow(cols)
        for tname, (dt, shape, n) in meta.items():
            start = 8 + hlen + header[tname]["data_offsets"][0]
            transform = "reinterpret_int8_as_fp4" if dt == "I8" else "copy"
            w.writerow([tname, tname, "mapped", "lazy_routed_expert", transform, dt, f"{shape[0]}x{shape[1]}", n,
                        shard, start, "True", "", "", n])
    return manifest


class _QLin(torch.nn.Module):
    def __init__(self, wshape, sshape):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.zeros(wshape, dtype=torch.uint8), requires_grad=False)
        self.scale = torch.nn.Parameter(torch.zeros(sshape, dtype=torch.uint8), requires_grad=False)


def official_stub(cfg):
    """Stand-ins for the official Gate / Expert (absent from the reference):
    parameters with the checkpoint's byte sizes, arithmetic by the oracle."""

    class Gate(torch.nn.Module):
        def __init__(self, layer_id, args):
            super().__init__()
            self.weight = torch.nn.Parameter(torch.zeros(cfg.n_routed, cfg.dim), requires_grad=False)
            self.bias = torch.nn.Parameter(torch.zeros(cfg.n_routed), requires_grad=False)
            self.last = None

        def forward(self, x, input_ids):
            w, idx, logits = O.gate_forward(x.float().numpy(), self.weight.numpy(), self.bias.numpy(), cfg.topk,
                                            cfg.route_scale)
            self.last = (w, idx, logits)
            return torch.from_numpy(w), torch.from_numpy(idx)

    class Expert(torch.nn.Module):
        def __init__(self, dim, inter, dtype=None, swiglu_limit=0.0):
            super().__init__()
            self.fp4 = dtype == torch.float4_e2m1fn_x2
            self.swiglu_limit = swiglu_limit
            if self.fp4:
                self.w1 = _QLin((inter, dim // 2), (inter, dim // 32))
                self.w2 = _QLin((dim, inter // 2), (dim, inter // 32))
                self.w3 = _QLin((inter, dim // 2), (inter, dim // 32))
            else:
                self.w1 = _QLin((inter, dim), (inter // 128, dim // 128))
                self.w2 = _QLin((dim, inter), (dim // 128, inter // 128))
                self.w3 = _QLin((inter, dim), (inter // 128, dim // 128))

        def forward(self, x, weights=None):
            ew = O.ExpertWeights(self.w1.weight.numpy(), self.w1.scale.numpy(), self.w2.weight.numpy(),
                                 self.w2.scale.numpy(), self.w3.weight.numpy(), self.w3.scale.numpy(), fp4=self.fp4)
            rw = None if weights is None else weights.float().numpy().reshape(-1)
            y = O.expert_forward(x.float().numpy(), ew, rw, self.swiglu_limit)
            return torch.from_numpy(y).to(torch.bfloat16)

    return SimpleNamespace(Gate=Gate, Expert=Expert)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_DIR"), required="REFERENCE_DIR" not in os.environ)
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "scripts"))
    cfg = CONFIGS["cpu_ref"]
    layer = make_layer(cfg, seed=0, device="cpu")
    blocks = layer["blocks"]
    out = {"config": "cpu_ref", "seed": 0, "layer": LAYER,
           "inputs": {"x": sha(layer["x"]), "gate_w": sha(layer["gate_w"]), "gate_bias": sha(layer["gate_bias"]),
                      "blocks": sha(blocks), **{f"shared.{k}": sha(v) for k, v in layer["shared"].items()}}}

    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        model_dir = tmp / "model"
        model_dir.mkdir()
        manifest = write_checkpoint(model_dir, blocks, cfg.dim, cfg.inter)
        # 1. reference layout builder
        import build_packed_expert_layout as bpl

        by_expert = bpl.load_manifest(manifest, None, None, None)
        ref_out = tmp / "ref_layout"
        ref_layout = bpl.build_layout(model_dir=model_dir, out_dir=ref_out, manifest_csv=manifest,
                                      by_expert=by_expert, overwrite=True)
        slab = (ref_out / f"layer_{LAYER:02d}.bin").read_bytes()
        stable = {k: v for k, v in ref_layout.items() if k not in VOLATILE}
        out["slab_sha256"] = sha(slab)
        out["slab_bytes"] = len(slab)
        out["layout"] = stable
        # our writer must give the same bytes and layout
        ours = write_packed_layout(tmp / "ours", {LAYER: {e: blocks[e].numpy() for e in range(cfg.n_routed)}},
                                   cfg.dim, cfg.inter)
        assert (tmp / "ours" / f"layer_{LAYER:02d}.bin").read_bytes() == slab, "writer bytes differ"
        assert {k: v for k, v in ours.items() if k not in VOLATILE} == stable, "writer layout differs"

        # 2.-3. reference store, loader and LazyMoE.forward
        os.environ.update({
            "DEEPSEEK_SPARK_PACKED_EXPERT_LAYOUT": str(ref_out / "layout.json"),
            "DEEPSEEK_SPARK_PACKED_NATIVE_LOADER": "1", "DEEPSEEK_SPARK_NATIVE_MATERIALIZER": "1",
            "DEEPSEEK_SPARK_NATIVE_COPY_PLAN": "1", "DEEPSEEK_SPARK_NATIVE_FUSED_MATERIALIZER": "1",
            "DEEPSEEK_SPARK_EXPERT_CACHE_ENTRIES": "64", "DEEPSEEK_SPARK_EMPTY_CACHE_ON_EVICT": "0"})
        import spark_runtime.lazy_official_runtime as lor

        ref_loader = load_ref_loader()
        lor.load_native_packed_loader = lambda: ref_loader
        store = lor.WeightStore(model_dir, manifest)
        cache = lor.configure_expert_cache(64)
        stub = official_stub(cfg)
        margs = SimpleNamespace(dim=cfg.dim, moe_inter_dim=cfg.inter, n_routed_experts=cfg.n_routed,
                                n_activated_experts=cfg.topk, n_shared_experts=1, expert_dtype="fp4",
                                swiglu_limit=cfg.swiglu_limit)
        moe = lor.LazyMoE(stub, LAYER, margs, store, cache)
        with torch.no_grad():
            moe.gate.weight.copy_(layer["gate_w"].float())
            moe.gate.bias.copy_(layer["gate_bias"])
            for n in ("w1", "w2", "w3"):
                getattr(moe.shared_experts, n).weight.copy_(layer["shared"][f"{n}.weight"])
                getattr(moe.shared_experts, n).scale.copy_(layer["shared"][f"{n}.scale"])
        x = layer["x"].view(1, cfg.tokens, cfg.dim)
        ids = torch.arange(cfg.tokens).view(1, -1)
        y = moe.forward(x, ids)
        w, idx, logits = moe.gate.last
        # materialized parameter bytes of every expert, through the reference store + loader
        mat = {}
        for e in range(cfg.n_routed):
            ex = moe.experts[e].materialize(torch.device("cpu"))
            mat[str(e)] = {name: sha(p.data) for name, p in ex.named_parameters()}
        out["materialized_sha256"] = mat
        out["cache_stats"] = {k: v for k, v in cache.snapshot().items()
                              if k in ("packed_loads", "packed_read_bytes", "copied_bytes", "routed_tokens",
                                       "routed_activations", "arena_allocations", "misses", "hits")}
        store.close()

    np.savez_compressed(HERE / "cpu_ref_seed0.npz", y_bits=O.f32_to_bf16_bits(y.float().numpy().reshape(cfg.tokens, -1)),
                        weights=w, indices=idx, logits=logits)
    (HERE / "cpu_ref_seed0.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "cpu_ref_seed0.npz", HERE / "cpu_ref_seed0.json")


if __name__ == "__main__":
    main()
