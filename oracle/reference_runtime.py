"""The reference's own MoE layer on the host cores, for the benchmark's
reference arm.  Test and measurement infrastructure: nothing in the product
imports this file.

It drives the reference runtime's ``LazyMoE.forward``
(spark_runtime/lazy_official_runtime.py:946-1002) through its own
``WeightStore`` / ``PackedExpertStore`` (:49-338, :356-400), its expert cache and
arena, and its native packed loader (spark_runtime/native/native_packed_loader.cpp,
compiled from the reference's source by oracle/Makefile into oracle/_ref/).
The reference is installed, unmodified, into ``baseline/_ref`` by
``pip install --target``.

The official ``Gate`` / ``Expert`` of DeepSeek-V4-Flash (``inference/model.py``,
absent from the reference) are stood in for by CPU classes with the oracle's
semantics: the gate is ``moe_oracle.gate_forward`` (sigmoid, bias for
selection, top-k, renormalise, x route_scale); an expert decodes its FP4 / FP8
parameters exactly to bf16 once, after the reference materialized them, and
keeps them resident (as the reference keeps materialized experts resident in
its cache and arena), then runs act_quant -> w1|w3 -> SwiGLU (clamp) ->
x routing weight -> bf16 -> act_quant -> w2 with bf16 products accumulated in
fp32 by torch's CPU GEMM.  Only the timing uses these classes; the layer's
arithmetic is pinned by the oracle tests.
"""

from __future__ import annotations

import csv
import os
import sys
import tempfile
import time
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

from . import moe_oracle as O

REPO = Path(__file__).resolve().parent.parent
REF_INSTALL = REPO / "baseline" / "_ref"


def import_reference():
    """spark_runtime.lazy_official_runtime from the pip-installed reference."""
    if not (REF_INSTALL / "spark_runtime" / "lazy_official_runtime.py").exists():
        raise RuntimeError(f"the reference is not installed in {REF_INSTALL}")
    if str(REF_INSTALL) not in sys.path:
        sys.path.insert(0, str(REF_INSTALL))
    import spark_runtime.lazy_official_runtime as lor

    return lor


def compiled_reference_loader():
    """The reference's native packed loader built from its own source (oracle/_ref)."""
    import importlib.util

    so = sorted((REPO / "oracle" / "_ref").glob("native_packed_loader_ref*.so"))
    if not so:
        return None
    spec = importlib.util.spec_from_file_location("native_packed_loader_ref", so[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _dequant_act(x: torch.Tensor) -> torch.Tensor:
    """act_quant (e4m3, ue8m0 per 128) and back: exact in bf16."""
    q, s = O.act_quant(x.float().numpy())
    return torch.from_numpy(O.act_dequant(q, s)).to(torch.bfloat16)


class _QLin(torch.nn.Module):
    def __init__(self, wshape, sshape):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.zeros(wshape, dtype=torch.uint8), requires_grad=False)
        self.scale = torch.nn.Parameter(torch.zeros(sshape, dtype=torch.uint8), requires_grad=False)


def official_model(topk: int, route_scale: float, n_routed: int):
    """CPU stand-ins for the official Gate / Expert (see the module docstring)."""

    class Gate(torch.nn.Module):
        def __init__(self, layer_id, args):
            super().__init__()
            self.weight = torch.nn.Parameter(torch.zeros(n_routed, args.dim), requires_grad=False)
            self.bias = torch.nn.Parameter(torch.zeros(n_routed), requires_grad=False)

        def forward(self, x, input_ids):
            w, idx, _ = O.gate_forward(x.float().numpy(), self.weight.numpy(), self.bias.numpy(), topk, route_scale)
            return torch.from_numpy(w), torch.from_numpy(idx)

    class Expert(torch.nn.Module):
        def __init__(self, dim, inter, dtype=None, swiglu_limit=0.0):
            super().__init__()
            self.fp4 = dtype == torch.float4_e2m1fn_x2
            self.limit = float(swiglu_limit or 0.0)
            if self.fp4:
                self.w1 = _QLin((inter, dim // 2), (inter, dim // 32))
                self.w2 = _QLin((dim, inter // 2), (dim, inter // 32))
                self.w3 = _QLin((inter, dim // 2), (inter, dim // 32))
            else:
                self.w1 = _QLin((inter, dim), (inter // 128, dim // 128))
                self.w2 = _QLin((dim, inter), (dim // 128, inter // 128))
                self.w3 = _QLin((inter, dim), (inter // 128, dim // 128))
            self._dense = None

        def _weights(self):
            if self._dense is None:  # exact: e2m1 / e4m3 x power-of-two scales fit bf16
                ew = O.ExpertWeights(self.w1.weight.numpy(), self.w1.scale.numpy(), self.w2.weight.numpy(),
                                     self.w2.scale.numpy(), self.w3.weight.numpy(), self.w3.scale.numpy(),
                                     fp4=self.fp4)
                self._dense = tuple(torch.from_numpy(w).to(torch.bfloat16) for w in ew.dense())
            return self._dense

        def forward(self, x, weights=None):
            w1, w2, w3 = self._weights()
            a = _dequant_act(x)
            g = (a @ w1.T).float()
            u = (a @ w3.T).float()
            if self.limit > 0:
                u = u.clamp(-self.limit, self.limit)
                g = g.clamp(max=self.limit)
            h = torch.nn.functional.silu(g) * u
            if weights is not None:
                h = h * weights.float().reshape(-1, 1)
            return (_dequant_act(h.to(torch.bfloat16)) @ w2.T).to(torch.bfloat16)

    return SimpleNamespace(Gate=Gate, Expert=Expert)


class ReferenceLayer:
    """One synthetic layer served by the reference's LazyMoE on the host."""

    def __init__(self, layer: dict, layer_id: int = 3, workdir: Path | None = None):
        cfg = layer["cfg"]
        self.cfg = cfg
        self.lor = import_reference()
        self._tmp = tempfile.TemporaryDirectory(dir=workdir)
        tmp = Path(self._tmp.name)
        # the packed slab and layout.json in the reference's format (every expert)
        sys.path.insert(0, str(REPO / "deepseek-v4-flash-dgx-spark_b200"))
        from spark_b200.packed_store import write_packed_layout

        blocks = layer["blocks"].cpu()
        write_packed_layout(tmp / "packed", {layer_id: {e: blocks[e].numpy() for e in range(cfg.n_routed)}},
                            cfg.dim, cfg.inter)
        # every expert tensor comes from the packed store: the manifest holds no rows
        model_dir = tmp / "model"
        model_dir.mkdir()
        manifest = model_dir / "weight-manifest.csv"
        with manifest.open("w", newline="") as f:
            csv.writer(f).writerow(["source_name", "target_name", "status", "role", "transform", "source_dtype",
                                    "source_shape", "source_bytes", "source_shard", "source_offset", "target_known",
                                    "target_dtype", "target_shape", "target_bytes"])
        os.environ.update({
            "DEEPSEEK_SPARK_PACKED_EXPERT_LAYOUT": str(tmp / "packed" / "layout.json"),
            "DEEPSEEK_SPARK_PACKED_NATIVE_LOADER": "1", "DEEPSEEK_SPARK_NATIVE_MATERIALIZER": "1",
            "DEEPSEEK_SPARK_NATIVE_COPY_PLAN": "1", "DEEPSEEK_SPARK_NATIVE_FUSED_MATERIALIZER": "1",
            "DEEPSEEK_SPARK_EMPTY_CACHE_ON_EVICT": "0"})
        loader = compiled_reference_loader()
        self.loader_kind = "oracle/_ref (compiled from the reference source)" if loader else "reference JIT build"
        if loader is not None:
            self.lor.load_native_packed_loader = lambda: loader
        self.store = self.lor.WeightStore(model_dir, manifest)
        self.cache = self.lor.configure_expert_cache(cfg.n_routed)
        margs = SimpleNamespace(dim=cfg.dim, moe_inter_dim=cfg.inter, n_routed_experts=cfg.n_routed,
                                n_activated_experts=cfg.topk, n_shared_experts=1, expert_dtype="fp4",
                                swiglu_limit=cfg.swiglu_limit)
        self.moe = self.lor.LazyMoE(official_model(cfg.topk, cfg.route_scale, cfg.n_routed), layer_id, margs,
                                    self.store, self.cache)
        with torch.no_grad():
            self.moe.gate.weight.copy_(layer["gate_w"].float().cpu())
            self.moe.gate.bias.copy_(layer["gate_bias"].cpu())
            for n in ("w1", "w2", "w3"):
                getattr(self.moe.shared_experts, n).weight.copy_(layer["shared"][f"{n}.weight"].cpu())
                getattr(self.moe.shared_experts, n).scale.copy_(layer["shared"][f"{n}.scale"].cpu())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        with torch.no_grad():
            return self.moe.forward(x.view(1, T, -1).cpu(), torch.arange(T).view(1, -1)).view(T, -1)

    def timed_step(self, x: torch.Tensor) -> float:
        t0 = time.perf_counter()
        self.forward(x)
        return time.perf_counter() - t0

    def close(self) -> None:
        self.store.close()
        self._tmp.cleanup()


def layer_matches_oracle(ref: ReferenceLayer, layer: dict, tokens: int = 4) -> float:
    """max |err| / rms of the reference layer (stand-ins included) against the
    oracle on the first tokens: the timed arm computes the same layer."""
    x = layer["x"][:tokens].cpu()
    y = ref.forward(x).float().numpy()
    cfg = layer["cfg"]
    xf = x.float().numpy()
    w, idx, _ = O.gate_forward(xf, layer["gate_w"].float().cpu().numpy(), layer["gate_bias"].cpu().numpy(),
                               cfg.topk, cfg.route_scale)
    mw = O.MoEWeights(gate_w=None, gate_bias=None,
                      experts={int(e): O.expert_from_block(layer["blocks"][int(e)].cpu().numpy(), cfg.dim, cfg.inter)
                               for e in np.unique(idx)},
                      shared=O.shared_from_tensors({k: v.cpu().numpy() for k, v in layer["shared"].items()}),
                      topk=cfg.topk, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)
    ref_y = O.moe_forward(xf, mw, routing=(w, idx), workers=min(16, os.cpu_count() or 1))[0]
    return float(np.max(np.abs(y - ref_y)) / (np.sqrt(np.mean(ref_y.astype(np.float64) ** 2)) + 1e-30))
