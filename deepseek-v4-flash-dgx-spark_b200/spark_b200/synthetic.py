"""Seeded synthetic MoE layers with the shapes and value distributions of the
benchmark configurations (there is no checkpoint or dataset on the box).

* ``cpu_ref``: T=4, H=1024, E=16 top-4 + 1 shared, I=512; x ~ N(0,1) bf16;
  gate W fp32 ~ N(0, 0.02); bias ~ U(-0.1, 0.1); sigmoid, renorm, x2.5;
  routed FP4 codes uniform over the 16 codes (bytes uniform 0..255), ue8m0
  scales uniform over the exponents -8..-4 (bytes 119..123); shared expert
  e4m3 codes of N(0,1) samples with 128x128 ue8m0 scales in the same range.
* ``decode``: H=4096, E=256 top-6 + 1 shared, I=2048, gate W bf16 ~ N(0,0.02),
  zero bias (every expert equally likely), T in {1, 8, 32, 64}.
* ``prefill``: same shapes, T=8192, gate bias tilted so expert popularity is
  Zipf(1.2) with ~30% of token-slots on the 8 most popular experts.

The generators are torch.Generator streams on the target device; on the CPU
they are reproducible across machines with the same torch build.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from .moe import ExpertArena, ModelArgs, MoE, packed_block_bytes


@dataclass(frozen=True)
class LayerConfig:
    name: str
    tokens: int
    dim: int
    inter: int
    n_routed: int
    topk: int
    n_shared: int = 1
    route_scale: float = 2.5
    swiglu_limit: float = 10.0
    gate_fp32: bool = False
    gate_std: float = 0.02
    bias: str = "zero"          # "zero" | "uniform" | "zipf"
    bias_range: float = 0.1
    zipf_alpha: float = 1.2
    zipf_top8_share: float = 0.30

    def args(self) -> ModelArgs:
        return ModelArgs(dim=self.dim, moe_inter_dim=self.inter, n_routed_experts=self.n_routed,
                         n_activated_experts=self.topk, n_shared_experts=self.n_shared,
                         swiglu_limit=self.swiglu_limit, route_scale=self.route_scale,
                         gate_dtype=torch.float32 if self.gate_fp32 else torch.bfloat16, gate_bias=True)

    def with_tokens(self, t: int) -> "LayerConfig":
        return replace(self, tokens=t)


CONFIGS = {
    "cpu_ref": LayerConfig("cpu_ref", 4, 1024, 512, 16, 4, gate_fp32=True, bias="uniform"),
    "decode": LayerConfig("decode", 64, 4096, 2048, 256, 6),
    "prefill": LayerConfig("prefill", 8192, 4096, 2048, 256, 6, bias="zipf"),
}

SCALE_LO, SCALE_HI = 119, 123  # ue8m0 bytes for 2^-8 .. 2^-4


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def routed_blocks(n: int, dim: int, inter: int, seed: int, device="cpu") -> torch.Tensor:
    """[n, block_bytes] packed expert blocks: three ue8m0 scale matrices then
    three e2m1x2 weight matrices (packed slab order)."""
    nbytes = packed_block_bytes(dim, inter)
    sc = 3 * inter * dim // 32
    out = torch.empty(n, nbytes, dtype=torch.uint8, device=device)
    g = _gen(device, seed)
    out[:, :sc] = torch.randint(SCALE_LO, SCALE_HI + 1, (n, sc), generator=g, device=device, dtype=torch.uint8)
    out[:, sc:] = torch.randint(0, 256, (n, nbytes - sc), generator=g, device=device, dtype=torch.uint8)
    return out


def shared_expert(dim: int, inter: int, seed: int, device="cpu") -> dict[str, torch.Tensor]:
    """fp8 e4m3 shared expert (codes of N(0,1) samples) + 128x128 ue8m0 scales."""
    g = _gen(device, seed)
    out = {}
    for name, (n, k) in (("w1", (inter, dim)), ("w2", (dim, inter)), ("w3", (inter, dim))):
        w = torch.randn(n, k, generator=g, device=device, dtype=torch.float32)
        out[f"{name}.weight"] = w.to(torch.float8_e4m3fn).view(torch.uint8)
        out[f"{name}.scale"] = torch.randint(SCALE_LO, SCALE_HI + 1, (n // 128, k // 128), generator=g,
                                             device=device, dtype=torch.uint8)
    return out


def zipf_bias(gate_w: torch.Tensor, cfg: LayerConfig, seed: int, sample_tokens: int = 512) -> torch.Tensor:
    """Gate bias giving Zipf(alpha) expert popularity: bias_e = gamma * log(p_e / p_max)
    with p_e ~ rank^-alpha over a seeded permutation, gamma bisected so that the
    top-8 experts receive ``zipf_top8_share`` of the token-slots on a sample."""
    E = cfg.n_routed
    dev = gate_w.device
    g = _gen("cpu", seed)
    ranks = torch.randperm(E, generator=g) + 1
    logp = (-cfg.zipf_alpha * torch.log(ranks.to(torch.float64))).to(torch.float32)
    logp = (logp - logp.max()).to(dev)
    xs = torch.randn(sample_tokens, cfg.dim, generator=_gen("cpu", seed + 1)).to(torch.bfloat16).to(dev)
    scores = torch.sigmoid(xs.float() @ gate_w.float().T)
    top8 = torch.argsort(ranks)[:8].to(dev)

    def share(gamma: float) -> float:
        sel = scores + gamma * logp
        idx = torch.topk(sel, cfg.topk, dim=-1).indices
        return float(torch.isin(idx, top8).float().sum() / idx.numel())

    lo, hi = 0.0, 2.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        if share(mid) < cfg.zipf_top8_share:
            lo = mid
        else:
            hi = mid
    return (0.5 * (lo + hi) * logp).to(torch.float32)


def make_layer(cfg: LayerConfig, seed: int = 0, device="cpu") -> dict:
    """All tensors of one synthetic layer on ``device``."""
    dev = torch.device(device)
    g = _gen(dev, seed)
    x = torch.randn(cfg.tokens, cfg.dim, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    gw = torch.randn(cfg.n_routed, cfg.dim, generator=_gen(dev, seed + 11), device=dev, dtype=torch.float32)
    gw = gw * cfg.gate_std
    gate_w = gw if cfg.gate_fp32 else gw.to(torch.bfloat16)
    if cfg.bias == "uniform":
        gb = (torch.rand(cfg.n_routed, generator=_gen(dev, seed + 12), device=dev, dtype=torch.float32) * 2 - 1)
        gate_bias = gb * cfg.bias_range
    elif cfg.bias == "zipf":
        gate_bias = zipf_bias(gate_w, cfg, seed + 13)
    else:
        gate_bias = torch.zeros(cfg.n_routed, dtype=torch.float32, device=dev)
    blocks = routed_blocks(cfg.n_routed, cfg.dim, cfg.inter, seed + 21, dev)
    shared = shared_expert(cfg.dim, cfg.inter, seed + 31, dev)
    return {"cfg": cfg, "x": x, "gate_w": gate_w, "gate_bias": gate_bias, "blocks": blocks, "shared": shared}


def build_moe(layer: dict, device="cuda", layer_id: int = 3, group=None, args: ModelArgs | None = None) -> MoE:
    """A ``MoE`` whose arena is filled by the device materializer from the
    synthetic packed blocks (uploaded as one slab) and whose gate and shared
    expert hold the synthetic tensors.  Under torch.distributed the layer is
    split over ``group`` (default: the world) and each rank materializes only
    the experts it owns.  ``args`` overrides the layer's ModelArgs (e.g. for
    a hash-routed layer, whose gate has no bias)."""
    cfg: LayerConfig = layer["cfg"]
    dev = torch.device(device)
    moe = MoE(layer_id, args or cfg.args(), device=dev, group=group)
    with torch.no_grad():
        moe.gate.weight.copy_(layer["gate_w"].to(dev))
        if moe.gate.bias is not None:
            moe.gate.bias.copy_(layer["gate_bias"].to(dev))
        sh = moe.shared_experts
        for name in ("w1", "w2", "w3"):
            getattr(sh, name).weight.view(torch.uint8).copy_(layer["shared"][f"{name}.weight"].to(dev))
            getattr(sh, name).scale.view(torch.uint8).copy_(layer["shared"][f"{name}.scale"].to(dev))
        sh.refresh_scale_atoms()
        slab = layer["blocks"].to(dev).reshape(-1)
        nb = packed_block_bytes(cfg.dim, cfg.inter)
        local = list(range(moe.experts_start_idx, moe.experts_end_idx))
        slots = [int(moe.expert_slot[e]) for e in local]
        moe.arena.materialize(slab, [e * nb for e in local], slots)
    return moe


def arena_for_blocks(blocks: torch.Tensor, dim: int, inter: int, device="cuda") -> ExpertArena:
    arena = ExpertArena(blocks.shape[0], dim, inter, device=device)
    slab = blocks.to(device).reshape(-1)
    nb = packed_block_bytes(dim, inter)
    arena.materialize(slab, [i * nb for i in range(blocks.shape[0])], list(range(blocks.shape[0])))
    return arena


def algorithmic_decode_bytes(cfg: LayerConfig, experts_touched: int, tokens: int) -> int:
    """HBM bytes one decode layer must move: touched experts' blocks + shared
    expert + gate + activations in/out."""
    shared = 3 * cfg.inter * cfg.dim + 3 * (cfg.inter // 128) * (cfg.dim // 128)
    gate = cfg.n_routed * cfg.dim * (4 if cfg.gate_fp32 else 2) + cfg.n_routed * 4
    return experts_touched * packed_block_bytes(cfg.dim, cfg.inter) + shared + gate + 4 * tokens * cfg.dim


def algorithmic_flops(cfg: LayerConfig, tokens: int) -> float:
    """Expert + gate FLOPs of one layer: T*(k+1)*3*2*H*I + 2*T*H*E."""
    return tokens * (cfg.topk + cfg.n_shared) * 3 * 2.0 * cfg.dim * cfg.inter + 2.0 * tokens * cfg.dim * cfg.n_routed


def expected_touched(cfg: LayerConfig, tokens: int) -> float:
    return cfg.n_routed * (1 - (1 - cfg.topk / cfg.n_routed) ** tokens)

