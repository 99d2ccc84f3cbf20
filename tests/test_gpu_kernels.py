"""GPU parity of every stage of the MoE hot path against the CPU oracle.

Bars: integer / byte / index results bit-exact; floating point within
max|err| <= 2e-2 * rms(reference) (the bf16-accumulation tolerance of the
benchmark statement), and the canonical-sigmoid routing bit-exact on identical
logits.
"""

import ctypes
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2  # max |err| relative to the reference RMS


def _lib():
    from spark_b200 import _lib

    return _lib


def _rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2)) + 1e-30
    return float(np.max(np.abs(got - ref)) / rms)


def _bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _no_device_error():
    _lib().raise_on_device_error()


# ---------------------------------------------------------------------------
# act_quant
# ---------------------------------------------------------------------------
def test_act_quant_bit_exact(cuda_device):
    L = _lib()
    g = torch.Generator().manual_seed(7)
    x = torch.randn(67, 1024, generator=g).to(torch.bfloat16)
    x[0, :128] = 0
    x[1, :128] = 0
    x[1, 3] = 3.5                      # amax = 448 * 2^-7 exactly
    x[2, 128:256] = -0.0
    x[3, 256:384] *= 1e-30             # tiny values
    x[4, 384:512] = 1.75 * 2 ** 10     # exact power-of-two ratio
    xd = x.to(cuda_device)
    q = torch.empty(67, 1024, dtype=torch.uint8, device=cuda_device)
    s = torch.empty(67, 8, dtype=torch.uint8, device=cuda_device)
    L.check(L.load().dsv4_act_quant(L.ptr(xd), 67, 1024, L.ptr(q), L.ptr(s), L.stream_ptr()))
    torch.cuda.synchronize()
    qo, so = O.act_quant(x.float().numpy())
    assert np.array_equal(s.cpu().numpy(), so)
    assert np.array_equal(q.cpu().numpy(), qo)


# ---------------------------------------------------------------------------
# gate
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("E,k,T", [(16, 4, 4), (256, 6, 64), (256, 6, 513)])
def test_gate_topk_bit_exact(cuda_device, E, k, T):
    L = _lib()
    g = torch.Generator().manual_seed(E * 1000 + T)
    logits = torch.randn(T, E, generator=g) * 1.5
    logits[0, :] = 0.0                        # full tie: lowest ids win
    logits[1, 5] = logits[1, 9] = 3.0         # pairwise tie
    bias = (torch.rand(E, generator=g) - 0.5) * 0.2
    ld, bd = logits.to(cuda_device), bias.to(cuda_device)
    w = torch.empty(T, k, device=cuda_device)
    idx = torch.empty(T, k, dtype=torch.int64, device=cuda_device)
    L.check(L.load().dsv4_gate_topk(L.ptr(ld), L.ptr(bd), T, E, k, 2.5, L.ptr(w), L.ptr(idx), L.stream_ptr()))
    torch.cuda.synchronize()
    wo, io = O.route_from_logits(logits.numpy(), bias.numpy(), k, 2.5)
    assert np.array_equal(idx.cpu().numpy(), io)
    assert np.array_equal(w.cpu().numpy().view(np.uint32), wo.view(np.uint32))


@pytest.mark.parametrize("fp32", [True, False])
def test_gate_logits(cuda_device, fp32):
    L = _lib()
    g = torch.Generator().manual_seed(11)
    T, H, E = 40, 4096, 256
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = torch.randn(E, H, generator=g) * 0.02
    w = w if fp32 else w.to(torch.bfloat16)
    out = torch.empty(T, E, device=cuda_device)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    L.check(L.load().dsv4_gate_logits(L.ptr(xd), L.ptr(wd), int(fp32), T, H, E, L.ptr(out), L.stream_ptr()))
    torch.cuda.synchronize()
    ref = O.gate_logits(x.float().numpy(), w.float().numpy())
    err = np.abs(out.cpu().numpy() - ref)
    scale = np.abs(x.float().numpy()) @ np.abs(w.float().numpy()).T
    assert np.all(err <= 1e-6 * scale + 1e-7), float((err / scale).max())


# ---------------------------------------------------------------------------
# experts
# ---------------------------------------------------------------------------
def _routed_expert(H, I, seed, device):
    from spark_b200.moe import Expert, FP4, packed_block_bytes
    from spark_b200.synthetic import routed_blocks

    blk = routed_blocks(1, H, I, seed)[0]
    e = Expert(H, I, dtype=FP4, swiglu_limit=10.0, device=device)
    e.block[: packed_block_bytes(H, I)].copy_(blk.to(device))
    e.refresh_scale_atoms()
    return e, O.expert_from_block(blk.numpy(), H, I)


@pytest.mark.parametrize("H,I,T", [(1024, 512, 4), (1024, 512, 37), (4096, 2048, 1), (4096, 2048, 200)])
def test_routed_expert_fp4(cuda_device, H, I, T):
    e, ew = _routed_expert(H, I, 100 + T, cuda_device)
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    rw = torch.rand(T, generator=g) + 0.25
    y = e(x.to(cuda_device), rw.to(cuda_device)[:, None])
    torch.cuda.synchronize()
    _no_device_error()
    ref = O.expert_forward(x.float().numpy(), ew, rw.numpy(), 10.0)
    err = _rel_err(_bf16_np(y), ref)
    assert err <= TOL, err


@pytest.mark.parametrize("H,I,T", [(1024, 512, 4), (4096, 2048, 70)])
def test_shared_expert_fp8(cuda_device, H, I, T):
    from spark_b200.moe import Expert
    from spark_b200.synthetic import shared_expert

    sh = shared_expert(H, I, 5 + T)
    e = Expert(H, I, swiglu_limit=10.0, device=cuda_device)
    with torch.no_grad():
        for n in ("w1", "w2", "w3"):
            getattr(e, n).weight.view(torch.uint8).copy_(sh[f"{n}.weight"].to(cuda_device))
            getattr(e, n).scale.view(torch.uint8).copy_(sh[f"{n}.scale"].to(cuda_device))
    e.refresh_scale_atoms()
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    y = e(x.to(cuda_device))
    torch.cuda.synchronize()
    _no_device_error()
    ref = O.expert_forward(x.float().numpy(), O.shared_from_tensors({k: v.numpy() for k, v in sh.items()}),
                           None, 10.0)
    err = _rel_err(_bf16_np(y), ref)
    assert err <= TOL, err


# ---------------------------------------------------------------------------
# materializer
# ---------------------------------------------------------------------------
def test_materialize_bit_exact(cuda_device):
    from spark_b200.moe import ExpertArena, packed_block_bytes
    from spark_b200.synthetic import routed_blocks

    H, I, n = 1024, 512, 6
    blocks = routed_blocks(n, H, I, 42)
    arena = ExpertArena(8, H, I, device=cuda_device)
    slab = blocks.to(cuda_device).reshape(-1)
    nb = packed_block_bytes(H, I)
    slots = [7, 0, 3, 5, 1, 2]
    bf16 = torch.zeros(8, 3 * H * I, dtype=torch.bfloat16, device=cuda_device)
    copied = arena.materialize(slab, [i * nb for i in range(n)], slots, bf16_out=bf16)
    torch.cuda.synchronize()
    assert copied == n * nb
    buf = arena.buffer.cpu().numpy()
    sf = arena.sf.cpu().numpy()
    bfn = bf16.view(torch.int16).cpu().numpy().view(np.uint16)
    for i, s in enumerate(slots):
        blk = blocks[i].numpy()
        assert np.array_equal(buf[s * arena.slot_stride: s * arena.slot_stride + nb], blk)
        p = O.materialize_block(blk, H, I)
        ref_sf = np.concatenate([O.sf_atoms(p["w1.scale"].reshape(I, H // 32)),
                                 O.sf_atoms(p["w3.scale"].reshape(I, H // 32)),
                                 O.sf_atoms(p["w2.scale"].reshape(H, I // 32))])
        assert np.array_equal(sf[s * arena.sf_stride:(s + 1) * arena.sf_stride], ref_sf)
        dec = O.decode_block_bf16(blk, H, I)
        ref_bf = np.concatenate([dec["w1"].reshape(-1), dec["w2"].reshape(-1), dec["w3"].reshape(-1)])
        assert np.array_equal(bfn[s], ref_bf)


def test_materialize_misaligned_offset_is_reported_not_loaded(cuda_device):
    """A source offset that is not 16-byte aligned is skipped by the vector
    copy / decode kernels and latched as DSV4_DEVERR_MISALIGNED; the slot keeps
    its previous bytes and no misaligned load is issued."""
    from spark_b200.moe import ExpertArena, packed_block_bytes
    from spark_b200.synthetic import routed_blocks

    H, I = 1024, 512
    nb = packed_block_bytes(H, I)
    blocks = routed_blocks(1, H, I, 3)
    slab = torch.zeros(nb + 64, dtype=torch.uint8, device=cuda_device)
    slab[8:8 + nb].copy_(blocks[0].to(cuda_device))
    arena = ExpertArena(2, H, I, device=cuda_device)
    arena.buffer.fill_(0x5A)
    bf16 = torch.zeros(2, 3 * H * I, dtype=torch.bfloat16, device=cuda_device)
    arena.materialize(slab, [8], [1], bf16_out=bf16)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="16-byte aligned"):
        _no_device_error()
    s = arena.slot_stride
    assert bool((arena.buffer[s:s + nb] == 0x5A).all())
    assert bool((bf16[1] == 0).all())
    _no_device_error()  # the flag was read and cleared


def test_shared_scale_atoms(cuda_device):
    from spark_b200.moe import Expert
    from spark_b200.synthetic import shared_expert

    H, I = 1024, 512
    sh = shared_expert(H, I, 3)
    e = Expert(H, I, device=cuda_device)
    with torch.no_grad():
        for n in ("w1", "w2", "w3"):
            getattr(e, n).scale.view(torch.uint8).copy_(sh[f"{n}.scale"].to(cuda_device))
    e.refresh_scale_atoms()
    ref = np.concatenate([O.sf_atoms_fp8(sh["w1.scale"].numpy(), I, H), O.sf_atoms_fp8(sh["w3.scale"].numpy(), I, H),
                          O.sf_atoms_fp8(sh["w2.scale"].numpy(), H, I)])
    assert np.array_equal(e.scale_atoms.cpu().numpy(), ref)


# ---------------------------------------------------------------------------
# full layer
# ---------------------------------------------------------------------------
def _layer_ws(moe, T):
    from spark_b200 import _lib as L

    d = moe.layer_desc()
    offs = (ctypes.c_longlong * 17)()
    L.check(L.load().dsv4_moe_workspace_layout(ctypes.byref(d), T, offs, 17))
    return list(offs)


def _oracle_weights(layer, experts):
    cfg = layer["cfg"]
    mw = O.MoEWeights(
        gate_w=layer["gate_w"].float().cpu().numpy(), gate_bias=layer["gate_bias"].cpu().numpy(),
        experts={e: O.expert_from_block(layer["blocks"][e].cpu().numpy(), cfg.dim, cfg.inter) for e in experts},
        shared=O.shared_from_tensors({k: v.cpu().numpy() for k, v in layer["shared"].items()}),
        topk=cfg.topk, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)
    return mw


@pytest.mark.parametrize("name,T", [("cpu_ref", 4), ("cpu_ref", 300), ("cpu_ref", 1000),
                                    ("decode", 1), ("decode", 8), ("decode", 32), ("decode", 64)])
def test_moe_layer(cuda_device, name, T):
    """The whole layer against the oracle on every token, at the decode batch
    sizes the benchmark times (T=64 touches ~200 of the 256 experts)."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS[name].with_tokens(T)
    layer = make_layer(cfg, seed=0, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].to(cuda_device)
    ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=cuda_device)
    y = moe.forward_tokens(x, workspace=ws)
    torch.cuda.synchronize()
    _no_device_error()
    offs = _layer_ws(moe, T)
    k, E = cfg.topk, cfg.n_routed
    logits = ws[offs[0]:offs[0] + T * E * 4].view(torch.float32).view(T, E).cpu().numpy()
    w_gpu = ws[offs[1]:offs[1] + T * k * 4].view(torch.float32).view(T, k).cpu().numpy()
    i_gpu = ws[offs[2]:offs[2] + T * k * 8].view(torch.int64).view(T, k).cpu().numpy()
    # gate: logits within fp32 accumulation error; routing bit-exact on the device's logits
    ref_logits = O.gate_logits(layer["x"].float().numpy(), layer["gate_w"].float().numpy())
    assert np.max(np.abs(logits - ref_logits)) < 1e-4
    w_ref, i_ref = O.route_from_logits(logits, layer["gate_bias"].numpy(), k, cfg.route_scale)
    assert np.array_equal(i_gpu, i_ref)
    assert np.array_equal(w_gpu.view(np.uint32), w_ref.view(np.uint32))
    # routing plan: per-expert counts are the bincount of the indices
    counts = ws[offs[3]:offs[3] + (E + 1) * 4].view(torch.int32).cpu().numpy()
    assert np.array_equal(counts[:E], np.bincount(i_gpu.reshape(-1), minlength=E))
    assert counts[E] == T
    # layer output on the device's routing
    experts = sorted(set(i_gpu.reshape(-1).tolist()))
    mw = _oracle_weights(layer, experts)
    y_ref = O.moe_forward(layer["x"].float().numpy(), mw, routing=(w_gpu, i_gpu), workers=_WORKERS)[0]
    err = _rel_err(_bf16_np(y), y_ref)
    assert err <= TOL, err


_WORKERS = max(1, min(16, os.cpu_count() or 1))


def _routing_flip_check(i_gpu, x_cpu, gate_w_cpu, bias_cpu, k):
    """Device top-k against the oracle's top-k on the oracle's own logits;
    every differing token must be a near tie (gap below 1e-5 of the boundary
    score).  Returns the flips for the report."""
    ref_logits = O.gate_logits(x_cpu, gate_w_cpu)
    flips = O.routing_flips(i_gpu, ref_logits, bias_cpu, k)
    bad = [(t, g) for t, g in flips if not g < 1e-5]
    assert not bad, f"routing flips that are not near ties: {bad[:8]}"
    return flips


@pytest.mark.parametrize("name,T", [("decode", 64), ("prefill", 8192)])
def test_routing_flips_are_near_ties(cuda_device, name, T):
    """Routing parity beyond the device's own logits: the device's top-6 on
    its tensor-core (fp32-accumulated) logits against the oracle's top-6 on
    float64-accumulated logits.  Any token whose expert set differs is
    reported with its score gap, and the gap must be within accumulation
    error."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS[name].with_tokens(T)
    layer = make_layer(cfg, seed=3, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].to(cuda_device)
    w, idx = moe.gate(x)
    torch.cuda.synchronize()
    _no_device_error()
    flips = _routing_flip_check(idx.cpu().numpy(), layer["x"].float().numpy(), layer["gate_w"].float().numpy(),
                                layer["gate_bias"].numpy(), cfg.topk)
    print(f"routing flips {name} T={T}: {len(flips)} of {T} tokens; gaps {[f'{g:.1e}' for _, g in flips[:8]]}")
    assert len(flips) <= max(2, T // 1000)


def test_moe_module_forward_shape_and_dtype(cuda_device):
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["cpu_ref"].with_tokens(6)
    layer = make_layer(cfg, seed=1)
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].view(2, 3, cfg.dim).to(cuda_device)
    ids = torch.arange(6, device=cuda_device).view(2, 3)
    y = moe(x, ids)
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    w, idx = moe.gate(x.view(-1, cfg.dim), ids.view(-1))
    assert w.shape == (6, cfg.topk) and idx.dtype == torch.int64


@pytest.mark.parametrize("T", [1, 3, 8])
def test_fused_small_batch_routing_equals_the_separate_kernels(cuda_device, T):
    """With dsv4_set_fused_routing(1), at T <= 8 the layer's own gate runs as
    split-K partials + one fused top-k / plan / scatter kernel.  Fed its
    routing back (which takes the separate plan and scatter kernels), the
    layer gives the same bits: output, counts, segments, tiles, every route's
    slot and the quantized rows."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["decode"].with_tokens(T)
    layer = make_layer(cfg, seed=40 + T, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].to(cuda_device)
    nb = moe.workspace_bytes(T)
    ws1 = torch.zeros(nb, dtype=torch.uint8, device=cuda_device)
    ws2 = torch.zeros(nb, dtype=torch.uint8, device=cuda_device)
    L = _lib()
    L.check(L.load().dsv4_set_fused_routing(1), "dsv4_set_fused_routing")
    try:
        y1 = moe.forward_tokens(x, workspace=ws1)
        torch.cuda.synchronize()
    finally:
        L.check(L.load().dsv4_set_fused_routing(0), "dsv4_set_fused_routing")
    offs = _layer_ws(moe, T)
    k, E, H = cfg.topk, cfg.n_routed, cfg.dim
    w = ws1[offs[1]:offs[1] + T * k * 4].view(torch.float32).view(T, k).clone()
    i = ws1[offs[2]:offs[2] + T * k * 8].view(torch.int64).view(T, k).clone()
    y2 = moe.forward_tokens(x, routing=(w, i), workspace=ws2)
    torch.cuda.synchronize()
    _no_device_error()
    assert torch.equal(y1, y2)

    def ints(ws, o, n):
        return ws[offs[o]:offs[o] + 4 * n].view(torch.int32).cpu().numpy()

    for o, n in ((3, E + 1), (4, E + 2), (5, 1), (6, T * k)):
        assert np.array_equal(ints(ws1, o, n), ints(ws2, o, n)), o
    rows = int(ints(ws1, 4, E + 2)[E + 1])
    assert np.array_equal(ints(ws1, 7, rows), ints(ws2, 7, rows))
    nt = int(ints(ws1, 5, 1)[0])
    assert np.array_equal(ints(ws1, 9, 4 * nt), ints(ws2, 9, 4 * nt))
    tok = ints(ws1, 7, rows)
    valid = np.nonzero(tok >= 0)[0]
    xq1 = ws1[offs[10]:offs[10] + rows * H].view(rows, H).cpu().numpy()
    xq2 = ws2[offs[10]:offs[10] + rows * H].view(rows, H).cpu().numpy()
    assert np.array_equal(xq1[valid], xq2[valid])
    y_ref = O.moe_forward(layer["x"].float().numpy(), _oracle_weights(layer, sorted(set(i.cpu().reshape(-1).tolist()))),
                          routing=(w.cpu().numpy(), i.cpu().numpy()), workers=_WORKERS)[0]
    assert _rel_err(_bf16_np(y1), y_ref) <= TOL


def test_module_forward_graph_replay_equals_the_eager_layer(cuda_device):
    """MoE.forward replays a captured graph per token count: every call,
    the capturing one included, equals the eager C ABI layer bit for bit; a
    second token count gets its own graph; a replaced weight tensor (a new
    address) is recaptured."""
    from spark_b200 import _lib
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["decode"].with_tokens(64)
    layer = make_layer(cfg, seed=11, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    g = torch.Generator().manual_seed(12)
    for T in (64, 64, 7, 64, 7):
        x = (torch.randn(T, cfg.dim, generator=g) * 0.5).to(torch.bfloat16).to(cuda_device)
        y = moe(x.view(1, T, cfg.dim)).view(T, cfg.dim)
        ref = moe.forward_tokens(x)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), T
    assert sorted(moe._graphs) == [7, 64]
    first = moe._graphs[64][0]
    with torch.no_grad():
        moe.gate.weight = torch.nn.Parameter(moe.gate.weight.detach().clone() * 0.5, requires_grad=False)
    x = (torch.randn(64, cfg.dim, generator=g) * 0.5).to(torch.bfloat16).to(cuda_device)
    y = moe(x.view(1, 64, cfg.dim)).view(64, cfg.dim)
    assert moe._graphs[64][0] is not first
    assert torch.equal(y, moe.forward_tokens(x))
    _lib.raise_on_device_error()


def test_prefill_layer_full_size_routing_and_sampled_rows(cuda_device):
    """T=8192 with the Zipf(1.2)-tilted gate: routing checked on every token
    (bit-exact on the device's logits, counts = bincount), outputs checked on a
    stratified sample of 160 tokens against the oracle (tokens are
    independent, so the sample needs only the experts it touches)."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["prefill"]
    T = cfg.tokens
    layer = make_layer(cfg, seed=5, device=cuda_device)
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"]
    ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=cuda_device)
    y = moe.forward_tokens(x, workspace=ws)
    torch.cuda.synchronize()
    _no_device_error()
    offs = _layer_ws(moe, T)
    k, E = cfg.topk, cfg.n_routed
    logits = ws[offs[0]:offs[0] + T * E * 4].view(torch.float32).view(T, E).cpu().numpy()
    w_gpu = ws[offs[1]:offs[1] + T * k * 4].view(torch.float32).view(T, k).cpu().numpy()
    i_gpu = ws[offs[2]:offs[2] + T * k * 8].view(torch.int64).view(T, k).cpu().numpy()
    w_ref, i_ref = O.route_from_logits(logits, layer["gate_bias"].cpu().numpy(), k, cfg.route_scale)
    assert np.array_equal(i_gpu, i_ref)
    assert np.array_equal(w_gpu.view(np.uint32), w_ref.view(np.uint32))
    counts = ws[offs[3]:offs[3] + (E + 1) * 4].view(torch.int32).cpu().numpy()
    assert np.array_equal(counts[:E], np.bincount(i_gpu.reshape(-1), minlength=E))
    top8 = np.sort(counts[:E])[::-1][:8].sum() / (T * k)
    assert 0.2 < top8 < 0.45, top8   # Zipf tilt: ~30% of token-slots on 8 experts
    # 160 tokens, stratified: 48 routed to the most popular experts (the
    # largest segments, tiles of 128 rows), 48 that use the least popular
    # experts (segments of one or a few rows), 64 uniform
    rng = np.random.default_rng(0)
    hot = np.argsort(-counts[:E], kind="stable")[:8]
    cold = [e for e in np.argsort(counts[:E], kind="stable") if counts[e] > 0][:24]
    on_hot = np.flatnonzero(np.isin(i_gpu, hot).any(axis=1))
    on_cold = np.flatnonzero(np.isin(i_gpu, cold).any(axis=1))
    picks = [rng.choice(on_hot, min(48, on_hot.size), replace=False),
             rng.choice(on_cold, min(48, on_cold.size), replace=False), rng.choice(T, 64, replace=False)]
    sample = np.unique(np.concatenate(picks))
    assert sample.size >= 128 and counts[cold[0]] <= 2
    experts = sorted(set(i_gpu[sample].reshape(-1).tolist()))
    cpu_layer = {**layer, "blocks": layer["blocks"].cpu(), "gate_w": layer["gate_w"].cpu(),
                 "gate_bias": layer["gate_bias"].cpu(), "shared": {a: b.cpu() for a, b in layer["shared"].items()}}
    mw = _oracle_weights(cpu_layer, experts)
    y_ref = O.moe_forward(x[sample].float().cpu().numpy(), mw, routing=(w_gpu[sample], i_gpu[sample]),
                          workers=_WORKERS)[0]
    err = _rel_err(_bf16_np(y)[sample], y_ref)
    assert err <= TOL, err


@pytest.mark.parametrize("T", [1, 37, 513, 2047, 9000])
def test_gate_route_tensor_core_path(cuda_device, T):
    """bf16 gate over 256 experts: tcgen05 logits with routing fused in the
    epilogue.  Logits within fp32-accumulation error of the oracle, routing
    bit-exact on the device's own logits (ragged last tile included)."""
    L = _lib()
    g = torch.Generator().manual_seed(T)
    H, E, k = 4096, 256, 6
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.rand(E, generator=g) - 0.5) * 0.2
    xd, wd, bd = x.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    logits = torch.empty(T, E, device=cuda_device)
    wt = torch.empty(T, k, device=cuda_device)
    idx = torch.empty(T, k, dtype=torch.int64, device=cuda_device)
    need = L.load().dsv4_gate_workspace_bytes(L.ptr(wd), 0, T, H, E)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=cuda_device)
    L.check(L.load().dsv4_gate_route(L.ptr(xd), L.ptr(wd), 0, L.ptr(bd), T, H, E, k, 2.5, L.ptr(logits),
                                     L.ptr(wt), L.ptr(idx), L.ptr(ws), need, L.stream_ptr()))
    torch.cuda.synchronize()
    _no_device_error()
    lg = logits.cpu().numpy()
    sel = slice(0, min(T, 600))
    ref = O.gate_logits(x[sel].float().numpy(), w.float().numpy())
    scale = np.abs(x[sel].float().numpy()) @ np.abs(w.float().numpy()).T
    assert np.all(np.abs(lg[sel] - ref) <= 1e-6 * scale + 1e-7)
    wo, io = O.route_from_logits(lg, bias.numpy(), k, 2.5)
    assert np.array_equal(idx.cpu().numpy(), io)
    assert np.array_equal(wt.cpu().numpy().view(np.uint32), wo.view(np.uint32))


# ---------------------------------------------------------------------------
# routing plan: bit-exact permutation against the oracle
# ---------------------------------------------------------------------------
def _plan_from_ws(ws, offs, T, k, E):
    i32 = lambda o, n: ws[o:o + 4 * n].view(torch.int32).cpu().numpy().astype(np.int64)
    seg = i32(offs[4], E + 2)
    rows = int(seg[E + 1])
    n_tiles = int(i32(offs[5], 1)[0])
    tiles = i32(offs[9], 4 * n_tiles).reshape(-1, 4)
    return {"counts": i32(offs[3], E + 1), "seg_start": seg, "route_slot": i32(offs[6], T * k),
            "slot_token": i32(offs[7], rows), "tiles": [tuple(int(v) for v in t[:3]) for t in tiles]}


@pytest.mark.parametrize("name,T,pattern", [("cpu_ref", 1, "random"), ("cpu_ref", 37, "random"),
                                            ("cpu_ref", 300, "one_hot"), ("cpu_ref", 1500, "random"),
                                            ("decode", 64, "random"), ("decode", 1100, "skewed"),
                                            ("decode", 2048, "random")])
def test_route_plan_matches_oracle(cuda_device, name, T, pattern):
    """counts, padded segment starts, every route's slot, every slot's token
    (-1 on padding) and the tile list equal the oracle's stable counting sort;
    covers one chunk, ragged chunks, both chunk sizes and a segment holding
    every token.  Up to 40 chunks x 256 experts the plan is built by one CTA,
    beyond that (T=2048) by the multi-CTA count / scan kernels."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS[name].with_tokens(T)
    layer = make_layer(cfg, seed=1, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    E, k = cfg.n_routed, cfg.topk
    g = torch.Generator().manual_seed(T)
    if pattern == "one_hot":  # every token routes to experts 0..k-1
        idx = torch.arange(k).repeat(T, 1)
    elif pattern == "skewed":  # half of all routes land on 8 experts
        hot = torch.randperm(E, generator=g)[:8]
        rows = []
        for _ in range(T):
            a = hot[torch.randperm(8, generator=g)[:k // 2]].tolist()
            rest = [e for e in torch.randperm(E, generator=g).tolist() if e not in a][:k - len(a)]
            rows.append(a + rest)
        idx = torch.tensor(rows)
    else:
        idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    x = layer["x"].to(cuda_device)
    ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=cuda_device)
    moe.forward_tokens(x, workspace=ws, routing=(w.to(cuda_device), idx.to(cuda_device)))
    torch.cuda.synchronize()
    _no_device_error()
    offs = _layer_ws(moe, T)
    got = _plan_from_ws(ws, offs, T, k, E)
    ref = O.route_plan(idx.numpy(), E, int(offs[16]), T)
    for key in ("counts", "seg_start", "route_slot", "slot_token"):
        assert np.array_equal(got[key], ref[key]), key
    assert got["tiles"] == ref["tiles"]


# ---------------------------------------------------------------------------
# hash-routed layers (gate.tid2eid)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name,T", [("cpu_ref", 5), ("decode", 1), ("decode", 37), ("decode", 3000)])
def test_hash_gate_bit_exact_on_device_logits(cuda_device, name, T):
    """Indices are the table rows of the token ids; weights equal the oracle's
    hash routing on the device's own logits bit for bit (SIMT logits for the
    fp32 gate, tensor-core partials otherwise, also above the fused size)."""
    from dataclasses import replace

    from spark_b200.moe import Gate
    from spark_b200.synthetic import CONFIGS, make_layer

    cfg = CONFIGS[name].with_tokens(T)
    layer = make_layer(cfg, seed=5, device="cpu")
    args = replace(cfg.args(), n_hash_layers=3, vocab_size=1000)
    gate = Gate(0, args, device=cuda_device)
    g = torch.Generator().manual_seed(T)
    table = torch.stack([torch.randperm(cfg.n_routed, generator=g)[:cfg.topk] for _ in range(1000)])
    ids = torch.randint(0, 1000, (T,), generator=g)
    with torch.no_grad():
        gate.weight.copy_(layer["gate_w"].to(cuda_device))
        gate.tid2eid.copy_(table.to(cuda_device))
    w, idx = gate(layer["x"].to(cuda_device), ids.to(cuda_device))
    torch.cuda.synchronize()
    _no_device_error()
    logits = gate.last_logits.cpu().numpy()
    ref_logits = O.gate_logits(layer["x"].float().numpy(), layer["gate_w"].float().numpy())
    assert np.max(np.abs(logits - ref_logits)) < 1e-4
    w_ref, i_ref = O.hash_route(logits, table.numpy(), ids.numpy(), cfg.route_scale)
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    assert np.array_equal(w.cpu().numpy().view(np.uint32), w_ref.view(np.uint32))


def test_hash_layer_forward_matches_oracle(cuda_device):
    """MoE.forward of a hash-routed layer: routing from the table, experts and
    combine as in the top-k layers."""
    from dataclasses import replace

    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["cpu_ref"].with_tokens(40)
    layer = make_layer(cfg, seed=6, device="cpu")
    moe = build_moe(layer, device=cuda_device, layer_id=0, args=replace(cfg.args(), n_hash_layers=3, vocab_size=64))
    g = torch.Generator().manual_seed(1)
    table = torch.stack([torch.randperm(cfg.n_routed, generator=g)[:cfg.topk] for _ in range(64)])
    ids = torch.randint(0, 64, (1, 40), generator=g)
    with torch.no_grad():
        moe.gate.tid2eid.copy_(table.to(cuda_device))
    y = moe(layer["x"].view(1, 40, -1).to(cuda_device), ids.to(cuda_device))
    torch.cuda.synchronize()
    _no_device_error()
    w_ref, i_ref = O.hash_route(moe.gate.last_logits.cpu().numpy(), table.numpy(), ids.numpy(), cfg.route_scale)
    mw = _oracle_weights(layer, sorted(set(i_ref.reshape(-1).tolist())))
    y_ref = O.moe_forward(layer["x"].float().numpy(), mw, routing=(w_ref, i_ref))[0]
    assert _rel_err(_bf16_np(y.view(40, -1)), y_ref) <= TOL


_CHILD = r"""
import sys, numpy as np, torch
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/deepseek-v4-flash-dgx-spark_b200"]
from spark_b200.synthetic import CONFIGS, build_moe, make_layer
cfg = CONFIGS[sys.argv[2]].with_tokens(int(sys.argv[3]))
layer = make_layer(cfg, seed=11, device="cpu")
moe = build_moe(layer, device=torch.device("cuda", 0))
y = moe.forward_tokens(layer["x"].cuda(), workspace=torch.empty(moe.workspace_bytes(cfg.tokens), dtype=torch.uint8, device="cuda"))
torch.cuda.synchronize()
from spark_b200 import _lib
_lib.raise_on_device_error()
np.save(sys.argv[4], y.view(torch.int16).cpu().numpy())
"""


def _layer_bits_under_env(tmp_path, cfg_name, T, env_sets):
    import os
    import subprocess
    import sys

    repo = str(Path(__file__).resolve().parent.parent)
    outs = []
    for i, extra in enumerate(env_sets):
        env = dict(os.environ, **extra)
        f = tmp_path / f"y_{i}.npy"
        r = subprocess.run([sys.executable, "-c", _CHILD, repo, cfg_name, str(T), str(f)], env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(f))
    return outs


@pytest.mark.parametrize("T", [600, 1000])
def test_pair_gemm_bit_identical_to_single_cta_gemm(cuda_device, tmp_path, T):
    """The CTA-pair grouped GEMM (256-row tiles, cta_group::2) and the
    single-CTA GEMM (128-row tiles) compute every output row with the same
    block-scaled products in the same k order: the layer outputs must be
    bit-identical.  DSV4_BLOCK_N picks the tile size at library load, so each
    form runs in its own process."""
    a, b = _layer_bits_under_env(tmp_path, "cpu_ref", T, [{"DSV4_BLOCK_N": "256"}, {"DSV4_BLOCK_N": "128"}])
    assert np.array_equal(a, b)


@pytest.mark.parametrize("T", [1, 8, 37])
def test_split_k_gemm_matches_unsplit_gemm(cuda_device, T):
    """With the split asked for, small decode batches cut every GEMM item's k range over several CTAs
    (fp32 partial sums added in slice order by the CTA that finishes the item
    last).  Against the unsplit GEMM only the fp32 summation order differs, so
    the outputs agree to bf16 rounding (a flipped rounding can move an element
    by one bf16 ulp, a little more after the SwiGLU and FP8 re-quantization:
    the bound is the layer tolerance and at most 1% of elements differing).
    Two runs of the split form are bit-identical: the partial sums are added
    in slice order whichever CTA finishes last."""
    from spark_b200 import _lib as L
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    lib = L.load()
    cfg = CONFIGS["decode"].with_tokens(T)
    layer = make_layer(cfg, seed=11, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].to(cuda_device)
    outs, splits = [], []
    try:
        for setting in (4, 4, 1):  # four slices per item twice, then no split
            L.check(lib.dsv4_set_k_split(setting), "dsv4_set_k_split")
            ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=cuda_device)
            outs.append(moe.forward_tokens(x, workspace=ws))
            d = moe.layer_desc()
            offs = (ctypes.c_longlong * 20)()
            L.check(lib.dsv4_moe_workspace_layout(ctypes.byref(d), T, offs, 20))
            splits.append((offs[18], offs[19]))
        torch.cuda.synchronize()
        _no_device_error()
    finally:
        lib.dsv4_set_k_split(1)  # the library's default: no split
    assert splits[0][0] > 1 and splits[0][1] > 1 and splits[2] == (1, 1), splits
    split, split2, unsplit = (o.view(torch.int16).cpu().numpy() for o in outs)
    assert np.array_equal(split, split2)
    assert _rel_err(_bf16_np(outs[0]), _bf16_np(outs[2])) <= TOL
    assert np.mean(split != unsplit) <= 0.01


def test_moe_forward_writes_the_route_trace(cuda_device, tmp_path):
    """With the reference's route-trace variable set, MoE.forward appends one
    expert_route line per call holding the gate's routing, and its output is
    bit-identical to the untraced call."""
    import json

    from spark_b200 import telemetry as tm
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["cpu_ref"].with_tokens(6)
    layer = make_layer(cfg, seed=1)
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].view(2, 3, cfg.dim).to(cuda_device)
    ids = torch.arange(6, device=cuda_device).view(2, 3)
    tm.set_expert_telemetry(tm.ExpertTelemetry(None))
    try:
        y_plain = moe(x, ids)
        tm.set_expert_telemetry(tm.ExpertTelemetry(tmp_path / "routes.jsonl"))
        y = moe(x, ids)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_plain.view(torch.int16))
        lines = (tmp_path / "routes.jsonl").read_text().splitlines()
        assert len(lines) == 1
        d = json.loads(lines[0])
        _, idx = moe.gate(x.view(-1, cfg.dim), ids.view(-1))
        assert d["event"] == "expert_route" and d["layer_id"] == moe.layer_id
        assert d["token_ids"] == list(range(6)) and d["token_count"] == 6
        assert d["expert_indices"] == idx.cpu().tolist() and d["activation_count"] == 6 * cfg.topk
    finally:
        tm.set_expert_telemetry(None)
