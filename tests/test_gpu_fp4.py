"""The opt-in FP4-activation mode on the GPU.

* dsv4_fp4_act_quant is bit-exact against the oracle's restatement of the
  official fp4_act_quant(x, 32) (codes and scale bytes), edge cases included.
* With dsv4_set_fp4_activations(1) the routed experts' GEMMs run as kind::mxf4
  products on FP4 activations (x before w1 / w3, h before w2); the output
  matches the oracle run in the same mode (the shared expert on e4m3) within
  the layer bar, at every tile size (32 / 64 / 128 rows).  How far the mode
  moves the layer from the reference's e4m3 arithmetic is reported beside it.
"""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2
_WORKERS = max(1, min(16, os.cpu_count() or 1))


def _rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / (np.sqrt(np.mean(ref ** 2)) + 1e-30))


def _rms_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(np.mean((got - ref) ** 2)) / (np.sqrt(np.mean(ref ** 2)) + 1e-30))


@pytest.fixture
def fp4_mode():
    from spark_b200 import _lib

    lib = _lib.load()
    _lib.check(lib.dsv4_set_fp4_activations(1), "dsv4_set_fp4_activations")
    yield
    _lib.check(lib.dsv4_set_fp4_activations(0), "dsv4_set_fp4_activations")


def test_fp4_act_quant_bit_exact(cuda_device):
    from spark_b200 import _lib

    g = torch.Generator().manual_seed(21)
    M, K = 37, 1024
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    x[0, :32] = 0
    x[1, :32] = 0
    x[1, 5] = 6.0 * 2 ** -4           # amax / 6 a power of two
    x[2, 32:64] = -0.0
    x[3, 64:96] *= 1e-30              # below the 1e-4 floor
    x[4, 96:128] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 4) * 2 ** -3 * (8 / 6)
    x[5, 128:160] = 1e4
    x[6, 160:192] = -3.0
    xd = x.to(cuda_device)
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=cuda_device)
    s = torch.empty(M, K // 32, dtype=torch.uint8, device=cuda_device)
    _lib.check(_lib.load().dsv4_fp4_act_quant(_lib.ptr(xd), M, K, _lib.ptr(q), _lib.ptr(s), _lib.stream_ptr()),
               "dsv4_fp4_act_quant")
    torch.cuda.synchronize()
    qo, so = O.fp4_act_quant(x.float().numpy())
    assert np.array_equal(s.cpu().numpy(), so)
    assert np.array_equal(q.cpu().numpy(), qo)
    from spark_b200 import ops

    q2, s2 = ops.load().fp4_act_quant(xd)  # the torch op: the same call
    assert torch.equal(q2, q) and torch.equal(s2, s)


@pytest.mark.parametrize("name,T", [("decode", 64), ("decode", 1000), ("cpu_ref", 300)])
def test_fp4_activation_layer_matches_the_fp4_oracle(cuda_device, fp4_mode, name, T):
    from spark_b200 import _lib
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS[name].with_tokens(T)
    layer = make_layer(cfg, seed=2, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    d = moe.layer_desc()
    offs = (ctypes.c_longlong * 21)()
    _lib.check(_lib.load().dsv4_moe_workspace_layout(ctypes.byref(d), T, offs, 21), "layout")
    assert offs[20] == 1, "the FP4 mode is not in force"
    x = layer["x"].to(cuda_device)
    ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=cuda_device)
    y = moe.forward_tokens(x, workspace=ws)
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    k = cfg.topk
    w_gpu = ws[offs[1]:offs[1] + T * k * 4].view(torch.float32).view(T, k).cpu().numpy()
    i_gpu = ws[offs[2]:offs[2] + T * k * 8].view(torch.int64).view(T, k).cpu().numpy()
    experts = sorted(set(i_gpu.reshape(-1).tolist()))
    mw = O.MoEWeights(
        gate_w=layer["gate_w"].float().numpy(), gate_bias=layer["gate_bias"].numpy(),
        experts={e: O.expert_from_block(layer["blocks"][e].numpy(), cfg.dim, cfg.inter) for e in experts},
        shared=O.shared_from_tensors({kk: v.numpy() for kk, v in layer["shared"].items()}),
        topk=cfg.topk, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)
    xs = layer["x"].float().numpy()
    got = y.float().cpu().numpy()
    y4 = O.moe_forward(xs, mw, routing=(w_gpu, i_gpu), workers=_WORKERS, fp4_act=True)[0]
    err = _rel_err(got, y4)
    assert err <= TOL, err
    # the mode's distance from the reference's e4m3 arithmetic (reported)
    y8 = O.moe_forward(xs, mw, routing=(w_gpu, i_gpu), workers=_WORKERS)[0]
    print(f"\n{name} T={T}: vs FP4 oracle max {err:.4f}, vs e4m3 oracle max {_rel_err(got, y8):.4f} "
          f"rms {_rms_err(got, y8):.4f} (of output RMS)")


def test_module_graphs_follow_the_fp4_setting(cuda_device):
    """MoE.forward's cached graphs hold the kernels of the settings in force:
    switching the FP4 mode recaptures, so each call equals the eager layer of
    the current setting."""
    from spark_b200 import _lib
    from spark_b200.moe import MoE
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS["decode"].with_tokens(32)
    layer = make_layer(cfg, seed=5, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    x = layer["x"].to(cuda_device)
    try:
        for on in (False, True, False):
            MoE.set_fp4_activations(on)
            y = moe(x.view(1, 32, -1)).view(32, -1)
            assert torch.equal(y, moe.forward_tokens(x)), on
        y8 = moe(x.view(1, 32, -1)).view(32, -1)
        MoE.set_fp4_activations(True)
        assert not torch.equal(moe(x.view(1, 32, -1)).view(32, -1), y8)
    finally:
        MoE.set_fp4_activations(False)
    _lib.raise_on_device_error()
