"""dsv4_expert_forward_static: the expert forward for callers that may not
allocate device memory (their host owns every allocation and passes only the
input and output buffers).  Its scratch is a fixed array of device memory owned
by the library; this file checks, through the C ABI, that it gives the same
results as the workspace entry point dsv4_expert_forward on two calls in a row
(the second call sees the first call's leftovers in the shared scratch), and
that it refuses a batch whose scratch would not fit.  Both entry points run
the same plan and kernels, so "the same results" means bit-identical.

Collected last on purpose, so a run that stops at the first failure has
already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

def _rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / (np.sqrt(np.mean(ref ** 2)) + 1e-30))


def _expert(kind, device, H=4096, I=2048):
    from spark_b200.moe import FP4, Expert, packed_block_bytes
    from spark_b200.synthetic import routed_blocks, shared_expert

    if kind == "routed":
        e = Expert(H, I, dtype=FP4, swiglu_limit=10.0, device=device)
        e.block[: packed_block_bytes(H, I)].copy_(routed_blocks(1, H, I, 77)[0].to(device))
    else:
        e = Expert(H, I, swiglu_limit=10.0, device=device)
        sh = shared_expert(H, I, 78)
        with torch.no_grad():
            for n in ("w1", "w2", "w3"):
                getattr(e, n).weight.view(torch.uint8).copy_(sh[f"{n}.weight"].to(device))
                getattr(e, n).scale.view(torch.uint8).copy_(sh[f"{n}.scale"].to(device))
    e.refresh_scale_atoms()
    return e


def _with_workspace(lib, L, e, x, w):
    from spark_b200._lib import check, ptr, stream_ptr

    T = x.shape[0]
    y = torch.empty_like(x)
    need = lib.dsv4_expert_workspace_bytes(ctypes.byref(L), T)
    ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    check(lib.dsv4_expert_forward(ctypes.byref(L), 0 if e.fp4 else -1, ptr(x), T, ptr(w), ptr(y), ptr(ws), need,
                                  stream_ptr()), "dsv4_expert_forward")
    return y


def _static(lib, L, e, x, w):
    from spark_b200._lib import check, ptr, stream_ptr

    y = torch.empty_like(x)
    check(lib.dsv4_expert_forward_static(ctypes.byref(L), 0 if e.fp4 else -1, ptr(x), x.shape[0], ptr(w), ptr(y),
                                         stream_ptr()), "dsv4_expert_forward_static")
    return y


def _largest_fitting_batch(lib, L):
    limit = lib.dsv4_expert_static_scratch_bytes()
    T = 1
    while lib.dsv4_expert_workspace_bytes(ctypes.byref(L), T + 1) <= limit:
        T += 1
    return T


@pytest.mark.parametrize("kind", ["routed", "shared"])
def test_static_scratch_matches_workspace_entry(cuda_device, kind):
    """Both entry points run the same plan and kernels, so their outputs must
    be bit-identical.  The shared scratch is first filled by a call at the
    largest batch that fits, on NaN inputs (so its quantized activations and
    intermediate codes are NaN codes); two calls in a row then run on those
    leftovers and must still equal the workspace entry bit for bit."""
    from spark_b200 import _lib

    lib = _lib.load()
    e = _expert(kind, cuda_device)
    L = e._desc()
    T_max = _largest_fitting_batch(lib, L)
    poison = torch.full((T_max, 4096), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    pw = torch.ones(T_max, device=cuda_device) if kind == "routed" else None
    _static(lib, L, e, poison, pw)
    torch.cuda.synchronize()
    g = torch.Generator().manual_seed(11 if kind == "routed" else 12)
    for T in (37, 5):
        x = torch.randn(T, 4096, generator=g).to(torch.bfloat16).to(cuda_device)
        w = (torch.rand(T, generator=g) + 0.25).to(cuda_device) if kind == "routed" else None
        ref = _with_workspace(lib, L, e, x, w)
        got = _static(lib, L, e, x, w)
        torch.cuda.synchronize()
        _lib.raise_on_device_error()
        assert bool(torch.isfinite(ref.float()).all()), (kind, T)
        assert torch.equal(got, ref), (kind, T, _rel_err(got.float().cpu().numpy(), ref.float().cpu().numpy()))


def test_static_scratch_rejects_batches_that_do_not_fit(cuda_device):
    from spark_b200 import _lib

    lib = _lib.load()
    e = _expert("routed", cuda_device)
    L = e._desc()
    limit = lib.dsv4_expert_static_scratch_bytes()
    assert limit == 4 << 20
    T_ok = 1
    while lib.dsv4_expert_workspace_bytes(ctypes.byref(L), T_ok + 32) <= limit:
        T_ok += 32
    T_bad = T_ok + 32
    assert lib.dsv4_expert_workspace_bytes(ctypes.byref(L), T_bad) > limit
    x = torch.zeros(T_bad, 4096, dtype=torch.bfloat16, device=cuda_device)
    y = torch.full_like(x, 7.0)
    rc = lib.dsv4_expert_forward_static(ctypes.byref(L), 0, _lib.ptr(x), T_bad, None, _lib.ptr(y),
                                        _lib.stream_ptr())
    assert rc == _lib.ERR_WORKSPACE
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())  # refused before any work
