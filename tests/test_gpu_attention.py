"""GPU parity of the attention block's hot ops against the oracle
(oracle/attention_oracle.py, pinned to the reference's own
sparse_attn_fallback): the tcgen05 sparse attention at h=64, d=512 on decode
and prefill shapes (split and unsplit index lists, ragged lists, invalid
indices, a query with none), and the FP8 linear at the attention projections'
shapes.

Sparse attention bar: the kernel multiplies bf16 probabilities with the bf16
rows (fp32 sums) and rounds the result to bf16, as the reference's output is.
Simulating exactly that on the CPU gives max |err| of 1.1-4.2% of the output
RMS on these cases (the bf16 output rounding alone: 0.8-2.5%, the max being
taken over up to 10^7 elements), and the kernel measured the same.  So the
test bounds the RMS of the error by 1% of the output RMS (a systematic defect
shows there) and the largest element error by 5%.  FP8 linear: max |err| <=
2e-2 of the RMS, the layer bar."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as A

pytestmark = pytest.mark.gpu


def _rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / (np.sqrt(np.mean(ref ** 2)) + 1e-30))


def _rms_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(np.mean((got - ref) ** 2)) / (np.sqrt(np.mean(ref ** 2)) + 1e-30))


def _attn_close(got, ref):
    assert _rms_err(got, ref) <= 1e-2, _rms_err(got, ref)
    assert _rel_err(got, ref) <= 5e-2, _rel_err(got, ref)


@pytest.fixture
def auto_split():
    """The split-K setting at auto for one test, back to off (the default) after."""
    from spark_b200 import _lib

    lib = _lib.load()
    _lib.check(lib.dsv4_set_k_split(0), "dsv4_set_k_split")
    yield
    _lib.check(lib.dsv4_set_k_split(1), "dsv4_set_k_split")


def _case(B, S, N, K, seed, invalid_frac=0.1, empty_query=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, 64, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(B, N, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(64, generator=g)
    idx = torch.stack([torch.stack([torch.randperm(N, generator=g)[:K] for _ in range(S)]) for _ in range(B)])
    idx = idx.to(torch.int32)
    drop = torch.rand(B, S, K, generator=g) < invalid_frac
    idx[drop] = -1
    if empty_query:
        idx[0, 0, :] = -1
    return q, kv, sink, idx


@pytest.mark.parametrize("B,S,N,K", [
    (1, 1, 4096, 2048),   # decode, one query: the index list split over many CTAs
    (1, 1, 700, 100),     # ragged list shorter than one 128-row chunk
    (2, 40, 300, 256),    # a few queries: two chunks, split in two
    (1, 320, 512, 128),   # many queries: one CTA per query, no combine
])
def test_sparse_attn_matches_the_reference_fallback(cuda_device, B, S, N, K):
    from spark_b200 import _lib
    from spark_b200.attention import sparse_attn

    q, kv, sink, idx = _case(B, S, N, K, seed=B * 1000 + S + K, empty_query=(S > 1))
    scale = 512 ** -0.5
    out = sparse_attn(q.to(cuda_device), kv.to(cuda_device), sink.to(cuda_device), idx.to(cuda_device), scale)
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    ref = A.sparse_attn(q.float().numpy(), kv.float().numpy(), sink.numpy(), idx.numpy(), scale)
    got = out.float().cpu().numpy()
    _attn_close(got, ref)
    if S > 1:
        assert np.all(got[0, 0] == 0)  # no valid index: zeros, as the reference


def test_sparse_attn_out_of_range_index_is_reported_and_skipped(cuda_device):
    from spark_b200 import _lib
    from spark_b200.attention import sparse_attn

    q, kv, sink, idx = _case(1, 2, 256, 64, seed=5, invalid_frac=0.0)
    bad = idx.clone()
    bad[0, 1, 3] = 256  # one past the last kv row
    out = sparse_attn(q.to(cuda_device), kv.to(cuda_device), sink.to(cuda_device), bad.to(cuda_device), 0.05)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="expert index out of range"):
        _lib.raise_on_device_error()
    skipped = idx.clone()
    skipped[0, 1, 3] = -1
    ref = A.sparse_attn(q.float().numpy(), kv.float().numpy(), sink.numpy(), skipped.numpy(), 0.05)
    _attn_close(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("M,K,N", [
    (1, 4096, 1024),      # one row tile, 4 items (k split in 8 under the auto split)
    (37, 4096, 512),
    (64, 4096, 1024),     # decode wq_a
    (16, 3072, 256),      # 6 scale groups (split in 2 under the auto split)
    (5, 1024, 32768),     # enough items: never split
    (200, 8192, 4096),
    (130, 4096, 8192),
])
@pytest.mark.parametrize("k_split", [1, 0])
def test_fp8_linear_matches_the_oracle(cuda_device, M, K, N, k_split):
    from spark_b200 import _lib
    from spark_b200.attention import FP8Linear

    g = torch.Generator().manual_seed(M + K + N)
    lin = FP8Linear(K, N, device=cuda_device)
    w = torch.randn(N, K, generator=g).to(torch.float8_e4m3fn)
    s = torch.randint(119, 124, (N // 128, K // 128), generator=g, dtype=torch.uint8)
    with torch.no_grad():
        lin.weight.view(torch.uint8).copy_(w.view(torch.uint8).to(cuda_device))
        lin.scale.view(torch.uint8).copy_(s.to(cuda_device))
    lin.refresh_scale_atoms()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    lib = _lib.load()
    _lib.check(lib.dsv4_set_k_split(k_split), "dsv4_set_k_split")
    try:
        y = lin(x.to(cuda_device))
        torch.cuda.synchronize()
    finally:
        _lib.check(lib.dsv4_set_k_split(1), "dsv4_set_k_split")
    _lib.raise_on_device_error()
    ref = A.fp8_linear(x.float().numpy(), w.view(torch.uint8).numpy(), s.numpy())
    assert _rel_err(y.float().cpu().numpy(), ref) <= 2e-2


def test_raw_c_abi_and_torch_op_agree_bit_for_bit(cuda_device):
    """The same kernel reached through ctypes (dsv4_sparse_attn with a caller
    workspace) and through torch.ops.dsv4moe.sparse_attn gives equal bytes."""
    from spark_b200 import _lib, ops

    q, kv, sink, idx = _case(1, 3, 900, 384, seed=17)
    q, kv, sink, idx = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda()
    lib = _lib.load()
    B, S, H, D = q.shape
    need = int(lib.dsv4_sparse_attn_workspace_bytes(B, S, idx.shape[-1]))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    _lib.check(lib.dsv4_sparse_attn(_lib.ptr(q), _lib.ptr(kv), _lib.ptr(sink), _lib.ptr(idx), B, S, H, kv.shape[1],
                                    D, idx.shape[-1], 0.05, _lib.ptr(out), _lib.ptr(ws), need, _lib.stream_ptr()),
               "dsv4_sparse_attn")
    via_op = ops.load().sparse_attn(q, kv, sink, idx, 0.05)
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    assert torch.equal(out, via_op)
    with pytest.raises(RuntimeError):
        _lib.check(lib.dsv4_sparse_attn(_lib.ptr(q), _lib.ptr(kv), _lib.ptr(sink), _lib.ptr(idx), B, S, H, kv.shape[1],
                                        D, idx.shape[-1], 0.05, _lib.ptr(out), _lib.ptr(ws), max(need - 256, 0),
                                        _lib.stream_ptr()), "dsv4_sparse_attn")


def test_split_fp8_linear_is_deterministic(cuda_device, auto_split):
    """Under the auto split a decode-sized linear splits its k range; the
    slices are added in slice order, so two calls give equal bytes."""
    from spark_b200 import _lib
    from spark_b200.attention import FP8Linear

    g = torch.Generator().manual_seed(5)
    lin = FP8Linear(4096, 1024, device=cuda_device)
    lin.weight.data.copy_(torch.randn(1024, 4096, generator=g).to(torch.float8_e4m3fn).to(cuda_device))
    lin.refresh_scale_atoms()
    # the workspace holds the 8 slices' fp32 partial sums
    assert int(_lib.load().dsv4_fp8_linear_workspace_bytes(64, 1024, 4096)) >= 8 * 64 * 1024 * 4
    x = torch.randn(64, 4096, generator=g).to(torch.bfloat16).to(cuda_device)
    a, b = lin(x), lin(x)
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    assert torch.equal(a, b)
