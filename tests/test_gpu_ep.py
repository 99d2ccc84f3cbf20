"""Expert parallelism through the C ABI on one GPU: W ranks are emulated in one
process (every rank's arena view is the same fully materialized arena, the
all-to-all exchanges are slices and concatenations), so the device dispatch,
owning-rank forward and combine are checked without a second GPU:

* send rows (codes, scales, route entries), counts and ret_pos equal the
  oracle's ``ep_dispatch`` byte for byte;
* the expert-parallel output equals ``dsv4_moe_forward`` on the same tokens
  bit for bit.

The peer-memory form (``dsv4_ep_*_p2p``) is emulated the same way with W
exchange buffers on the one GPU.  The real multi-process runs, over NCCL and
over peer memory, are ``test_ep_two_gpus`` (needs 2 GPUs)."""

import ctypes
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture
def unsplit_gemms():
    """Bit-identity between the expert-parallel and the single-GPU layer needs
    both to sum each expert GEMM in the same order; small batches would split
    the k range differently on the two sides (their item counts differ), so
    these comparisons run with the split-K GEMM turned off."""
    from spark_b200 import _lib

    lib = _lib.load()
    _lib.check(lib.dsv4_set_k_split(1), "dsv4_set_k_split")
    yield
    _lib.check(lib.dsv4_set_k_split(1), "dsv4_set_k_split")  # the library's default


REPO = Path(__file__).resolve().parent.parent


def _lib():
    from spark_b200 import _lib as L

    return L


def _dispatch(lib, x, w, idx, E, W):
    L = _lib()
    T, H = x.shape
    k = idx.shape[1]
    rb = lib.dsv4_ep_row_bytes(H, k)
    send = torch.zeros((max(T * min(W, k), 1), rb), dtype=torch.uint8, device=x.device)
    counts = torch.empty((W, 2), dtype=torch.int32, device=x.device)
    ret_pos = torch.empty((max(T, 1), k), dtype=torch.int32, device=x.device)
    ws = torch.empty(max(lib.dsv4_ep_dispatch_workspace_bytes(T, W), 1), dtype=torch.uint8, device=x.device)
    L.check(lib.dsv4_ep_dispatch(L.ptr(x), L.ptr(idx), L.ptr(w), T, H, k, E, W, L.ptr(send), send.shape[0],
                                 L.ptr(counts), L.ptr(ret_pos), L.ptr(ws), ws.numel(), L.stream_ptr()),
            "dsv4_ep_dispatch")
    return send, counts, ret_pos


def _emulated_ep(moe, xs, routings, W):
    """Run the five expert-parallel steps for W emulated ranks; returns each
    rank's y and its dispatch outputs."""
    L = _lib()
    lib = L.load()
    E, H = moe.n_routed_experts, moe.dim
    d = moe.layer_desc()
    disp = [_dispatch(lib, x, r[0], r[1], E, W) for x, r in zip(xs, routings)]
    counts = [c.cpu() for _, c, _ in disp]
    # rows: block for rank d inside source s's send buffer
    row_off = [np.concatenate([[0], np.cumsum(c[:, 0].numpy())]) for c in counts]
    route_off = [np.concatenate([[0], np.cumsum(c[:, 1].numpy())]) for c in counts]
    rets, states = [], []
    for dst in range(W):
        recv = torch.cat([disp[s][0][row_off[s][dst]:row_off[s][dst + 1]] for s in range(W)])
        recv_counts = torch.stack([counts[s][dst] for s in range(W)]).to(torch.int32).cuda()
        R = recv.shape[0]
        n_ret = int(sum(int(counts[s][dst, 1]) for s in range(W)))
        T = xs[dst].shape[0]
        ws = torch.empty(max(lib.dsv4_ep_expert_workspace_bytes(ctypes.byref(d), W, T, R), 1), dtype=torch.uint8,
                         device="cuda")
        ret_send = torch.empty((max(n_ret, 1), H), dtype=torch.bfloat16, device="cuda")
        L.check(lib.dsv4_ep_expert_forward(ctypes.byref(d), dst, W, L.ptr(xs[dst]), T, L.ptr(recv.contiguous()), R,
                                           L.ptr(recv_counts), L.ptr(ret_send), n_ret, L.ptr(ws), ws.numel(),
                                           L.stream_ptr()), "dsv4_ep_expert_forward")
        rets.append((ret_send, recv_counts.cpu()))
        states.append((ws, R))
    ys = []
    for s in range(W):
        # return block of rank d for source s: after the routes d received from sources < s
        parts = []
        for dst in range(W):
            rc = rets[dst][1]
            base = int(rc[:s, 1].sum())
            parts.append(rets[dst][0][base:base + int(rc[s, 1])])
        ret_recv = torch.cat(parts).contiguous()
        y = torch.empty_like(xs[s])
        ws, R = states[s]
        L.check(lib.dsv4_ep_combine(ctypes.byref(d), s, W, L.ptr(ret_recv), L.ptr(disp[s][2]),
                                    L.ptr(routings[s][1]), xs[s].shape[0], R, L.ptr(ws), ws.numel(), L.ptr(y),
                                    L.stream_ptr()), "dsv4_ep_combine")
        ys.append(y)
    torch.cuda.synchronize()
    return ys, disp


@pytest.mark.parametrize("name,W,tokens", [("cpu_ref", 2, (9, 4)), ("cpu_ref", 4, (1, 0, 40, 300)),
                                           ("decode", 8, (64, 64, 64, 64, 64, 64, 64, 64)),
                                           ("decode", 2, (1100, 7))])
def test_emulated_ep_is_bit_identical_to_single_gpu(cuda_device, unsplit_gemms, name, W, tokens):
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    L = _lib()
    cfg = CONFIGS[name].with_tokens(max(tokens))
    layer = make_layer(cfg, seed=2, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    E, k, H = cfg.n_routed, cfg.topk, cfg.dim
    xs, routings = [], []
    for r, n in enumerate(tokens):
        g = torch.Generator().manual_seed(50 + r)
        x = torch.randn(n, H, generator=g).to(torch.bfloat16).to(cuda_device)
        w, idx = moe.gate(x) if n else (torch.empty(0, k, device=cuda_device),
                                        torch.empty(0, k, dtype=torch.int64, device=cuda_device))
        xs.append(x.contiguous())
        routings.append((w.float().contiguous(), idx.to(torch.int64).contiguous()))
    ys, disp = _emulated_ep(moe, xs, routings, W)
    L.raise_on_device_error()
    for r, (x, (w, idx)) in enumerate(zip(xs, routings)):
        if x.shape[0] == 0:
            continue
        y_ref = moe.forward_tokens(x, routing=(w, idx))
        torch.cuda.synchronize()
        assert torch.equal(ys[r].view(torch.int16), y_ref.view(torch.int16)), r
        # dispatch bytes against the oracle (the defined part of each row)
        send, counts, ret_pos = disp[r]
        o_send, o_counts, o_ret = O.ep_dispatch(x.float().cpu().numpy(), w.cpu().numpy(), idx.cpu().numpy(), E, W)
        assert np.array_equal(counts.cpu().numpy(), o_counts)
        assert np.array_equal(ret_pos[:x.shape[0]].cpu().numpy(), o_ret)
        used = H + H // 128 + 12 * k
        assert np.array_equal(send[:o_send.shape[0], :used].cpu().numpy(), o_send[:, :used])


def _emulated_peer_ep(moe, xs, routings, W, epochs=(1, 2)):
    """The peer-memory steps for W emulated ranks on one GPU: W exchange
    buffers, peer_bases = those W buffers.  All of one step's launches (every
    rank's dispatch, then every owner's forward, then every combine) precede
    the next step's in one stream, so each flag a wait kernel polls was raised
    by a kernel that already finished: nothing waits on a concurrent kernel."""
    L = _lib()
    lib = L.load()
    E, H, k = moe.n_routed_experts, moe.dim, moe.n_activated_experts
    d = moe.layer_desc()
    cap = max(max(x.shape[0] for x in xs), 1)
    nbytes = lib.dsv4_ep_exchange_bytes(H, k, W, cap)
    assert nbytes > 0
    bufs = []
    for _ in range(W):
        p = ctypes.c_void_p()
        L.check(lib.dsv4_ep_exchange_alloc(torch.cuda.current_device(), nbytes, ctypes.byref(p)), "alloc")
        bufs.append(p)
    bases = torch.tensor([b.value for b in bufs], dtype=torch.int64, device="cuda")
    out = []
    try:
        for epoch in epochs:
            disp = []
            for r, (x, (w, idx)) in enumerate(zip(xs, routings)):
                T = x.shape[0]
                ret_pos = torch.empty((max(T, 1), k), dtype=torch.int32, device="cuda")
                ws = torch.empty(max(lib.dsv4_ep_p2p_dispatch_workspace_bytes(T, W), 1), dtype=torch.uint8,
                                 device="cuda")
                L.check(lib.dsv4_ep_dispatch_p2p(L.ptr(x), L.ptr(idx), L.ptr(w), T, H, k, E, W, r, L.ptr(bases),
                                                 cap, epoch, L.ptr(ret_pos), L.ptr(ws), ws.numel(), L.stream_ptr()),
                        "dsv4_ep_dispatch_p2p")
                disp.append((ret_pos, ws))
            wss = []
            for r, x in enumerate(xs):
                T = x.shape[0]
                ws = torch.empty(max(lib.dsv4_ep_p2p_expert_workspace_bytes(ctypes.byref(d), W, T, cap), 1),
                                 dtype=torch.uint8, device="cuda")
                L.check(lib.dsv4_ep_expert_forward_p2p(ctypes.byref(d), r, W, L.ptr(x), T, bufs[r], L.ptr(bases),
                                                       cap, epoch, L.ptr(ws), ws.numel(), L.stream_ptr()),
                        "dsv4_ep_expert_forward_p2p")
                wss.append(ws)
            ys = []
            for r, (x, (w, idx)) in enumerate(zip(xs, routings)):
                y = torch.empty_like(x)
                L.check(lib.dsv4_ep_combine_p2p(ctypes.byref(d), r, W, bufs[r], L.ptr(disp[r][0]), L.ptr(idx),
                                                x.shape[0], cap, epoch, L.ptr(wss[r]), wss[r].numel(), L.ptr(y),
                                                L.stream_ptr()), "dsv4_ep_combine_p2p")
                ys.append(y)
            torch.cuda.synchronize()
            L.raise_on_device_error()
            out.append(ys)
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            lib.dsv4_ep_exchange_free(b)
    return out


@pytest.mark.parametrize("name,W,tokens,epochs", [("cpu_ref", 2, (9, 4), (1, 2)),
                                                  ("cpu_ref", 4, (1, 0, 40, 300), (1, 2)),
                                                  ("cpu_ref", 4, (1, 0, 40, 300), (0, 0, 0)),
                                                  ("decode", 8, (64, 64, 64, 64, 64, 64, 64, 64), (0, 0)),
                                                  ("decode", 2, (1100, 7), (1, 2))])
def test_emulated_peer_ep_is_bit_identical_to_single_gpu(cuda_device, unsplit_gemms, name, W, tokens, epochs):
    """Dispatch rows stored into the owners' exchange buffers, return rows into
    the sources', epoch flags in both directions (epochs given by the host, or
    0: counted on the device): every rank's result equals the single-GPU layer
    bit for bit, on consecutive calls (buffer reuse)."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    cfg = CONFIGS[name].with_tokens(max(tokens))
    layer = make_layer(cfg, seed=2, device="cpu")
    moe = build_moe(layer, device=cuda_device)
    k, H = cfg.topk, cfg.dim
    xs, routings = [], []
    for r, n in enumerate(tokens):
        g = torch.Generator().manual_seed(70 + r)
        x = torch.randn(n, H, generator=g).to(torch.bfloat16).to(cuda_device)
        w, idx = moe.gate(x) if n else (torch.empty(0, k, device=cuda_device),
                                        torch.empty(0, k, dtype=torch.int64, device=cuda_device))
        xs.append(x.contiguous())
        routings.append((w.float().contiguous(), idx.to(torch.int64).contiguous()))
    runs = _emulated_peer_ep(moe, xs, routings, W, epochs)
    for ys in runs:
        for r, (x, (w, idx)) in enumerate(zip(xs, routings)):
            if x.shape[0] == 0:
                continue
            y_ref = moe.forward_tokens(x, routing=(w, idx))
            torch.cuda.synchronize()
            assert torch.equal(ys[r].view(torch.int16), y_ref.view(torch.int16)), r


def test_peer_wait_times_out_with_an_error_not_a_hang(cuda_device):
    """An owner whose sources never signal: the wait kernel gives up after its
    bound, latches DSV4_DEVERR_TIMEOUT_PEER, and the context stays usable."""
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    L = _lib()
    lib = L.load()
    cfg = CONFIGS["cpu_ref"].with_tokens(4)
    moe = build_moe(make_layer(cfg, seed=2, device="cpu"), device=cuda_device)
    d = moe.layer_desc()
    W, cap = 2, 4
    p = ctypes.c_void_p()
    L.check(lib.dsv4_ep_exchange_alloc(torch.cuda.current_device(),
                                       lib.dsv4_ep_exchange_bytes(cfg.dim, cfg.topk, W, cap), ctypes.byref(p)),
            "alloc")
    try:
        bases = torch.tensor([p.value, p.value], dtype=torch.int64, device="cuda")
        ws = torch.empty(lib.dsv4_ep_p2p_expert_workspace_bytes(ctypes.byref(d), W, 0, cap), dtype=torch.uint8,
                         device="cuda")
        L.check(lib.dsv4_ep_expert_forward_p2p(ctypes.byref(d), 0, W, None, 0, p, L.ptr(bases), cap, 7,
                                               L.ptr(ws), ws.numel(), L.stream_ptr()), "forward")
        # the exchange learns of the latched timeout without synchronising:
        # the word is copied back after the call and read by the next call
        from spark_b200.ep import PeerExchange

        ex = PeerExchange.__new__(PeerExchange)
        ex.lib, ex.poisoned, ex._err_event = lib, None, None
        ex._err_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        ex.check_poisoned()  # nothing recorded yet: no error
        ex.note_call_end()
        torch.cuda.synchronize()
        # inside a stream capture (a CUDA graph of the layer) the check must not
        # touch the event, which cannot be queried then
        g, s = torch.cuda.CUDAGraph(), torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=s):
            ex.check_poisoned()
            ex.note_call_end()  # no copy is enqueued into the graph either
            torch.ones(4, device="cuda").mul_(2)
        del g
        for _ in range(2):  # poisoned for good, not just once
            with pytest.raises(RuntimeError, match="poisoned"):
                ex.check_poisoned()
        with pytest.raises(RuntimeError, match="exchange flag"):
            L.raise_on_device_error()
        x = torch.ones(8, device="cuda")
        assert float((x * 2).sum()) == 16.0  # the context still works
    finally:
        torch.cuda.synchronize()
        lib.dsv4_ep_exchange_free(p)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_ep_two_gpus(mode):
    """Two processes, one GPU each, exchanging through NCCL all-to-all or
    through NVLink peer memory: every rank's MoE.forward equals the single-GPU
    layer on its tokens bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", EP_MODE=mode,
               PYTHONPATH=f"{REPO}:{REPO / 'deepseek-v4-flash-dgx-spark_b200'}")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(REPO / "tests" / "ep_nccl_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("EP_OK") == 2, r.stdout[-3000:]
