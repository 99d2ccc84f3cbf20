"""Expert-parallel orchestration on CPU: two ``gloo`` ranks run
``spark_b200.ep.ep_forward`` with the oracle's restatement of the device steps
(same buffer formats as libdsv4moe.so), and each rank's output must equal the
single-device oracle layer on its tokens bit for bit.  Covers balanced and
one-sided routing and a rank with no tokens."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent
for p in (str(REPO), str(REPO / "deepseek-v4-flash-dgx-spark_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle import moe_oracle as O  # noqa: E402


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


class OracleEPOps:
    """The device steps of ``CudaEPOps`` restated by the oracle."""

    def __init__(self, mw, n_experts, rank, world, hidden):
        self.mw, self.n_experts, self.rank, self.world = mw, n_experts, rank, world
        self.hidden, self.topk = hidden, mw.topk

    def empty(self, shape, dtype, like):
        return torch.empty(shape, dtype=dtype)

    def gate(self, x):
        w, idx, _ = O.gate_forward(x.float().numpy(), self.mw.gate_w, self.mw.gate_bias, self.mw.topk,
                                   self.mw.route_scale)
        return torch.from_numpy(w), torch.from_numpy(idx.astype(np.int64))

    def dispatch(self, x, weights, indices):
        send, counts, ret_pos = O.ep_dispatch(x.float().numpy(), weights.numpy(), indices.numpy(),
                                              self.n_experts, self.world)
        if send.shape[0] == 0:
            send = np.zeros((1, O.ep_row_bytes(self.hidden, self.topk)), np.uint8)
        return torch.from_numpy(send), torch.from_numpy(counts), torch.from_numpy(ret_pos)

    def expert_forward(self, x, recv, recv_counts, n_ret):
        ret, shared = O.ep_expert_forward(self.mw, self.n_experts, self.rank, self.world, x.float().numpy(),
                                          recv.numpy(), recv_counts.numpy())
        assert ret.shape[0] == n_ret
        return _bf16(ret), shared

    def combine(self, ret_recv, ret_pos, indices, x, R, state):
        return _bf16(O.ep_combine(ret_recv.float().numpy(), ret_pos.numpy(), indices.numpy(), state))


def _weights():
    from spark_b200.synthetic import CONFIGS, make_layer

    cfg = CONFIGS["cpu_ref"]
    layer = make_layer(cfg, seed=0, device="cpu")
    mw = O.MoEWeights(
        gate_w=layer["gate_w"].float().numpy(), gate_bias=layer["gate_bias"].numpy(),
        experts={e: O.expert_from_block(layer["blocks"][e].numpy(), cfg.dim, cfg.inter)
                 for e in range(cfg.n_routed)},
        shared=O.shared_from_tensors({k: v.numpy() for k, v in layer["shared"].items()}),
        topk=cfg.topk, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)
    return cfg, mw


def _tokens(cfg, rank, case):
    n = {"balanced": (5, 7, 3, 6), "empty_rank": (6, 0), "one_sided": (4, 3, 2, 5)}[case][rank]
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(n, cfg.dim, generator=g).to(torch.bfloat16)


def _worker(rank, world, port, case, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from spark_b200.ep import ep_forward

        cfg, mw = _weights()
        x = _tokens(cfg, rank, case)
        ops = OracleEPOps(mw, cfg.n_routed, rank, world, cfg.dim)
        routing = None
        if case == "one_sided":  # every route lands on rank 0's experts
            per = cfg.n_routed // world
            g = torch.Generator().manual_seed(7 + rank)
            idx = torch.stack([torch.randperm(per, generator=g)[:cfg.topk] for _ in range(x.shape[0])])
            routing = (torch.rand(x.shape[0], cfg.topk, generator=g), idx.to(torch.int64))
        y = ep_forward(ops, x, routing=routing)
        if routing is None:
            ref = O.moe_forward(x.float().numpy(), mw)[0]
        else:
            ref = O.moe_forward(x.float().numpy(), mw, routing=(routing[0].numpy(), routing[1].numpy()))[0]
        same = bool(np.array_equal(O.f32_to_bf16_bits(y.float().numpy()), O.f32_to_bf16_bits(ref)))
        results[rank] = (tuple(y.shape), same)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case,world", [("balanced", 2), ("empty_rank", 2), ("one_sided", 2),
                                        ("balanced", 4), ("one_sided", 4)])
def test_ep_forward_gloo_ranks_matches_single_device(case, world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), case, results), nprocs=world, join=True,
                           start_method="spawn")
        res = dict(results)
    for rank in range(world):
        n = _tokens(_weights()[0], rank, case).shape[0]
        assert res[rank] == ((n, 1024), True), (rank, res[rank])


def test_ep_dispatch_format_and_positions():
    """Send rows: destination-major, token order; codes and scales are
    act_quant of the token; route entries point at each route's return row."""
    cfg, mw = _weights()
    x = _tokens(cfg, 0, "balanced").float().numpy()
    w, idx, _ = O.gate_forward(x, mw.gate_w, mw.gate_bias, mw.topk, mw.route_scale)
    world, H, k = 4, cfg.dim, cfg.topk
    send, counts, ret_pos = O.ep_dispatch(x, w, idx, cfg.n_routed, world)
    per = cfg.n_routed // world
    q, s = O.act_quant(x)
    assert send.shape == (int(counts[:, 0].sum()), O.ep_row_bytes(H, k)) and O.ep_row_bytes(H, k) % 16 == 0
    n = 0
    for d in range(world):
        toks = [t for t in range(x.shape[0]) if (idx[t] // per == d).any()]
        assert counts[d, 0] == len(toks) and counts[d, 1] == int((idx // per == d).sum())
        for t in toks:
            row = send[n]
            assert np.array_equal(row[:H], q[t]) and np.array_equal(row[H:H + H // 128], s[t])
            meta = np.ascontiguousarray(row[H + H // 128:H + H // 128 + 12 * k]).view(O.EP_META)
            for j in range(k):
                if idx[t, j] // per == d:
                    assert meta["e"][j] == idx[t, j] and meta["w"][j] == w[t, j]
                    assert ret_pos[t, j] == counts[:d, 1].sum() + meta["r"][j]
                else:
                    assert meta["e"][j] == -1 and meta["r"][j] == -1
            n += 1
    assert sorted(ret_pos.reshape(-1).tolist()) == list(range(int(counts[:, 1].sum())))
