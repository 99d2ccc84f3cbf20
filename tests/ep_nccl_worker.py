"""One rank of the two-GPU expert-parallel check (launched by
tests/test_gpu_ep.py::test_ep_two_gpus through torch.distributed.run;
EP_MODE=peer exchanges over NVLink peer memory, else over NCCL).

Every rank builds the same synthetic layer, keeps the experts it owns in its
arena, routes its own tokens and runs ``MoE.forward`` over NCCL; the result
must equal the single-GPU layer (a second, world-size-1 MoE holding every
expert) bit for bit.  Prints EP_OK on success."""

import datetime
import os
import sys

import torch
import torch.distributed as dist


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from spark_b200.synthetic import CONFIGS, build_moe, make_layer

        cfg = CONFIGS["decode"].with_tokens(64)
        layer = make_layer(cfg, seed=4, device="cpu")
        singles = [dist.new_group([r]) for r in range(world)]  # every rank creates every group
        full = build_moe(layer, device=dev, group=singles[rank])  # single-GPU layer, every expert
        ep = build_moe(layer, device=dev)  # expert-parallel over the world: own experts only
        assert ep.world == world and ep.n_local_experts == cfg.n_routed // world
        if os.environ.get("EP_MODE", "nccl") == "peer":
            ep.enable_peer_exchange(64)
        ok = True
        # the second call reuses the exchange buffers; over peer memory
        # MoE.forward captures a graph per token count, and the third call
        # replays the graphs of the first (the ranks' counts differ)
        for step in range(3):
            n = ((64, 37), (5, 64), (64, 37))[step][rank % 2]
            g = torch.Generator().manual_seed(1000 + 10 * step + rank)
            x = torch.randn(1, n, cfg.dim, generator=g).to(torch.bfloat16).to(dev)
            y = ep(x)
            y_ref = full(x)
            torch.cuda.synchronize()
            ok = ok and torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
        from spark_b200 import _lib

        _lib.raise_on_device_error()
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if ok:
            print("EP_OK", rank, flush=True)
        else:
            diff = (y.float() - y_ref.float()).abs().max().item()
            print("EP_MISMATCH", rank, diff, flush=True)
        if getattr(ep, "peer_exchange", None) is not None:
            dist.barrier()  # no rank unmaps a buffer another may still store to
            ep.peer_exchange.close()
        return 0 if int(flag.item()) == 1 else 1
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
