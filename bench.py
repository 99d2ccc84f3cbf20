"""Benchmark of the B200 routed-expert MoE layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|prefill|stack|attention] [--tokens T]

One step = one MoE layer forward (gate -> route plan -> permute/quant ->
grouped GEMM1 -> grouped GEMM2 -> combine) over one batch of synthetic tokens,
inputs resident in HBM.  The default workload is the single-GPU decode layer
(H=4096, 256 routed experts top-6 + 1 shared, I=2048, FP4 routed / FP8 shared,
64 tokens, uniform routing).  The L2 cache (126 MB) is flushed between timed
steps by writing a 256 MB buffer outside the timed events.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's
own ``LazyMoE.forward`` on the host cores instead, at the same configuration:
its packed store, expert cache and native packed loader (the reference
installed into baseline/_ref, its loader compiled from source into
oracle/_ref), with the official Gate / Expert - absent from the reference -
stood in for by CPU classes with the oracle's semantics
(oracle/reference_runtime.py).  Without baseline/_ref it falls back to the
oracle restatement and says so.

With torchrun (N > 1) the layer is expert-parallel: rank r owns experts
[r*E/N, (r+1)*E/N), routes its own tokens (64 per GPU for decode, 4096 for
prefill) and exchanges FP8 rows / bf16 route outputs with the owning ranks over
NCCL (weak scaling: tokens per GPU fixed).  Each step is timed with CUDA events
on every rank; the reported time is the max over ranks.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "deepseek-v4-flash-dgx-spark_b200"))
sys.path.insert(0, str(REPO))

METRIC = "moe_layer_tokens_per_s"
UNIT = "tokens/s"


def _parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="decode", choices=["decode", "prefill", "stack", "attention"],
                   help="stack: the full-depth MoE-only decode stack (--layers layers, bf16 residual)")
    p.add_argument("--layers", type=int, default=43)
    p.add_argument("--tokens", type=int, default=None)
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true", help="skip the output check against the oracle")
    p.add_argument("--no-config4", action="store_true",
                   help="N>1: skip the 4096-token/GPU expert-parallel measurements after the headline")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                   help="expert-parallel exchange (N>1): NVLink peer memory from the kernels, or NCCL all-to-all")
    p.add_argument("--experts", type=int, default=None,
                   help="routed experts per layer (default: the workload's 256); profiling runs use fewer")
    return p.parse_args()


def _dist_init(n):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _traffic_record(workload: str):
    """ncu DRAM traffic per GEMM launch, committed under profiles/ (null if absent)."""
    try:
        data = json.loads((REPO / "profiles" / "traffic.json").read_text())
        return data.get(workload)
    except (OSError, ValueError):
        return None


def _parity_block(layer, x_rows, y_rows, w_rows, i_rows):
    """Checker, outside every timed region: the layer outputs of a few tokens
    against the oracle restatement on the device's own routing (tokens are
    independent, so only the experts they touch are decoded).  The oracle
    only checks here; nothing it computes is measured or returned as output."""
    import numpy as np

    from oracle import moe_oracle as O

    cfg = layer["cfg"]
    x_rows, y_rows = x_rows.float().cpu().numpy(), y_rows.float().cpu().numpy()
    w_rows, i_rows = w_rows.float().cpu().numpy(), i_rows.cpu().numpy().astype(np.int64)
    experts = sorted(set(int(e) for e in i_rows.reshape(-1).tolist()))
    mw = O.MoEWeights(
        gate_w=None, gate_bias=None,
        experts={e: O.expert_from_block(layer["blocks"][e].cpu().numpy(), cfg.dim, cfg.inter) for e in experts},
        shared=O.shared_from_tensors({k: v.cpu().numpy() for k, v in layer["shared"].items()}),
        topk=cfg.topk, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)
    ref = O.moe_forward(x_rows, mw, routing=(w_rows, i_rows), workers=min(16, os.cpu_count() or 1))[0]
    err = float(np.max(np.abs(y_rows.astype(np.float64) - ref)) / (np.sqrt(np.mean(ref.astype(np.float64) ** 2))
                                                                  + 1e-30))
    return {"checked_tokens": int(x_rows.shape[0]), "experts": len(experts), "max_err_rms": round(err, 6),
            "tol": 2e-2, "ok": bool(err <= 2e-2), "against": "oracle restatement on the device's routing"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, world, rank, local):
    if world > 1:
        return run_ours_ep(args, world, rank, local)
    import torch
    import torch.distributed as dist

    from spark_b200 import _lib
    from spark_b200.synthetic import (CONFIGS, algorithmic_decode_bytes, algorithmic_flops, build_moe,
                                      make_layer)

    dev = torch.device("cuda", local)
    base = CONFIGS[args.workload]
    if args.experts:
        from dataclasses import replace as _replace

        base = _replace(base, n_routed=args.experts)
    T = args.tokens or (64 if args.workload == "decode" else base.tokens)
    cfg = base.with_tokens(T)
    layer = make_layer(cfg, seed=args.seed + 1000 * rank, device=dev)
    moe = build_moe(layer, device=dev)
    x = layer["x"]
    lib = _lib.load()
    ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=dev)
    y = torch.empty_like(x)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def step():
        moe.forward_tokens(x, workspace=ws, out=y)

    # warm-up, then capture the layer in CUDA graphs (launch-bound at decode sizes):
    # `graph` is the timed layer; `graph_prof` adds the library's stage events
    # and is replayed separately for the per-stage times
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    n_launch0 = lib.dsv4_kernel_launches()
    with torch.cuda.graph(graph, stream=s):
        step()
    launches_per_step = lib.dsv4_kernel_launches() - n_launch0  # kernels in the captured layer
    lib.dsv4_profile_enable(1)
    with torch.cuda.stream(s):
        step()  # profiling events exist before capture
    torch.cuda.current_stream().wait_stream(s)
    graph_prof = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_prof, stream=s):
        step()
    graph.replay()
    graph_prof.replay()
    torch.cuda.synchronize()
    lib.dsv4_profile_enable(0)

    # output parity of a sample of tokens (checker, before the timed region)
    parity = None
    if not args.no_parity:
        y_chk = moe.forward_tokens(x, workspace=ws)
        w_chk, i_chk = moe.gate(x)
        torch.cuda.synchronize()
        pick = torch.arange(0, T, max(1, T // 8), device=dev)[:8]
        parity = _parity_block(layer, x[pick], y_chk[pick], w_chk[pick], i_chk[pick])

    # touched experts of this batch (for the algorithmic-bytes count)
    offs = (ctypes.c_longlong * 17)()
    d = moe.layer_desc()
    lib.dsv4_moe_workspace_layout(ctypes.byref(d), T, offs, 17)
    counts = ws[offs[3]:offs[3] + (cfg.n_routed + 1) * 4].view(torch.int32)[: cfg.n_routed]
    touched = int((counts > 0).sum())
    rows = int(counts.sum()) + T

    # timed region
    times = []
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    for _ in range(args.steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    _lib.raise_on_device_error()
    ms = sum(times) / len(times)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # per-stage times (library events on the launching stream), outside the timed region
    lib.dsv4_profile_enable(1)
    stage = torch.zeros(6, dtype=torch.float64)
    buf = (ctypes.c_float * 6)()
    for _ in range(args.steps):
        flush.fill_(1)
        graph_prof.replay()
        torch.cuda.synchronize()
        lib.dsv4_profile_read(buf, 6)
        stage += torch.tensor(list(buf), dtype=torch.float64)
    lib.dsv4_profile_enable(0)
    stage_ms = (stage / args.steps).tolist()

    # end to end with host buffers (pinned), copies inside the timed region:
    # through the module call a user makes (MoE.forward, which replays its
    # captured graph for this token count), and beside it one eager C ABI
    # call per step (MoE.forward_tokens -> dsv4_moe_forward)
    x_host = x.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_run(call):
        ts = []
        for i in range(args.warmup + args.steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            x_dev.copy_(x_host, non_blocking=True)
            y_host.copy_(call(), non_blocking=True)
            e1.record()
            e1.synchronize()
            if i >= args.warmup:
                ts.append(e0.elapsed_time(e1))
        ms_ = sum(ts) / len(ts)
        if world > 1:
            t = torch.tensor([ms_], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_ = float(t.item())
        return ms_

    e2e_ms = e2e_run(lambda: moe(x_dev.view(1, T, -1)).view(T, -1))
    e2e_eager_ms = e2e_run(lambda: moe.forward_tokens(x_dev, workspace=ws, out=y))

    peaks, peak_src = _peaks()
    if min(stage_ms) < 0:
        raise RuntimeError(f"stage timing events were not recorded: {stage_ms}")
    gemm_ms = stage_ms[3] + stage_ms[4]
    if args.workload == "decode":
        alg = algorithmic_decode_bytes(cfg, touched, T)
        # the expert GEMMs move the touched experts' blocks + the shared expert
        gemm_bytes = alg - cfg.n_routed * cfg.dim * 2 - cfg.n_routed * 4 - 4 * T * cfg.dim
        achieved = gemm_bytes / (gemm_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": _traffic_record("decode"),
                "kernel": "expert_gemm_kernel (GEMM1 w1|w3 + GEMM2 w2), per layer",
                "algorithmic_bytes": gemm_bytes, "kernel_ms": round(gemm_ms, 4), "peak_source": peak_src}
    else:
        flops = algorithmic_flops(cfg, T) - 2.0 * T * cfg.dim * cfg.n_routed
        achieved = flops / (gemm_ms * 1e-3) / 1e12
        fp8_peak = 2 * peaks.get("bf16_tflops", 1590.0)
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": fp8_peak, "unit": "TFLOP/s",
                "frac": round(achieved / fp8_peak, 4), "traffic": _traffic_record("prefill"),
                "kernel": "expert_gemm_kernel (GEMM1 + GEMM2), kind::mxf8f6f4 (e4m3 x e2m1, FP8 rate)",
                "algorithmic_flops": flops, "kernel_ms": round(gemm_ms, 4),
                "peak_source": f"{peak_src} bf16 x2 (dense FP8 rate)"}

    result = {
        "metric": METRIC, "value": round(world * T / (ms * 1e-3), 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e2m1/e4m3 x e4m3 -> f32 (bf16 out)",
        "data": "synthetic (seeded; random-init weights of the V4-Flash MoE shapes)",
        "config": {"workload": f"{args.workload}_moe_layer", "tokens_per_gpu": T, "hidden": cfg.dim,
                   "inter": cfg.inter, "routed_experts": cfg.n_routed, "topk": cfg.topk, "shared_experts": 1,
                   "routing": "uniform" if cfg.bias == "zero" else "zipf1.2",
                   "experts_touched": touched, "rows": rows, "l2": "flushed (256 MB write) between steps",
                   "parallelism": "single",
                   "cuda_graph": True},
        "stage_ms": dict(zip(["gate", "plan", "permute", "gemm1", "gemm2", "combine"],
                             [round(v, 5) for v in stage_ms])),
        "roofline": roof,
        "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 2), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": y.numel() * 2,
                "ms_per_step": round(e2e_ms, 5),
                "path": "MoE.forward (module call; replays the layer's captured CUDA graph for this token count)",
                "eager_c_abi": {"ms_per_step": round(e2e_eager_ms, 5),
                                "value": round(world * T / (e2e_eager_ms * 1e-3), 2),
                                "path": "MoE.forward_tokens -> dsv4_moe_forward, one eager call per step"}},
        "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
    }
    if parity is not None:
        result["parity"] = parity
    return result, cfg, layer, moe


def run_ours_ep(args, world, rank, local):
    """Expert-parallel layer over `world` GPUs (one process each)."""
    import torch
    import torch.distributed as dist

    from spark_b200 import _lib
    from spark_b200.ep import ep_moe_forward
    from spark_b200.moe import packed_block_bytes
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    dev = torch.device("cuda", local)
    base = CONFIGS[args.workload]
    if args.experts:
        from dataclasses import replace as _replace

        base = _replace(base, n_routed=args.experts)
    T = args.tokens or (64 if args.workload == "decode" else 4096)
    cfg = base.with_tokens(T)
    layer = make_layer(cfg, seed=args.seed, device=dev)  # same weights on every rank
    moe = build_moe(layer, device=dev)                   # own experts only
    g = torch.Generator(device=dev).manual_seed(args.seed + 1000 * (rank + 1))
    x = torch.randn(T, cfg.dim, generator=g, device=dev).to(torch.bfloat16)
    lib = _lib.load()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    exchange = args.exchange
    exchange_note = ""
    if exchange == "peer":
        try:
            moe.enable_peer_exchange(T)  # collective: every rank, same capacity, same outcome
        except RuntimeError as exc:  # raised on every rank together: all fall back to NCCL
            exchange, exchange_note = "nccl", f" (peer-memory set-up failed: {exc})"

    for _ in range(max(args.warmup, 3)):
        y = ep_moe_forward(moe, x)
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    parity = _ep_parity(args, moe, layer, x, world, rank, dev) if not args.no_parity else None
    n0 = lib.dsv4_kernel_launches()
    y = ep_moe_forward(moe, x)
    launches_per_step = lib.dsv4_kernel_launches() - n0
    torch.cuda.synchronize()

    # work this rank's experts do per step (from every rank's routing)
    w_idx = moe.gate(x)[1].to(torch.int64).reshape(-1)
    all_idx = torch.empty(world * w_idx.numel(), dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(all_idx, w_idx)
    e0_, e1_ = moe.experts_start_idx, moe.experts_end_idx
    local_routes = int(((all_idx >= e0_) & (all_idx < e1_)).sum())
    touched = int(torch.unique(all_idx[(all_idx >= e0_) & (all_idx < e1_)]).numel())
    global_touched = int(torch.unique(all_idx).numel())

    # Over peer memory a layer call has no host collective or host sync: every
    # rank captures it in a CUDA graph and replays it in lockstep (the epochs
    # are counted on the device).  Through NCCL it runs eagerly.
    graph = None
    if exchange == "peer":
        s_cap = torch.cuda.Stream(device=dev)
        s_cap.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s_cap):
            y = ep_moe_forward(moe, x)
        torch.cuda.current_stream().wait_stream(s_cap)
        graph.replay()
        torch.cuda.synchronize()
        _lib.raise_on_device_error()

    times = []
    clocks = ClockSampler(local)
    dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    for _ in range(args.steps):
        flush.fill_(1)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if graph is not None:
            graph.replay()
        else:
            y = ep_moe_forward(moe, x)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    _lib.raise_on_device_error()
    ms_local = sum(times) / len(times)

    # per-stage times of the owning-rank forward (library events), eager, outside the timed region
    lib.dsv4_profile_enable(1)
    stage = torch.zeros(6, dtype=torch.float64)
    buf = (ctypes.c_float * 6)()
    for _ in range(args.steps):
        dist.barrier()
        y = ep_moe_forward(moe, x)
        torch.cuda.synchronize()
        lib.dsv4_profile_read(buf, 6)
        stage += torch.tensor(list(buf), dtype=torch.float64)
    lib.dsv4_profile_enable(0)
    _lib.raise_on_device_error()
    stage_ms = (stage / args.steps).tolist()
    gemm_ms_local = stage_ms[3] + stage_ms[4]
    t = torch.tensor([ms_local, gemm_ms_local], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, gemm_ms = float(t[0]), float(t[1])

    # end to end: pinned host tokens in, MoE.forward over NCCL, result to the host
    x_host = x.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    e2e = []
    for i in range(args.warmup + args.steps):
        flush.fill_(1)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        xd = x_host.to(dev, non_blocking=True)
        yd = moe(xd.view(1, T, -1)).view(T, -1)
        y_host.copy_(yd, non_blocking=True)
        e1.record()
        e1.synchronize()
        if i >= args.warmup:
            e2e.append(e0.elapsed_time(e1))
    t = torch.tensor([sum(e2e) / len(e2e)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())

    peaks, peak_src = _peaks()
    H, I = cfg.dim, cfg.inter
    shared_bytes = 3 * I * H + 3 * (I // 128) * (H // 128)
    if args.workload == "decode":
        gemm_bytes = touched * packed_block_bytes(H, I) + shared_bytes
        achieved = gemm_bytes / (gemm_ms_local * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                "kernel": "expert_gemm_kernel (GEMM1 + GEMM2) of rank 0's owned experts, per layer",
                "algorithmic_bytes": gemm_bytes, "kernel_ms": round(gemm_ms_local, 4), "peak_source": peak_src}
    else:
        flops = (local_routes + T) * 3 * 2.0 * H * I
        fp8_peak = 2 * peaks.get("bf16_tflops", 1590.0)
        achieved = flops / (gemm_ms_local * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": fp8_peak, "unit": "TFLOP/s",
                "frac": round(achieved / fp8_peak, 4), "traffic": None,
                "kernel": "expert_gemm_kernel (GEMM1 + GEMM2) of rank 0's owned experts",
                "algorithmic_flops": flops, "kernel_ms": round(gemm_ms_local, 4),
                "peak_source": f"{peak_src} bf16 x2 (dense FP8 rate)"}
    rb = lib.dsv4_ep_row_bytes(H, cfg.topk)
    result = {
        "metric": METRIC, "value": round(world * T / (ms * 1e-3), 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e2m1/e4m3 x e4m3 -> f32 (bf16 out)",
        "data": "synthetic (seeded; random-init weights of the V4-Flash MoE shapes)",
        "config": {"workload": f"{args.workload}_moe_layer", "tokens_per_gpu": T, "hidden": H, "inter": I,
                   "routed_experts": cfg.n_routed, "topk": cfg.topk, "shared_experts": 1,
                   "routing": "uniform" if cfg.bias == "zero" else "zipf1.2",
                   "experts_touched": global_touched, "rank0_experts_touched": touched,
                   "rank0_routes": local_routes, "l2": "flushed (256 MB write) between steps",
                   "parallelism": f"ep{world}", "exchange": (
                       "NVLink peer memory: the pack kernel stores FP8 rows into the owners' buffers, the "
                       "return kernel stores bf16 route rows into the sources' (epoch flags, no host sync)"
                       if exchange == "peer" else "NCCL all-to-all" + exchange_note) +
                   f"; {rb} B per token and owning rank, {2 * H} B per route",
                   "cuda_graph": graph is not None},
        "stage_ms_rank0": dict(zip(["unpack", "plan", "scatter", "gemm1", "gemm2", "return_gather"],
                                   [round(v, 5) for v in stage_ms])),
        "roofline": roof,
        "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 2), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": y.numel() * 2,
                "ms_per_step": round(e2e_ms, 5),
                "path": "MoE.forward -> spark_b200.ep (C ABI, " +
                        ("NVLink peer memory; the module call replays its captured CUDA graph for this "
                         "token count when it is at most 1024)" if exchange == "peer" else "NCCL, eager)")},
        "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
    }
    if parity is not None:
        result["parity"] = parity
    del graph
    if getattr(moe, "peer_exchange", None) is not None:
        torch.cuda.synchronize()
        dist.barrier()  # no rank frees its buffer while a peer could still store into it
        moe.peer_exchange.close()
        moe.peer_exchange = None
    if args.workload == "decode" and not args.no_config4:
        del moe, layer
        torch.cuda.empty_cache()
        result["config4"] = _ep_config4(args, world, rank, local)
        return result, cfg, None, None
    return result, cfg, layer, moe


def _ep_parity(args, moe, layer, x, world, rank, dev):
    """Checker, before the timed region: a few tokens of every rank (their
    inputs, expert-parallel outputs and routing) gathered to rank 0 and
    compared with the oracle there.  Every rank takes the same collective
    steps; the other ranks wait at the barrier while rank 0 checks."""
    import torch
    import torch.distributed as dist

    from spark_b200.ep import ep_moe_forward

    T, H = x.shape
    y = ep_moe_forward(moe, x)
    w, idx = moe.gate(x)
    n = min(T, 4 if world <= 2 else 2)
    pick = torch.arange(0, T, max(1, T // n), device=dev)[:n]
    parts = {"x": x[pick].contiguous(), "y": y[pick].contiguous(), "w": w[pick].float().contiguous(),
             "i": idx[pick].to(torch.int64).contiguous()}
    gathered = {}
    for key, t in parts.items():
        g = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
        dist.all_gather_into_tensor(g, t)
        gathered[key] = g
    torch.cuda.synchronize()
    res = None
    if rank == 0:
        res = _parity_block(layer, gathered["x"], gathered["y"], gathered["w"], gathered["i"])
        res["ranks"] = world
    dist.barrier()
    return res


def _ep_config4(args, world, rank, local):
    """The expert-parallel layer at 4096 tokens per GPU (256 experts split over
    the ranks, top-6, FP4 routed experts, FP8 dispatch rows with per-128
    scales, bf16 return rows), with uniform and Zipf(1.2) routing; measured
    after the headline, outside its timed region.  Per routing: the layer time
    (CUDA events, max over ranks), tokens/s, the bytes each GPU stores into
    its peers (dispatch rows to remote owners + return rows to remote
    sources) and the resulting NVLink GB/s per direction against the measured
    770 GB/s peer copy, and the routed rows per GPU (max / mean: the load
    imbalance the even expert split gives)."""
    import torch
    import torch.distributed as dist

    from spark_b200 import _lib
    from spark_b200.ep import ep_moe_forward
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    dev = torch.device("cuda", local)
    lib = _lib.load()
    T = 4096
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    out = {"tokens_per_gpu": T, "nvlink_peer_copy_gbs": 770.0}
    for routing, base in (("uniform", "decode"), ("zipf1.2", "prefill")):
        cfg = CONFIGS[base].with_tokens(T)
        layer = make_layer(cfg, seed=args.seed + 77, device=dev)
        moe = build_moe(layer, device=dev)
        del layer
        g = torch.Generator(device=dev).manual_seed(args.seed + 5000 + rank)
        x = torch.randn(T, cfg.dim, generator=g, device=dev).to(torch.bfloat16)
        exchange = "peer"
        try:
            moe.enable_peer_exchange(T)
        except RuntimeError:
            exchange = "nccl"
        for _ in range(3):
            ep_moe_forward(moe, x)
        torch.cuda.synchronize()
        _lib.raise_on_device_error()
        idx = moe.gate(x)[1].to(torch.int64).contiguous()
        every = torch.empty(world * idx.numel(), dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(every, idx.view(-1))
        graph = None
        if exchange == "peer":
            s_cap = torch.cuda.Stream(device=dev)
            s_cap.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s_cap):
                ep_moe_forward(moe, x)
            torch.cuda.current_stream().wait_stream(s_cap)
            graph.replay()
            torch.cuda.synchronize()
        times = []
        for _ in range(10):
            flush.fill_(1)
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            if graph is not None:
                graph.replay()
            else:
                ep_moe_forward(moe, x)
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        _lib.raise_on_device_error()
        t = torch.tensor([statistics.median(times)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        # traffic and load from every rank's routing (host arithmetic)
        e_per = cfg.n_routed // world
        own = (every.view(world, T, cfg.topk) // e_per).cpu()
        row_b = int(lib.dsv4_ep_row_bytes(cfg.dim, cfg.topk))
        out_b, routes = [], []
        for r in range(world):
            rows_out = sum(int((own[r] == d).any(dim=1).sum()) for d in range(world) if d != r)
            ret_out = int(((own == r).sum(dim=2)[[s for s in range(world) if s != r]]).sum())
            out_b.append(rows_out * row_b + ret_out * 2 * cfg.dim)
            routes.append(int((own == r).sum()))
        max_out = max(out_b)
        del graph
        if getattr(moe, "peer_exchange", None) is not None:
            torch.cuda.synchronize()
            dist.barrier()
            moe.peer_exchange.close()
            moe.peer_exchange = None
        del moe, x
        torch.cuda.empty_cache()
        out[routing] = {
            "ms": round(ms, 4), "tokens_per_s": round(world * T / (ms * 1e-3), 1), "exchange": exchange,
            "bytes_out_per_gpu_max": max_out, "nvlink_gbs_per_direction": round(max_out / (ms * 1e-3) / 1e9, 1),
            "nvlink_frac_of_peer_copy": round(max_out / (ms * 1e-3) / 1e9 / 770.0, 4),
            "routed_rows_per_gpu_max": max(routes), "routed_rows_per_gpu_mean": round(sum(routes) / world, 1),
            "imbalance_max_over_mean": round(max(routes) * world / max(sum(routes), 1), 3),
            "expert_tflops_per_gpu_max": round((max(routes) + T) * 6.0 * cfg.dim * cfg.inter / (ms * 1e-3) / 1e12, 1),
        }
    return out


def run_stack(args, world, rank, local):
    """Full-depth MoE-only decode stack: ``--layers`` distinct seeded layers
    (seed = layer id; H=4096, 256 experts top-6 + shared, I=2048, FP4 routed /
    FP8 shared), every expert of every layer resident in HBM (with N GPUs each
    rank holds its E/N experts per layer and the layers run expert-parallel over
    NVLink peer memory).  One step = T tokens per GPU through every layer,
    x <- x + MoE_l(rms_norm(x)) in bf16, the whole step one CUDA graph per rank."""
    import torch
    import torch.distributed as dist

    from spark_b200 import _lib
    from spark_b200.moe import packed_block_bytes
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    dev = torch.device("cuda", local)
    T = args.tokens or 8
    cfg = CONFIGS["decode"].with_tokens(T)
    H, I, E = cfg.dim, cfg.inter, cfg.n_routed
    block = packed_block_bytes(H, I)
    shared_bytes = 3 * I * H + 3 * (I // 128) * (H // 128)
    per_layer = (E // world) * (block + 3 * I * H // 32) + shared_bytes + E * H * 2
    free, _total = torch.cuda.mem_get_info(dev)
    if per_layer * args.layers * 1.03 + (4 << 30) > free:
        raise RuntimeError(f"{args.layers} layers need {per_layer * args.layers / 2**30:.0f} GiB per GPU, "
                           f"{free / 2**30:.0f} GiB free")
    lib = _lib.load()
    layers = []
    for l in range(args.layers):
        lay = make_layer(cfg, seed=l, device=dev)
        moe = build_moe(lay, device=dev, layer_id=l)
        del lay
        if world > 1:
            moe.enable_peer_exchange(T)
        layers.append(moe)
    torch.cuda.synchronize()
    g = torch.Generator(device=dev).manual_seed(args.seed + 1000 * (rank + 1))
    x0 = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    ws = torch.empty(max(layers[0].workspace_bytes(T), 1), dtype=torch.uint8, device=dev) if world == 1 else None

    def layer_out(moe, x):
        if world == 1:
            return moe.forward_tokens(x, workspace=ws)
        from spark_b200.ep import ep_moe_forward

        return ep_moe_forward(moe, x)

    def rms_norm(x):
        # the block's pre-MoE normalisation without learned weights: keeps the
        # residual stream from drifting into a few shared directions, so the
        # routing stays as diverse as a real stack's
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)

    # eager pass: the experts each layer touches (all ranks' tokens), for the bytes count
    touched = 0
    x = x0.clone()
    for moe in layers:
        h = rms_norm(x)
        idx = moe.gate(h)[1].to(torch.int64).reshape(-1)
        if world > 1:
            every = torch.empty(world * idx.numel(), dtype=torch.int64, device=dev)
            dist.all_gather_into_tensor(every, idx)
            idx = every[(every >= moe.experts_start_idx) & (every < moe.experts_end_idx)]
        touched += int(torch.unique(idx).numel())
        x = x + layer_out(moe, h)
    torch.cuda.synchronize()
    _lib.raise_on_device_error()

    xs = x0.clone()

    def step():
        xs.copy_(x0)
        for moe in layers:
            xs.add_(layer_out(moe, rms_norm(xs)))

    for _ in range(max(args.warmup, 2)):
        step()
    torch.cuda.synchronize()
    s_cap = torch.cuda.Stream(device=dev)
    s_cap.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    n0 = lib.dsv4_kernel_launches()
    with torch.cuda.graph(graph, stream=s_cap):
        step()
    launches_per_step = lib.dsv4_kernel_launches() - n0
    torch.cuda.current_stream().wait_stream(s_cap)
    graph.replay()
    torch.cuda.synchronize()
    _lib.raise_on_device_error()

    times = []
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    for _ in range(args.steps):
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    clk = clocks.stop()
    _lib.raise_on_device_error()
    ms = sum(times) / len(times)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    peaks, peak_src = _peaks()
    bytes_step = touched * block + args.layers * (shared_bytes + E * H * 2 + 4 * T * H)
    achieved = bytes_step / (ms * 1e-3) / 1e9
    del graph
    for moe in layers:
        if getattr(moe, "peer_exchange", None) is not None:
            torch.cuda.synchronize()
            dist.barrier()
            moe.peer_exchange.close()
            moe.peer_exchange = None
    result = {
        "metric": METRIC, "value": round(world * T / (ms * 1e-3), 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e2m1/e4m3 x e4m3 -> f32 (bf16 out)",
        "data": "synthetic (seeded per layer; random-init weights of the V4-Flash MoE shapes)",
        "config": {"workload": f"moe_stack_{args.layers}_layers_decode", "tokens_per_gpu": T, "hidden": H,
                   "inter": I, "routed_experts": E, "topk": cfg.topk, "shared_experts": 1,
                   "layers": args.layers, "experts_resident_per_gpu": args.layers * (E // world),
                   "rank0_experts_touched_per_step": touched, "residual": "bf16, x += MoE_l(rms_norm(x)) (weight-free pre-norm)",
                   "l2": f"not flushed: a step streams {bytes_step / 1e9:.1f} GB, far above the 126 MB L2",
                   "parallelism": "single" if world == 1 else f"ep{world} over NVLink peer memory",
                   "cuda_graph": True},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "kernel": "whole step (rank 0): touched experts + shared + gate bytes of every layer",
                     "algorithmic_bytes": bytes_step, "peak_source": peak_src},
        "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
    }
    return result


def _sweep(args, local):
    """Other decode batch sizes and the prefill layer, short runs."""
    import torch

    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    out = {}
    dev = torch.device("cuda", local)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for wl, T in (("decode", 1), ("decode", 8), ("decode", 32), ("prefill", 8192)):
        if wl == "decode" and T == (args.tokens or 64) and args.workload == "decode":
            continue
        cfg = CONFIGS[wl].with_tokens(T)
        layer = make_layer(cfg, seed=args.seed + 7, device=dev)
        moe = build_moe(layer, device=dev)
        ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=dev)
        y = torch.empty_like(layer["x"])
        for _ in range(3):
            moe.forward_tokens(layer["x"], workspace=ws, out=y)
        torch.cuda.synchronize()
        # the layer as a replayed CUDA graph, as the headline times it (eager
        # calls at these sizes would time the host's launch path instead)
        s_cap = torch.cuda.Stream(device=dev)
        s_cap.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s_cap):
            moe.forward_tokens(layer["x"], workspace=ws, out=y)
        torch.cuda.current_stream().wait_stream(s_cap)
        ts = []
        for _ in range(10):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = statistics.median(ts)
        del graph
        entry = {"ms": round(ms, 4), "tokens_per_s": round(T / (ms * 1e-3), 1), "cuda_graph": True}
        if wl == "prefill":
            entry["roofline"] = _prefill_roofline(moe, layer, ws, y, flush, cfg, T)
        else:
            entry.update(_decode_roofline(moe, layer, ws, y, flush, cfg, T, ms))
        out[f"{wl}_T{T}"] = entry
        del moe, layer, ws, y
        torch.cuda.empty_cache()
    out["prefill_T8192_fp4act"] = _prefill_fp4(args, dev, flush)
    out.update(_materializer(args, dev, flush))
    out["upload_32_experts"] = _upload_rate(args, dev)
    out["attention"] = _attention(args, dev, flush)
    return out


def _upload_rate(args, dev):
    """The slab upload path (packed_store.upload_experts): 32 packed expert
    blocks of the decode shapes (428 MB) written in the reference's layout to a
    temporary directory, then pread in chunks of 8 into reused pinned staging,
    copied to the device on a copy stream and materialized into a 32-slot arena,
    the three stages overlapped.  The file was just written, so it is read
    from the page cache: the figure is the host-memory -> HBM pipeline, not a
    disk.  Beside it, one plain pinned -> device copy of the same bytes (the
    PCIe ceiling of this host)."""
    import tempfile

    import torch

    from spark_b200.moe import ExpertArena
    from spark_b200.packed_store import PackedExpertStore, write_packed_layout
    from spark_b200.synthetic import routed_blocks

    H, I, n = 4096, 2048, 32
    blocks = routed_blocks(n, H, I, args.seed + 17)
    with tempfile.TemporaryDirectory() as tmp:
        write_packed_layout(Path(tmp), {0: {e: blocks[e].numpy() for e in range(n)}}, H, I)
        store = PackedExpertStore(Path(tmp) / "layout.json")
        arena = ExpertArena(n, H, I, device=dev)
        store.upload_experts(0, list(range(n)), arena, list(range(n)))  # warm: staging, rings, page cache
        runs = [store.upload_experts(0, list(range(n)), arena, list(range(n))) for _ in range(3)]
        store.close()
    best = max(runs, key=lambda r: r["upload_gbs"])
    host = blocks.reshape(-1).pin_memory()
    devbuf = torch.empty_like(host, device=dev)
    ts = []
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        devbuf.copy_(host, non_blocking=True)
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    h2d = host.numel() / (min(ts) * 1e-3) / 1e9
    del arena, devbuf
    torch.cuda.empty_cache()
    return {"bytes": int(best["packed_read_bytes"]), "upload_gbs": round(best["upload_gbs"], 2),
            "pread_seconds": round(best["packed_read_seconds"], 4), "wall_seconds": round(best["upload_seconds"], 4),
            "plain_pinned_h2d_gbs": round(h2d, 2), "frac_of_h2d": round(best["upload_gbs"] / h2d, 3),
            "source": "page-cache resident file, chunks of 8 experts"}


def _decode_roofline(moe, layer, ws, y, flush, cfg, T, layer_ms):
    """HBM roofline of a decode layer: the algorithmic bytes (touched experts'
    blocks + shared expert + gate + activations) over the graph-replayed layer
    time, and the expert GEMMs' weight bytes over their stage-event time."""
    import torch

    from spark_b200 import _lib
    from spark_b200.synthetic import algorithmic_decode_bytes

    lib = _lib.load()
    offs = (ctypes.c_longlong * 20)()
    d = moe.layer_desc()
    lib.dsv4_moe_workspace_layout(ctypes.byref(d), T, offs, 20)
    counts = ws[offs[3]:offs[3] + (cfg.n_routed + 1) * 4].view(torch.int32)[: cfg.n_routed]
    touched = int((counts > 0).sum())
    alg = algorithmic_decode_bytes(cfg, touched, T)
    gemm_bytes = alg - cfg.n_routed * cfg.dim * 2 - cfg.n_routed * 4 - 4 * T * cfg.dim
    lib.dsv4_profile_enable(1)
    buf = (ctypes.c_float * 6)()
    gemm = []
    for _ in range(5):
        flush.fill_(1)
        moe.forward_tokens(layer["x"], workspace=ws, out=y)
        torch.cuda.synchronize()
        lib.dsv4_profile_read(buf, 6)
        gemm.append(buf[3] + buf[4])
    lib.dsv4_profile_enable(0)
    gemm_ms = statistics.median(gemm)
    hbm = _peaks()[0]["hbm_gbs"]
    return {"experts_touched": touched, "split_k": [int(offs[18]), int(offs[19])],
            "layer_frac_of_measured_hbm": round(alg / (layer_ms * 1e-3) / 1e9 / hbm, 4),
            "gemm_ms": round(gemm_ms, 4),
            "gemm_frac_of_measured_hbm": round(gemm_bytes / (gemm_ms * 1e-3) / 1e9 / hbm, 4)}


def _prefill_roofline(moe, layer, ws, y, flush, cfg, T):
    """Tensor roofline of the prefill layer's expert GEMMs: their algorithmic
    FLOPs (T*(k+1)*3*2*H*I) over the GEMM1 + GEMM2 time taken by the library's
    stage events on the launching stream (median of 5, L2 flushed between),
    against the dense FP8 rate (what kind::mxf8f6f4 with e4m3 activations
    runs at) and the dense FP4 rate, both scaled from the measured bf16 peak
    by the nominal dense ratios (FP8 = 2x, FP4 = 4x bf16)."""
    import torch

    from spark_b200 import _lib
    from spark_b200.synthetic import algorithmic_flops

    lib = _lib.load()
    lib.dsv4_profile_enable(1)
    buf = (ctypes.c_float * 6)()
    gemm = []
    for _ in range(5):
        flush.fill_(1)
        moe.forward_tokens(layer["x"], workspace=ws, out=y)
        torch.cuda.synchronize()
        lib.dsv4_profile_read(buf, 6)
        gemm.append(buf[3] + buf[4])
    lib.dsv4_profile_enable(0)
    gemm_ms = statistics.median(gemm)
    flops = algorithmic_flops(cfg, T) - 2.0 * T * cfg.dim * cfg.n_routed
    achieved = flops / (gemm_ms * 1e-3) / 1e12
    peaks, src = _peaks()
    bf16 = peaks.get("bf16_tflops", 1590.0)
    return {"bound": "tensor", "achieved": round(achieved, 1), "unit": "TFLOP/s", "algorithmic_flops": flops,
            "kernel_ms": round(gemm_ms, 4), "peak_fp8": round(2 * bf16, 1), "frac_fp8": round(achieved / (2 * bf16), 4),
            "peak_fp4": round(4 * bf16, 1), "frac_fp4": round(achieved / (4 * bf16), 4),
            "kernel": "expert_gemm_kernel (GEMM1 + GEMM2), kind::mxf8f6f4 (e4m3 x e2m1, FP8 rate)",
            "peak_source": f"{src} bf16 x2 (FP8) / x4 (FP4), nominal dense ratios"}


def _prefill_fp4(args, dev, flush, T=8192, sample=16):
    """The prefill layer in the opt-in FP4-activation mode
    (dsv4_set_fp4_activations): the routed experts' w1 | w3 and w2 as
    kind::mxf4 products on FP4 activations (x and h quantized per 32), the
    shared expert as in the default layer.  Time: the graph-replayed layer
    (median of 10, L2 flushed between), and the expert GEMMs' stage time
    against their mixed roofline (routed FLOPs at the FP4 rate, the shared
    expert's at the FP8 rate, both scaled from the measured bf16 peak).  Outside the timings: the first
    `sample` tokens against the oracle run in the same mode (the bar) and
    against the default e4m3 oracle (how far the mode moves the layer)."""
    import numpy as np
    import torch

    from oracle import moe_oracle as O
    from spark_b200 import _lib
    from spark_b200.synthetic import CONFIGS, build_moe, make_layer

    lib = _lib.load()
    _lib.check(lib.dsv4_set_fp4_activations(1), "dsv4_set_fp4_activations")
    try:
        cfg = CONFIGS["prefill"].with_tokens(T)
        layer = make_layer(cfg, seed=args.seed + 7, device=dev)
        moe = build_moe(layer, device=dev)
        d = moe.layer_desc()
        offs = (ctypes.c_longlong * 21)()
        _lib.check(lib.dsv4_moe_workspace_layout(ctypes.byref(d), T, offs, 21), "dsv4_moe_workspace_layout")
        if offs[20] != 1:
            return {"error": "the FP4-activation mode is not in force for this layout"}
        ws = torch.empty(moe.workspace_bytes(T), dtype=torch.uint8, device=dev)
        y = torch.empty_like(layer["x"])
        ms = _graph_ms(lambda: moe.forward_tokens(layer["x"], workspace=ws, out=y), flush)
        # stage times of the expert GEMMs (library events on the launching stream)
        lib.dsv4_profile_enable(1)
        buf = (ctypes.c_float * 6)()
        gemm = []
        for _ in range(5):
            flush.fill_(1)
            moe.forward_tokens(layer["x"], workspace=ws, out=y)
            torch.cuda.synchronize()
            lib.dsv4_profile_read(buf, 6)
            gemm.append(buf[3] + buf[4])
        lib.dsv4_profile_enable(0)
        gemm_ms = statistics.median(gemm)
        _lib.raise_on_device_error()
        k, H, I = cfg.topk, cfg.dim, cfg.inter
        w_dev = ws[offs[1]:offs[1] + T * k * 4].view(torch.float32).view(T, k)
        i_dev = ws[offs[2]:offs[2] + T * k * 8].view(torch.int64).view(T, k)
        routes = int((i_dev >= 0).sum())
        f_fp4 = 2.0 * routes * 3 * H * I               # routed w1 | w3 and w2
        f_fp8 = 2.0 * T * 3 * H * I                    # the shared expert
        peaks, src = _peaks()
        bf16 = peaks.get("bf16_tflops", 1590.0)
        ideal_ms = (f_fp4 / (4 * bf16 * 1e12) + f_fp8 / (2 * bf16 * 1e12)) * 1e3
        # parity on sampled tokens, outside the timings
        xs, ys = layer["x"][:sample], y[:sample]
        ws_, is_ = w_dev[:sample].cpu().numpy(), i_dev[:sample].cpu().numpy()
        experts = sorted(set(int(e) for e in is_.reshape(-1).tolist()))
        mw = O.MoEWeights(
            gate_w=None, gate_bias=None,
            experts={e: O.expert_from_block(layer["blocks"][e].cpu().numpy(), H, I) for e in experts},
            shared=O.shared_from_tensors({kk: v.cpu().numpy() for kk, v in layer["shared"].items()}),
            topk=k, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)
        xn, yn = xs.float().cpu().numpy(), ys.float().cpu().numpy().astype(np.float64)
        workers = min(16, os.cpu_count() or 1)
        r4 = O.moe_forward(xn, mw, routing=(ws_, is_), workers=workers, fp4_act=True)[0].astype(np.float64)
        r8 = O.moe_forward(xn, mw, routing=(ws_, is_), workers=workers)[0].astype(np.float64)

        def rel(a, b, rms=False):
            den = np.sqrt(np.mean(b ** 2)) + 1e-30
            return float((np.sqrt(np.mean((a - b) ** 2)) if rms else np.max(np.abs(a - b))) / den)

        return {
            "tokens": T, "ms": round(ms, 4), "tokens_per_s": round(T / (ms * 1e-3), 1), "cuda_graph": True,
            "gemm_ms": round(gemm_ms, 4),
            "roofline": {"bound": "tensor", "algorithmic_flops_fp4": f_fp4, "algorithmic_flops_fp8": f_fp8,
                         "achieved": round((f_fp4 + f_fp8) / (gemm_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                         "ideal_ms": round(ideal_ms, 4), "frac": round(ideal_ms / gemm_ms, 4),
                         "peak_source": f"{src} bf16 {bf16} x4 (FP4) / x2 (FP8), nominal dense ratios"},
            "parity": {"checked_tokens": sample, "max_err_vs_fp4_oracle": round(rel(yn, r4), 6), "tol": 2e-2,
                       "ok": bool(rel(yn, r4) <= 2e-2),
                       "deviation_from_e4m3_layer": {"max_of_rms": round(rel(yn, r8), 4),
                                                     "rms_of_rms": round(rel(yn, r8, rms=True), 4)}},
            "numerics": "routed experts on fp4_act_quant(., 32) activations (x before w1 | w3, h before w2; e2m1, "
                        "per-32 ue8m0); the reference's layer uses act_quant(., 128) e4m3"}
    finally:
        _lib.check(lib.dsv4_set_fp4_activations(0), "dsv4_set_fp4_activations")
        torch.cuda.empty_cache()


def _materializer(args, dev, flush):
    """The packed-slab materializer on one layer: 256 packed expert blocks (a
    slab already in HBM) -> a 256-slot FP4 arena plus scale atoms, and the same
    with the exact bf16 decode of every weight.  HBM roofline: the block is
    read once, the slot, atoms (and bf16 weights) written once."""
    import torch

    from spark_b200 import _lib
    from spark_b200.moe import ExpertArena, packed_block_bytes
    from spark_b200.synthetic import routed_blocks

    lib = _lib.load()
    H, I, n = 4096, 2048, 256
    nb = packed_block_bytes(H, I)
    slab = routed_blocks(n, H, I, args.seed + 9, dev).reshape(-1)
    arena = ExpertArena(n, H, I, device=dev)
    off = torch.arange(n, dtype=torch.int64, device=dev) * nb
    slots = torch.arange(n, dtype=torch.int32, device=dev)
    bf16_stride = 3 * I * H
    bf16 = torch.empty(n * bf16_stride, dtype=torch.bfloat16, device=dev)
    peak = _peaks()[0]["hbm_gbs"]
    out = {}
    for name, dst in (("materialize_fp4_arena_256", None), ("materialize_fp4_and_bf16_256", bf16)):
        def run():
            _lib.check(lib.dsv4_materialize(_lib.ptr(slab), _lib.ptr(off), _lib.ptr(slots), n, H, I,
                                            _lib.ptr(arena.buffer), arena.slot_stride, _lib.ptr(arena.sf),
                                            arena.sf_stride, _lib.ptr(dst), bf16_stride if dst is not None else 0,
                                            _lib.stream_ptr()), "dsv4_materialize")
        for _ in range(2):
            run()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = statistics.median(ts)
        nbytes = n * (2 * nb + arena.sf_stride) + (n * bf16_stride * 2 if dst is not None else 0)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "bytes": nbytes, "GB_per_s": round(gbs, 1),
                     "frac_of_measured_hbm": round(gbs / peak, 4)}
    _lib.raise_on_device_error()
    del slab, arena, bf16
    torch.cuda.empty_cache()
    return out


def _graph_ms(fn, flush, reps=10):
    """Median CUDA-event time of fn replayed as a CUDA graph, L2 flushed
    before each replay (outside the events)."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s_cap = torch.cuda.Stream()
    s_cap.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s_cap):
        fn()
    torch.cuda.current_stream().wait_stream(s_cap)
    ts = []
    for _ in range(reps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    del graph
    return statistics.median(ts)


def _attention(args, dev, flush):
    """The attention block's hot ops (h=64 heads, d=512): sparse attention at
    decode and prefill shapes and the FP8 linear at the projection shapes,
    each as a replayed CUDA graph with L2 flushed between replays.  Sparse
    attention's algorithmic work is 4*B*S*64*512*K FLOPs (the score and the
    output product over the K gathered rows), bounded by the measured bf16
    tensor peak; its gathered bytes (K rows of 1 KB per query) are given
    beside.  FP8 linear: decode M=64 is bound by the weight bytes (HBM),
    prefill M=8192 by the FP8 rate (2x the measured bf16 peak).  A small case
    of each is checked against the oracle first (outside the timings)."""
    import numpy as np
    import torch

    from oracle import attention_oracle as A
    from spark_b200 import _lib
    from spark_b200.attention import FP8Linear, sparse_attn

    peaks, src = _peaks()
    bf16_peak, hbm = peaks.get("bf16_tflops", 1590.0), peaks.get("hbm_gbs", 6650.0)
    g = torch.Generator(device=dev).manual_seed(args.seed + 23)
    out = {}

    # parity, small cases
    gc = torch.Generator().manual_seed(args.seed + 29)
    q = torch.randn(1, 3, 64, 512, generator=gc).to(torch.bfloat16)
    kv = torch.randn(1, 700, 512, generator=gc).to(torch.bfloat16)
    sink = torch.randn(64, generator=gc)
    idx = torch.stack([torch.randperm(700, generator=gc)[:300] for _ in range(3)])[None].to(torch.int32)
    got = sparse_attn(q.to(dev), kv.to(dev), sink.to(dev), idx.to(dev), 0.044).float().cpu().numpy()
    ref = A.sparse_attn(q.float().numpy(), kv.float().numpy(), sink.numpy(), idx.numpy(), 0.044)
    rms = float(np.sqrt(np.mean((got - ref) ** 2)) / np.sqrt(np.mean(ref ** 2)))
    lin = FP8Linear(1024, 512, device=dev)
    lin.weight.data.view(torch.uint8).copy_(torch.randint(0, 126, (512, 1024), generator=gc, dtype=torch.uint8))
    lin.scale.data.view(torch.uint8).copy_(torch.randint(120, 130, (4, 8), generator=gc, dtype=torch.uint8))
    lin.refresh_scale_atoms()
    xl = torch.randn(8, 1024, generator=gc).to(torch.bfloat16)
    yl = lin(xl.to(dev)).float().cpu().numpy()
    refl = A.fp8_linear(xl.float().numpy(), lin.weight.view(torch.uint8).cpu().numpy(),
                        lin.scale.view(torch.uint8).cpu().numpy())
    out["parity"] = {"sparse_attn_rms_err": round(rms, 6),
                     "fp8_linear_max_err_rms": round(float(np.max(np.abs(yl - refl)) / np.sqrt(np.mean(refl ** 2))), 6),
                     "oracle": "oracle/attention_oracle.py (the reference's sparse_attn_fallback, float64)"}

    # the profiled small prefill case runs first
    for name, (B, S, N, K) in (("prefill_S512_K512", (1, 512, 4096, 512)),
                               ("decode_B1_K2048", (1, 1, 65536, 2048)),
                               ("decode_B8_K2048", (8, 1, 65536, 2048)),
                               ("prefill_S2048_K2048", (1, 2048, 8192, 2048))):
        q = torch.randn(B, S, 64, 512, device=dev, generator=g).to(torch.bfloat16)
        kv = torch.randn(B, N, 512, device=dev, generator=g).to(torch.bfloat16)
        sink = torch.randn(64, device=dev, generator=g)
        idx = torch.randint(0, N, (B, S, K), device=dev, dtype=torch.int32, generator=g)
        ms = _graph_ms(lambda: sparse_attn(q, kv, sink, idx, 0.044), flush)
        flops = 4.0 * B * S * 64 * 512 * K
        tf = flops / (ms * 1e-3) / 1e12
        out[f"sparse_attn_{name}"] = {
            "B": B, "S": S, "N": N, "K": K, "ms": round(ms, 4), "achieved_tflops": round(tf, 1),
            "frac_bf16": round(tf / bf16_peak, 4), "gathered_gb_per_s": round(B * S * K * 1024 / (ms * 1e-3) / 1e9, 1)}
        del q, kv, sink, idx
    for name, (M, K, N) in (("decode_M64_K4096_N1024", (64, 4096, 1024)),
                            ("decode_M64_K1024_N32768", (64, 1024, 32768)),
                            ("prefill_M8192_K1024_N32768", (8192, 1024, 32768))):
        lin = FP8Linear(K, N, device=dev)
        lin.weight.data.view(torch.uint8).copy_(torch.randint(0, 126, (N, K), device=dev, generator=g,
                                                              dtype=torch.uint8))
        lin.refresh_scale_atoms()
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        ms = _graph_ms(lambda: lin(x), flush)
        nbytes = N * K + (N // 128) * (K // 128) + 2 * M * K + 2 * M * N
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        entry = {"M": M, "K": K, "N": N, "ms": round(ms, 4), "achieved_tflops": round(tf, 1),
                 "GB_per_s": round(nbytes / (ms * 1e-3) / 1e9, 1)}
        if M <= 64:
            entry["frac_hbm"] = round(entry["GB_per_s"] / hbm, 4)
        else:
            entry["frac_fp8"] = round(tf / (2 * bf16_peak), 4)
        out[f"fp8_linear_{name}"] = entry
        del lin, x
    _lib.raise_on_device_error()
    out["peak_source"] = f"{src}: bf16 {bf16_peak} TFLOP/s (FP8 = 2x), HBM {hbm} GB/s"
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# CPU arm: the oracle restatement of the reference's layer on the host cores
# ---------------------------------------------------------------------------
def cpu_layer_rate(cfg_name: str, sample_tokens: int, seed: int, threads: int | None = None):
    """tokens/s of the oracle layer (numpy, fp32/fp64 over the e2m1/e4m3 codes)
    on a bounded sample of tokens.  Only the experts the sample touches are
    generated (outside the timed region); the timed region is gate + experts +
    combine, including the per-step decode of the FP4/FP8 weights."""
    import numpy as np
    import torch

    from oracle import moe_oracle as O
    from spark_b200.synthetic import CONFIGS, routed_blocks, shared_expert

    if threads:
        torch.set_num_threads(threads)
    cfg = CONFIGS[cfg_name].with_tokens(sample_tokens)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(sample_tokens, cfg.dim, generator=g).to(torch.bfloat16).float().numpy()
    gw = (torch.randn(cfg.n_routed, cfg.dim, generator=g) * cfg.gate_std).to(torch.bfloat16).float().numpy()
    bias = np.zeros(cfg.n_routed, np.float32)
    logits = O.gate_logits(x, gw)
    _, idx0 = O.route_from_logits(logits, bias, cfg.topk, cfg.route_scale)
    blocks = {int(e): routed_blocks(1, cfg.dim, cfg.inter, seed * 1000 + int(e))[0].numpy() for e in np.unique(idx0)}
    sh_t = {k: v.numpy() for k, v in shared_expert(cfg.dim, cfg.inter, seed + 31).items()}
    t0 = time.perf_counter()
    wts, idx, _ = O.gate_forward(x, gw, bias, cfg.topk, cfg.route_scale)
    experts = {e: O.expert_from_block(b, cfg.dim, cfg.inter) for e, b in blocks.items()}
    mw = O.MoEWeights(gate_w=gw, gate_bias=bias, experts=experts, shared=O.shared_from_tensors(sh_t),
                      topk=cfg.topk, route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit)
    O.moe_forward(x, mw, routing=(wts, idx))
    dt = time.perf_counter() - t0
    return sample_tokens / dt, dt


def run_reference(args, world, rank):
    if rank != 0:
        return None
    if args.workload == "stack":  # the oracle's per-layer rate already bounds it: layers x one layer
        return {"impl": "reference", "unavailable": "the full-depth stack has no CPU arm of its own; "
                "the per-layer CPU rate is the decode workload's reference line"}
    if args.workload == "attention":
        return {"impl": "reference", "unavailable": "the reference's attention fallback is a per-token Python loop; "
                "its restatement is the parity oracle of the attention block, not a timed arm"}
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    T = args.tokens or (64 if args.workload == "decode" else 8192)
    try:
        v, info = reference_layer_rate(args, T, args.steps, args.warmup)
        kind = "reference"
        sample = (f"the full {T}-token {args.workload} batch per step through the reference's LazyMoE.forward "
                  f"(packed store + native loader; official Gate/Expert stood in by the oracle's CPU classes), "
                  f"{info['timed_steps']} timed steps")
        dtype = "bf16 x bf16 -> f32 (torch CPU GEMM) over exactly decoded e2m1/e4m3 weights"
    except Exception as exc:  # the reference is not installed: the oracle port instead
        sample_t = 1 if args.workload == "decode" else 8
        rates = []
        for i in range(args.warmup + args.steps):
            r, _ = cpu_layer_rate(args.workload, sample_t, args.seed + i, threads)
            if i >= args.warmup:
                rates.append(r)
        v, kind, info = statistics.median(rates), "port", {"reference_unavailable": repr(exc)[:200]}
        sample = f"{sample_t} tokens of the {args.workload} layer per step (oracle restatement)"
        dtype = "f32 (numpy) over e2m1/e4m3 codes"
    return {
        "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(T / v * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "impl": "reference", "dtype": dtype,
        "data": "synthetic", "config": {"workload": f"{args.workload}_moe_layer", "tokens_per_gpu": T,
                                        "same_config": kind == "reference"},
        "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": kind, "sample": sample,
                         **info},
        "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_layer_rate(args, T, steps, warmup, budget_s=150.0):
    """The reference's own LazyMoE.forward on the host cores at T tokens (see
    oracle/reference_runtime.py): every step is the full T-token batch; the
    warm-up steps materialize the touched experts through the reference's
    packed store and compiled loader.  Steps past ``budget_s`` seconds of timed
    host work are not run (the line says how many were).  Returns (tokens/s,
    details)."""
    from oracle import reference_runtime as R
    from spark_b200.synthetic import CONFIGS, make_layer

    cfg = CONFIGS[args.workload].with_tokens(T)
    layer = make_layer(cfg, seed=args.seed, device="cpu")
    ref = R.ReferenceLayer(layer)
    try:
        err = R.layer_matches_oracle(ref, layer, tokens=2)
        x = layer["x"]
        t_warm = [ref.timed_step(x) for _ in range(max(warmup, 1))]
        times = []
        while len(times) < max(steps, 1) and sum(times) < budget_s:
            times.append(ref.timed_step(x))
        snap = ref.cache.snapshot()
        loader = ref.loader_kind
    finally:
        ref.close()
    return T / statistics.median(times), {"timed_steps": len(times), "first_step_s": round(t_warm[0], 2),
                                          "err_vs_oracle_rms": round(err, 6),
                                          "experts_resident": snap.get("entries"), "loader": loader}


def main():
    args = _parse()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        res = run_reference(args, world, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    world, rank, local = _dist_init(args.gpus)
    if args.workload == "attention":
        # the attention block's ops alone (one GPU; the other ranks idle)
        if rank == 0:
            import torch

            dev = torch.device("cuda", local)
            flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
            print(json.dumps({"workload": "attention", **_attention(args, dev, flush)}), flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
        return
    if args.workload == "stack":
        res = run_stack(args, world, rank, local)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
        return
    res, cfg, layer, moe = run_ours(args, world, rank, local)
    del moe, layer
    if rank == 0 and world == 1:
        if not args.no_sweep:
            try:
                res["sweep"] = _sweep(args, local)
            except Exception as exc:  # keep the headline line even if a sweep case fails
                res["sweep"] = {"error": repr(exc)}
        if not args.no_cpu_baseline:
            import torch

            torch.set_num_threads(os.cpu_count() or 1)
            T = args.tokens or (64 if args.workload == "decode" else 8192)
            try:  # the reference's own LazyMoE on the host, same config, a few steps
                rate, info = reference_layer_rate(args, T, 5, 1, budget_s=20.0)
                res["cpu_baseline"] = {"value": round(rate, 3), "unit": UNIT, "cores": os.cpu_count(),
                                       "kind": "reference",
                                       "sample": f"the full {T}-token batch per step through the reference's "
                                                 "LazyMoE.forward (official Gate/Expert stood in by the oracle's "
                                                 "CPU classes)", **info}
            except Exception as exc:
                n = 12
                rate, dt = cpu_layer_rate(args.workload, n, args.seed, os.cpu_count())
                res["cpu_baseline"] = {"value": round(rate, 3), "unit": UNIT, "cores": os.cpu_count(),
                                       "kind": "port", "reference_unavailable": repr(exc)[:200],
                                       "sample": f"{n} tokens of the {args.workload} layer, {dt:.1f} s "
                                                 "(oracle restatement, numpy)"}
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
