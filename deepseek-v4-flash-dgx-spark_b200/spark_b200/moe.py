"""B200 MoE layer with the official DeepSeek module interface.

Drop-in for the modules the reference builds its MoE from:

* ``MoE(layer_id, args)`` / ``forward(x, input_ids)`` - the class the reference
  patches in as ``official_model.MoE`` (``BoundLazyMoE``,
  spark_runtime/lazy_official_runtime.py:946-1002,1052-1061);
* ``Gate(layer_id, args)`` / ``forward(x, input_ids) -> (weights, indices)``
  (official Gate, called at :966,983);
* ``Expert(dim, inter_dim, dtype=, swiglu_limit=)`` / ``forward(x, weights)``
  (official Expert, constructed at :769-774 and :976-978);
* ``ExpertArena(max_slots).acquire(factory) -> (expert, reused)`` /
  ``release(expert) -> bool`` (:641-667).

Submodule and parameter names follow the official state dict
(``gate.weight``, ``gate.bias``, ``experts.{i}.w1.weight``, ``.scale``, ...,
``shared_experts.w1.weight``), so checkpoint names still resolve.  All compute
goes through libdsv4moe.so; nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import nn

from contextlib import nullcontext as _nullcontext

from . import _lib, ops
from ._lib import MoELayerDesc, ptr

FP4 = torch.float4_e2m1fn_x2
E8M0 = torch.float8_e8m0fnu
E4M3 = torch.float8_e4m3fn


@dataclass
class ModelArgs:
    """The ``ModelArgs`` fields the MoE path reads (lazy_official_runtime.py:959-978,767-774)."""

    dim: int = 4096
    moe_inter_dim: int = 2048
    n_routed_experts: int = 256
    n_activated_experts: int = 6
    n_shared_experts: int = 1
    expert_dtype: str = "fp4"
    swiglu_limit: float = 10.0
    route_scale: float = 2.5
    score_func: str = "sigmoid"
    gate_dtype: torch.dtype = torch.bfloat16
    gate_bias: bool = True
    n_hash_layers: int = 0          # layers [0, n_hash_layers) route by gate.tid2eid[input_ids]
    vocab_size: int = 129280


# ---------------------------------------------------------------------------
# packed expert block (scripts/build_packed_expert_layout.py:76-86)
# ---------------------------------------------------------------------------
# MoE.forward replays a captured CUDA graph per token count up to this many
# tokens (decode batches); DSV4_CUDA_GRAPHS=0 keeps every call eager.
GRAPH_MAX_TOKENS = 1024
GRAPH_MAX_ENTRIES = 8
_GRAPHS_ON = os.environ.get("DSV4_CUDA_GRAPHS", "1") != "0"

PACKED_ORDER = ("w1.scale", "w2.scale", "w3.scale", "w1.weight", "w2.weight", "w3.weight")


def packed_block_layout(dim: int, inter: int) -> dict[str, tuple[int, int, torch.dtype, tuple[int, int]]]:
    """name -> (offset, bytes, dtype, shape) of the six routed-expert tensors in
    one packed block, in the slab's tensor order."""
    shapes = {
        "w1.scale": ((inter, dim // 32), E8M0),
        "w2.scale": ((dim, inter // 32), E8M0),
        "w3.scale": ((inter, dim // 32), E8M0),
        "w1.weight": ((inter, dim // 2), FP4),
        "w2.weight": ((dim, inter // 2), FP4),
        "w3.weight": ((inter, dim // 2), FP4),
    }
    out, off = {}, 0
    for name in PACKED_ORDER:
        shape, dtype = shapes[name]
        n = shape[0] * shape[1]
        out[name] = (off, n, dtype, shape)
        off += n
    return out


def packed_block_bytes(dim: int, inter: int) -> int:
    return 3 * inter * dim // 32 + 3 * inter * dim // 2


def scale_atom_bytes(dim: int, inter: int) -> int:
    return 3 * inter * dim // 32


class _QLinear(nn.Module):
    """Holder of one quantized projection: ``weight`` and ``scale`` parameters."""

    def __init__(self, weight: torch.Tensor, scale: torch.Tensor):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.scale = nn.Parameter(scale, requires_grad=False)


# ---------------------------------------------------------------------------
# Expert
# ---------------------------------------------------------------------------
class Expert(nn.Module):
    """Official ``Expert(dim, inter_dim, dtype=None|float4_e2m1fn_x2, swiglu_limit=)``.

    Routed (fp4): the six tensors are views into one packed block (its own
    buffer, or an arena slot passed as ``storage``), so a materialized block's
    bytes are the parameters.  Shared (dtype None): fp8 e4m3 weights with
    128x128 ue8m0 block scales.  ``scale_atoms`` holds the tensor-memory scale
    layout the kernels read; call ``refresh_scale_atoms()`` after writing the
    parameters (``load_state_dict`` does it automatically)."""

    def __init__(self, dim: int, inter_dim: int, dtype=None, swiglu_limit: float = 0.0, *,
                 storage: torch.Tensor | None = None, scale_atoms: torch.Tensor | None = None,
                 device=None):
        super().__init__()
        self.dim, self.inter_dim = dim, inter_dim
        self.swiglu_limit = float(swiglu_limit or 0.0)
        self.fp4 = dtype == FP4
        device = torch.device(device) if device is not None else (
            storage.device if storage is not None else torch.device("cuda"))
        if self.fp4:
            nbytes = packed_block_bytes(dim, inter_dim)
            if storage is None:
                storage = torch.zeros(_round_up(nbytes, 256), dtype=torch.uint8, device=device)
            if storage.numel() < nbytes or storage.dtype != torch.uint8:
                raise RuntimeError("expert storage is smaller than one packed block")
            self.register_buffer("block", storage, persistent=False)
            lay = packed_block_layout(dim, inter_dim)
            views = {}
            for name, (off, n, dt, shape) in lay.items():
                views[name] = storage[off:off + n].view(dt).view(*shape)
            self.w1 = _QLinear(views["w1.weight"], views["w1.scale"])
            self.w2 = _QLinear(views["w2.weight"], views["w2.scale"])
            self.w3 = _QLinear(views["w3.weight"], views["w3.scale"])
        else:
            self.register_buffer("block", None, persistent=False)
            self.w1 = _QLinear(torch.zeros(inter_dim, dim, dtype=torch.uint8, device=device).view(E4M3),
                               torch.full((inter_dim // 128, dim // 128), 127, dtype=torch.uint8,
                                          device=device).view(E8M0))
            self.w2 = _QLinear(torch.zeros(dim, inter_dim, dtype=torch.uint8, device=device).view(E4M3),
                               torch.full((dim // 128, inter_dim // 128), 127, dtype=torch.uint8,
                                          device=device).view(E8M0))
            self.w3 = _QLinear(torch.zeros(inter_dim, dim, dtype=torch.uint8, device=device).view(E4M3),
                               torch.full((inter_dim // 128, dim // 128), 127, dtype=torch.uint8,
                                          device=device).view(E8M0))
        if scale_atoms is None:
            scale_atoms = torch.zeros(scale_atom_bytes(dim, inter_dim), dtype=torch.uint8, device=device)
        self.register_buffer("scale_atoms", scale_atoms, persistent=False)
        self.register_buffer("_slot0", torch.zeros(1, dtype=torch.int32, device=device), persistent=False)
        self.register_load_state_dict_post_hook(lambda m, _keys: m.refresh_scale_atoms())

    def refresh_scale_atoms(self, stream=None) -> None:
        dsv4 = ops.load()
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            if self.fp4:
                dsv4.build_scale_atoms(self.block, self.block.numel(), self._slot0, self.dim, self.inter_dim,
                                       self.scale_atoms, self.scale_atoms.numel())
            else:
                dsv4.build_shared_scale_atoms(self.w1.scale, self.w2.scale, self.w3.scale, self.dim, self.inter_dim,
                                              self.scale_atoms)

    def _desc(self) -> MoELayerDesc:
        d = MoELayerDesc()
        d.hidden, d.inter = self.dim, self.inter_dim
        d.swiglu_limit = self.swiglu_limit
        d.route_scale = 1.0
        if self.fp4:
            d.n_routed, d.topk, d.n_shared = 1, 1, 0
            d.arena = ptr(self.block)
            d.slot_stride = _round_up(self.block.numel(), 32) if self.block.numel() % 32 else self.block.numel()
            d.n_slots = 1
            d.arena_sf = ptr(self.scale_atoms)
            d.sf_slot_stride = self.scale_atoms.numel()
            d.expert_slot = ptr(self._slot0)
        else:
            d.n_routed, d.topk, d.n_shared = 0, 1, 1
            d.shared_w1, d.shared_w2, d.shared_w3 = ptr(self.w1.weight), ptr(self.w2.weight), ptr(self.w3.weight)
            d.shared_sf = ptr(self.scale_atoms)
        return d

    def layer_args(self) -> tuple[list, list[int], list[float]]:
        """The op layer's (layer, dims, scalars) lists for this expert."""
        if self.fp4:
            tensors = [None, None, self.block, self.scale_atoms, self._slot0, None, None, None, None]
        else:
            tensors = [None, None, None, None, None, self.w1.weight, self.w2.weight, self.w3.weight,
                       self.scale_atoms]
        return ops.layer_args(self._desc(), tensors)

    def forward(self, x: torch.Tensor, weights: torch.Tensor | None = None) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.dim)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        w = None
        if weights is not None:
            w = weights.reshape(-1).to(torch.float32).contiguous()
            if w.numel() != x2.shape[0]:
                raise RuntimeError("routing weights must have one entry per row")
        y = ops.load().expert_forward(x2, 0 if self.fp4 else -1, w, *self.layer_args())
        return y.view(*shape[:-1], self.dim).to(x.dtype)


def _round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


# ---------------------------------------------------------------------------
# ExpertArena: slots of one device buffer
# ---------------------------------------------------------------------------
class ExpertArena:
    """Pool of routed-expert slots in one device buffer.

    Same contract as the reference's ``ExpertArena`` (lazy_official_runtime.py:
    641-667): ``acquire(factory) -> (expert, reused)`` hands out a slot-backed
    ``Expert`` (``factory`` is only called when every slot is taken),
    ``release(expert) -> bool`` returns its slot to the pool.  On B200 the slots
    are one contiguous allocation, so a layer's resident experts form the
    arena the grouped GEMM streams (one tensor map over all slots)."""

    def __init__(self, max_slots: int, dim: int = 4096, inter: int = 2048, *, device="cuda",
                 swiglu_limit: float = 0.0):
        self.max_slots = max(0, int(max_slots))
        self.enabled = self.max_slots > 0
        self.dim, self.inter = dim, inter
        self.swiglu_limit = swiglu_limit
        self.block_bytes = packed_block_bytes(dim, inter)
        self.slot_stride = _round_up(self.block_bytes, 256)
        self.sf_stride = scale_atom_bytes(dim, inter)
        self.device = torch.device(device)
        n = max(self.max_slots, 1)
        self.buffer = torch.zeros(n * self.slot_stride, dtype=torch.uint8, device=self.device)
        self.sf = torch.zeros(n * self.sf_stride, dtype=torch.uint8, device=self.device)
        from .telemetry import expert_telemetry

        expert_telemetry().register_resident(max_slots, self.buffer.numel() + self.sf.numel())
        self._free = list(range(self.max_slots - 1, -1, -1))
        self._experts: dict[int, Expert] = {}
        self._released: set[int] = set()

    def slot_storage(self, slot: int) -> tuple[torch.Tensor, torch.Tensor]:
        s = self.buffer[slot * self.slot_stride:(slot + 1) * self.slot_stride]
        f = self.sf[slot * self.sf_stride:(slot + 1) * self.sf_stride]
        return s, f

    def expert_for_slot(self, slot: int) -> Expert:
        e = self._experts.get(slot)
        if e is None:
            s, f = self.slot_storage(slot)
            e = Expert(self.dim, self.inter, dtype=FP4, swiglu_limit=self.swiglu_limit, storage=s,
                       scale_atoms=f)
            e._arena_slot = slot
            self._experts[slot] = e
        return e

    def acquire(self, factory=None) -> tuple[nn.Module, bool]:
        if self.enabled and self._free:
            slot = self._free.pop()
            reused = slot in self._released
            return self.expert_for_slot(slot), reused
        if factory is None:
            raise RuntimeError("expert arena is full")
        return factory(), False

    def release(self, expert: nn.Module) -> bool:
        slot = getattr(expert, "_arena_slot", None)
        if not self.enabled or slot is None or slot in self._free:
            return False
        self._free.append(slot)
        self._released.add(slot)
        return True

    def materialize(self, slab: torch.Tensor, src_offsets: list[int], slots: list[int], *,
                    bf16_out: torch.Tensor | None = None, stream=None) -> int:
        """Device-side materializer: packed blocks already in device memory
        (``slab``, byte offsets ``src_offsets``) -> arena ``slots`` (bit-exact),
        plus their scale atoms and, optionally, an exact bf16 decode.  Returns the
        bytes copied (ExpertCopyPlan's copied_bytes)."""
        n = len(slots)
        if n == 0:
            return 0
        if len(src_offsets) != n:
            raise RuntimeError("targets and offsets length mismatch")
        off = torch.tensor(src_offsets, dtype=torch.int64).to(slab.device, non_blocking=True)
        sl = torch.tensor(slots, dtype=torch.int32).to(slab.device, non_blocking=True)
        bf16_stride = 0
        if bf16_out is not None:
            bf16_stride = bf16_out.shape[-1] if bf16_out.dim() > 1 else bf16_out.numel() // max(self.max_slots, 1)
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            ops.load().materialize(slab, off, sl, self.buffer, self.slot_stride, self.sf, self.sf_stride, bf16_out,
                                   bf16_stride, self.dim, self.inter)
        from .telemetry import expert_telemetry

        expert_telemetry().record_materialize(n * self.block_bytes)
        return n * self.block_bytes


# ---------------------------------------------------------------------------
# Gate
# ---------------------------------------------------------------------------
class Gate(nn.Module):
    """Official ``Gate(layer_id, args)``; ``forward(x, input_ids) -> (weights, indices)``.

    Sigmoid scores of ``x . weight^T`` (fp32), selection on score + ``bias``,
    top-k, weights renormalised to sum 1 and scaled by ``route_scale``
    (weights fp32 [N,k], indices int64 [N,k])."""

    def __init__(self, layer_id: int, args: ModelArgs, *, device=None):
        super().__init__()
        self.layer_id = layer_id
        self.dim = args.dim
        self.n_experts = args.n_routed_experts
        self.topk = args.n_activated_experts
        self.route_scale = float(args.route_scale)
        if args.score_func != "sigmoid":
            raise RuntimeError(f"unsupported score function {args.score_func!r}")
        device = device or "cuda"
        self.hashed = layer_id < args.n_hash_layers
        self.weight = nn.Parameter(torch.zeros(self.n_experts, self.dim, dtype=args.gate_dtype, device=device),
                                   requires_grad=False)
        if self.hashed:  # checkpoint tensor gate.tid2eid [vocab, k] int64; no correction bias
            self.register_buffer("tid2eid", torch.zeros(args.vocab_size, self.topk, dtype=torch.int64,
                                                        device=device))
            self.register_parameter("bias", None)
        elif args.gate_bias:
            self.bias = nn.Parameter(torch.zeros(self.n_experts, dtype=torch.float32, device=device),
                                     requires_grad=False)
        else:
            self.register_parameter("bias", None)

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        x = x.reshape(-1, self.dim).to(torch.bfloat16).contiguous()
        return ops.load().gate_logits(x, self.weight)

    def route(self, logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return ops.load().gate_topk(logits.to(torch.float32).contiguous(), self.bias, self.topk, self.route_scale)

    def forward(self, x: torch.Tensor, input_ids: torch.Tensor | None = None):
        x = x.reshape(-1, self.dim).to(torch.bfloat16).contiguous()
        dsv4 = ops.load()
        if self.hashed:
            if input_ids is None:
                raise RuntimeError(f"layer {self.layer_id} routes by token id: input_ids is required")
            ids = input_ids.reshape(-1).to(device=x.device, dtype=torch.int64).contiguous()
            if ids.numel() != x.shape[0]:
                raise RuntimeError("input_ids must hold one id per token")
            w, idx, logits = dsv4.gate_route(x, self.weight, None, self.topk, self.route_scale, self.tid2eid, ids)
        else:
            w, idx, logits = dsv4.gate_route(x, self.weight, self.bias, self.topk, self.route_scale)
        self.last_logits = logits
        return w, idx


# ---------------------------------------------------------------------------
# MoE
# ---------------------------------------------------------------------------
class MoE(nn.Module):
    """``MoE(layer_id, args)``; ``forward(x [B,S,H] bf16, input_ids [B,S]) -> [B,S,H]``.

    Expert ownership follows the reference's expert-parallel split
    (lazy_official_runtime.py:956-965): rank r of W owns experts
    [r*E/W, (r+1)*E/W).  With one rank the whole layer is one call of
    ``dsv4_moe_forward`` (no host synchronisation); with several ranks tokens
    are dispatched to the owning ranks (see ``spark_b200.ep``)."""

    def __init__(self, layer_id: int, args: ModelArgs, *, device=None, arena: ExpertArena | None = None,
                 group=None):
        super().__init__()
        self.group = group
        world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_available() and dist.is_initialized() else 0
        if args.n_routed_experts % world:
            raise AssertionError("n_routed_experts must divide evenly across ranks")
        if args.n_shared_experts != 1:
            raise AssertionError("exactly one shared expert is supported")
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        self.layer_id = layer_id
        self.args = args
        self.dim = args.dim
        self.world, self.rank = world, rank
        self.n_routed_experts = args.n_routed_experts
        self.n_local_experts = args.n_routed_experts // world
        self.n_activated_experts = args.n_activated_experts
        self.experts_start_idx = rank * self.n_local_experts
        self.experts_end_idx = self.experts_start_idx + self.n_local_experts
        self.gate = Gate(layer_id, args, device=device)
        self.arena = arena if arena is not None else ExpertArena(
            self.n_local_experts, args.dim, args.moe_inter_dim, device=device, swiglu_limit=args.swiglu_limit)
        slots = torch.full((self.n_routed_experts,), 0, dtype=torch.int32)
        experts = []
        for i in range(self.n_routed_experts):
            if self.experts_start_idx <= i < self.experts_end_idx:
                e, _ = self.arena.acquire()
                slots[i] = e._arena_slot
                experts.append(e)
            else:
                experts.append(None)
        self.experts = nn.ModuleList(experts)
        self.register_buffer("expert_slot", slots.to(device), persistent=False)
        self.shared_experts = Expert(args.dim, args.moe_inter_dim, swiglu_limit=args.swiglu_limit, device=device)
        self.register_load_state_dict_post_hook(lambda m, _keys: m.refresh_scale_atoms())

    def enable_peer_exchange(self, cap_tokens: int) -> None:
        """Expert parallelism over NVLink peer memory from now on (collective:
        every rank of the group calls it with the same cap_tokens, the most
        tokens any rank will pass per call)."""
        if self.world == 1:
            return
        from .ep import PeerExchange

        old = getattr(self, "peer_exchange", None)
        self.reset_graphs()
        if old is not None:
            old.close()
        self.peer_exchange = PeerExchange(self, cap_tokens, group=self.group)

    def refresh_scale_atoms(self) -> None:
        slots = self.expert_slot[self.experts_start_idx:self.experts_end_idx].contiguous()
        ops.load().build_scale_atoms(self.arena.buffer, self.arena.slot_stride, slots, self.dim,
                                     self.args.moe_inter_dim, self.arena.sf, self.arena.sf_stride)
        self.shared_experts.refresh_scale_atoms()

    def layer_desc(self) -> MoELayerDesc:
        a = self.args
        d = MoELayerDesc()
        d.hidden, d.inter = a.dim, a.moe_inter_dim
        d.n_routed, d.topk, d.n_shared = a.n_routed_experts, a.n_activated_experts, 1
        d.route_scale, d.swiglu_limit = float(a.route_scale), float(a.swiglu_limit or 0.0)
        d.gate_w = ptr(self.gate.weight)
        d.gate_w_fp32 = int(self.gate.weight.dtype == torch.float32)
        d.gate_bias = ptr(self.gate.bias)
        d.arena, d.slot_stride, d.n_slots = ptr(self.arena.buffer), self.arena.slot_stride, max(self.arena.max_slots, 1)
        d.arena_sf, d.sf_slot_stride = ptr(self.arena.sf), self.arena.sf_stride
        d.expert_slot = ptr(self.expert_slot)
        sh = self.shared_experts
        d.shared_w1, d.shared_w2, d.shared_w3 = ptr(sh.w1.weight), ptr(sh.w2.weight), ptr(sh.w3.weight)
        d.shared_sf = ptr(sh.scale_atoms)
        return d

    def layer_args(self) -> tuple[list, list[int], list[float]]:
        """The op layer's (layer, dims, scalars) lists for this layer."""
        sh = self.shared_experts
        tensors = [self.gate.weight, self.gate.bias, self.arena.buffer, self.arena.sf, self.expert_slot,
                   sh.w1.weight, sh.w2.weight, sh.w3.weight, sh.scale_atoms]
        return ops.layer_args(self.layer_desc(), tensors)

    def workspace_bytes(self, T: int) -> int:
        d = self.layer_desc()
        return int(_lib.load().dsv4_moe_workspace_bytes(ctypes.byref(d), T))

    def forward_tokens(self, x: torch.Tensor, *, routing: tuple[torch.Tensor, torch.Tensor] | None = None,
                       workspace: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Single-rank layer over x [T,H] bf16 -> [T,H] bf16 (no host sync), one
        ``torch.ops.dsv4moe.moe_forward`` call."""
        rw = ri = None
        if routing is not None:
            rw = routing[0].to(torch.float32).contiguous()
            ri = routing[1].to(torch.int64).contiguous()
        dsv4 = ops.load()
        if out is None:
            return dsv4.moe_forward(x, *self.layer_args(), rw, ri, workspace)
        dsv4.moe_forward_out(x, *self.layer_args(), rw, ri, workspace, out)
        return out

    def forward(self, x: torch.Tensor, input_ids: torch.Tensor | None = None) -> torch.Tensor:
        shape = x.size()
        x2 = x.reshape(-1, self.dim)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        routing = self.gate(x2, input_ids) if self.gate.hashed else None
        from .telemetry import expert_telemetry

        tel = expert_telemetry()
        if tel.route_trace_path is not None:
            # the reference's route trace needs this call's routing on the host;
            # the layer then runs on exactly that routing
            if routing is None:
                routing = self.gate(x2, input_ids)
            ids = input_ids if input_ids is not None else torch.empty(0, dtype=torch.int64)
            tel.record_routing(layer_id=self.layer_id, input_ids=ids, expert_indices=routing[1],
                               tokens=x2.shape[0])
        else:
            tel.count_routing(x2.shape[0], x2.shape[0] * self.n_activated_experts)
        if self._graph_ok(x2, routing, tel):
            y = self._graph_forward(x2)
        elif self.world == 1:
            y = self.forward_tokens(x2, routing=routing)
        else:
            from .ep import ep_moe_forward

            y = ep_moe_forward(self, x2, routing=routing)
        return y.type_as(x).view(shape)

    # ------------------------------------------------------------ graphs
    def _graph_ok(self, x2, routing, tel) -> bool:
        """Graph replay applies to decode-sized calls whose routing the layer
        computes itself, with no route trace, on one rank or over peer memory
        (the host-collective exchange needs the host between its steps), and
        not while the caller is capturing a graph of its own."""
        return (_GRAPHS_ON and routing is None and tel.route_trace_path is None
                and 0 < x2.shape[0] <= GRAPH_MAX_TOKENS
                and (self.world == 1 or getattr(self, "peer_exchange", None) is not None)
                and not torch.cuda.is_current_stream_capturing())

    def _graph_key(self) -> tuple:
        """Every address a captured layer holds, and the library's settings
        generation (split-K, FP4 activations): a change of any recaptures."""
        sh = self.shared_experts
        ex = getattr(self, "peer_exchange", None)
        return (_lib.load().dsv4_settings_generation(), self.gate.weight.data_ptr(), ptr(self.gate.bias), self.arena.buffer.data_ptr(),
                self.arena.sf.data_ptr(), self.expert_slot.data_ptr(), sh.w1.weight.data_ptr(),
                sh.w2.weight.data_ptr(), sh.w3.weight.data_ptr(), sh.scale_atoms.data_ptr(),
                ex.buf.value if ex is not None else 0)

    def _graph_body(self, x2: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return self.forward_tokens(x2)
        from .ep import ep_forward_peer

        return ep_forward_peer(self.peer_exchange, x2)

    def _graph_forward(self, x2: torch.Tensor) -> torch.Tensor:
        """The layer as a replayed CUDA graph, one per token count.  A new
        token count is captured (nothing runs while capturing) and then
        replayed, so every call, the first included, is exactly one layer
        call: expert-parallel ranks stay in step whatever their own counts.
        Under expert parallelism the exchange's poisoning check and error-word
        copy run on the host around each replay, as around an eager call."""
        graphs = self.__dict__.setdefault("_graphs", {})
        T = x2.shape[0]
        key = self._graph_key()
        entry = graphs.get(T)
        if entry is not None and entry[3] != key:
            del graphs[T]
            entry = None
        ex = getattr(self, "peer_exchange", None) if self.world > 1 else None
        if ex is not None:
            ex.check_poisoned()
        if entry is None:
            while len(graphs) >= GRAPH_MAX_ENTRIES:
                graphs.pop(next(iter(graphs)))
            if ex is not None:
                ex.workspace(T)  # sized outside the capture, shared with eager calls
            static_x = x2.clone()
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(device=x2.device)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(graph, stream=side):
                static_y = self._graph_body(static_x)
            torch.cuda.current_stream().wait_stream(side)
            entry = (graph, static_x, static_y, key)
            graphs[T] = entry
        else:
            entry[1].copy_(x2)
        entry[0].replay()
        if ex is not None:
            ex.note_call_end()
        return entry[2].clone()

    @staticmethod
    def set_fp4_activations(on: bool) -> None:
        """Opt-in FP4 activations for the routed experts' w1 | w3
        (``dsv4_set_fp4_activations``): the FP4 tensor rate at prefill, at the
        cost of the layer's numerics (the reference quantizes to e4m3).
        Process-wide; set it before sizing workspaces."""
        _lib.check(_lib.load().dsv4_set_fp4_activations(1 if on else 0), "dsv4_set_fp4_activations")

    def reset_graphs(self) -> None:
        """Drop the captured graphs (they are recaptured on the next calls)."""
        self.__dict__.pop("_graphs", None)
