"""Packed routed-expert slab: reader (drop-in for PackedExpertStore) and writer.

Format (scripts/build_packed_expert_layout.py:76-86,179-237): one
``layer_XX.bin`` per layer holding each expert's tensors contiguously in the
order w1.scale, w2.scale, w3.scale, w1.weight, w2.weight, w3.weight, plus a
``layout.json`` ``{version, created_at_unix, model_dir, manifest_csv,
layers: {L: {path, bytes, experts: {E: {offset, bytes, tensors: {name:
{offset, bytes, source_dtype, source_shape, transform}}}}}}}`` written
atomically (tmp + rename).

``PackedExpertStore`` keeps the reference's constructor, ``from_env``,
``tensors_for_expert``, ``native_plan_for_expert``, ``read_and_copy_with_plan``,
``copy_storage_to_tensors``, ``copy_storage_with_plan`` and ``close``
(spark_runtime/lazy_official_runtime.py:49-338), and adds the B200 bulk path
``upload_experts``: one pread per expert into a single pinned buffer, one
host-to-device copy of all blocks, then the device materializer fills the
arena slots (``ExpertArena.materialize``).
"""

from __future__ import annotations

import json
import os
import threading
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import native_packed_loader as _native
from .moe import PACKED_ORDER, ExpertArena

_TRUE = {"1", "true", "yes"}


def _flag(name: str) -> bool:
    return os.getenv(name, "0") in _TRUE


@dataclass(frozen=True)
class PackedExpertBatch:
    tensors: dict[str, torch.Tensor]
    tensor_infos: dict[str, dict[str, Any]]
    read_seconds: float
    read_bytes: int
    _storage: Any


@dataclass(frozen=True)
class NativeExpertCopyPlan:
    plan: Any
    parameter_indices: tuple[int, ...]
    fallback_indices: tuple[int, ...]


def _source_dtype_to_torch(dtype_name: str) -> torch.dtype:
    """lazy_official_runtime.py:341-353."""
    mapping = {
        "BF16": torch.bfloat16,
        "F32": torch.float32,
        "F8_E8M0": torch.float8_e8m0fnu,
        "I8": torch.int8,
        "I32": torch.int32,
        "I64": torch.int64,
    }
    try:
        return mapping[dtype_name]
    except KeyError as exc:
        raise ValueError(f"unsupported packed source dtype: {dtype_name}") from exc


class PackedExpertStore:
    def __init__(self, layout_path: Path):
        self.layout_path = Path(layout_path)
        self.base_dir = self.layout_path.parent
        self.layout = json.loads(self.layout_path.read_text())
        self.layers: dict[str, Any] = self.layout.get("layers", {})
        self.native_pinned_staging = _flag("DEEPSEEK_SPARK_PACKED_NATIVE_PINNED_STAGING")
        self.native_cuda_memcpy = _flag("DEEPSEEK_SPARK_NATIVE_CUDA_MEMCPY")
        self.native_copy_plan = True
        self.native_fused_materializer = True
        self._native_module = _native.load_native_packed_loader()
        self._fds: dict[Path, int] = {}
        self._lock = threading.Lock()
        self._thread_local = threading.local()
        self._copy_plans: dict[tuple[int, int, tuple[str, ...]], NativeExpertCopyPlan] = {}

    @classmethod
    def from_env(cls) -> "PackedExpertStore | None":
        value = os.getenv("DEEPSEEK_SPARK_PACKED_EXPERT_LAYOUT")
        return cls(Path(value)) if value else None

    def close(self) -> None:
        with self._lock:
            for fd in self._fds.values():
                os.close(fd)
            self._fds.clear()

    def _fd(self, path: Path) -> int:
        with self._lock:
            fd = self._fds.get(path)
            if fd is None:
                fd = os.open(path, os.O_RDONLY)
                self._fds[path] = fd
            return fd

    def _expert_entry(self, layer_id: int, expert_id: int):
        layer = self.layers.get(str(layer_id))
        if layer is None:
            return None
        expert = layer.get("experts", {}).get(str(expert_id))
        if expert is None:
            return None
        path = Path(layer["path"])
        if not path.is_absolute():
            path = self.base_dir / path
        return path, int(expert["offset"]), int(expert["bytes"]), expert["tensors"]

    def _native_staging(self, size: int) -> torch.Tensor:
        staging = getattr(self._thread_local, "staging", None)
        pinned = self.native_pinned_staging and torch.cuda.is_available()
        if staging is None or staging.numel() < size or getattr(self._thread_local, "pinned", False) != pinned:
            staging = torch.empty(size, dtype=torch.uint8, device="cpu", pin_memory=pinned)
            self._thread_local.staging = staging
            self._thread_local.pinned = pinned
        return staging[:size]

    @staticmethod
    def _tensor_from_storage(storage: torch.Tensor, tensor_info: dict[str, Any]) -> torch.Tensor:
        offset = int(tensor_info["offset"])
        size = int(tensor_info["bytes"])
        dtype = _source_dtype_to_torch(tensor_info["source_dtype"])
        shape = [int(d) for d in tensor_info["source_shape"]]
        return storage[offset:offset + size].view(dtype).reshape(shape)

    def tensors_for_expert(self, layer_id: int, expert_id: int) -> PackedExpertBatch | None:
        entry = self._expert_entry(layer_id, expert_id)
        if entry is None:
            return None
        path, offset, size, tensor_infos = entry
        fd = self._fd(path)
        start = time.monotonic()
        view = self._native_staging(size)
        got = self._native_module.read_into(fd, view, size, offset)
        read_seconds = time.monotonic() - start
        if got != size:
            raise OSError(f"short packed expert read: layer={layer_id} expert={expert_id}")
        tensors = {name: self._tensor_from_storage(view, info) for name, info in tensor_infos.items()}
        return PackedExpertBatch(tensors, tensor_infos, read_seconds, size, view)

    def native_plan_for_expert(self, layer_id: int, expert_id: int, prefix: str,
                               parameters: list[tuple[str, torch.nn.Parameter]]) -> NativeExpertCopyPlan | None:
        entry = self._expert_entry(layer_id, expert_id)
        if entry is None:
            return None
        _, _, _, tensor_infos = entry
        key = (layer_id, expert_id, tuple(name for name, _ in parameters))
        plan = self._copy_plans.get(key)
        if plan is not None:
            return plan
        offsets, sizes, idx, fallback = [], [], [], []
        for index, (name, param) in enumerate(parameters):
            info = tensor_infos.get(f"{prefix}.{name}")
            if info is None:
                fallback.append(index)
                continue
            offsets.append(int(info["offset"]))
            sizes.append(param.numel() * param.element_size())
            idx.append(index)
        native = self._native_module.ExpertCopyPlan(offsets, sizes) if offsets else None
        plan = NativeExpertCopyPlan(native, tuple(idx), tuple(fallback))
        self._copy_plans[key] = plan
        return plan

    def read_and_copy_with_plan(self, layer_id: int, expert_id: int, plan, targets: list[torch.Tensor], *,
                                non_blocking: bool):
        entry = self._expert_entry(layer_id, expert_id)
        if entry is None:
            return None
        path, offset, size, _ = entry
        fd = self._fd(path)
        staging = self._native_staging(size)
        if self.native_cuda_memcpy:
            res = plan.read_into_and_copy_cuda(fd, staging, size, offset, targets)
        else:
            res = plan.read_into_and_copy(fd, staging, size, offset, targets, non_blocking)
        return int(res[0]), int(res[1]), float(res[2]), float(res[3])

    def copy_storage_to_tensors(self, storage, targets, offsets, *, non_blocking: bool) -> int:
        return int(self._native_module.copy_storage_to_tensors(storage, targets, offsets, non_blocking))

    def copy_storage_with_plan(self, plan, storage, targets, *, non_blocking: bool) -> int:
        if self.native_cuda_memcpy:
            return int(plan.copy_storage_to_tensors_cuda(storage, targets))
        return int(plan.copy_storage_to_tensors(storage, targets, non_blocking))

    # -------------------------------------------------------------- B200 bulk path
    def read_blocks(self, layer_id: int, experts: list[int]) -> tuple[torch.Tensor, list[int], float]:
        """All blocks of ``experts`` in one (pinned when CUDA is present) host
        buffer: returns (buffer, byte offset of each block, read seconds)."""
        entries = [self._expert_entry(layer_id, e) for e in experts]
        if any(e is None for e in entries):
            missing = [x for x, e in zip(experts, entries) if e is None]
            raise KeyError(f"experts missing from the packed layout: layer={layer_id} experts={missing}")
        offs, total = [], 0
        for _, _, size, _ in entries:
            offs.append(total)
            total += (size + 255) // 256 * 256
        buf = torch.empty(max(total, 1), dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        t0 = time.monotonic()
        for (path, offset, size, _), o in zip(entries, offs):
            got = self._native_module.read_into(self._fd(path), buf[o:o + size], size, offset)
            if got != size:
                raise RuntimeError("short packed expert read")
        dt = time.monotonic() - t0
        from .telemetry import expert_telemetry

        expert_telemetry().record_packed_read(len(experts), sum(e[2] for e in entries), dt)
        return buf, offs, dt

    def upload_experts(self, layer_id: int, experts: list[int], arena: ExpertArena, slots: list[int], *,
                       bf16_out: torch.Tensor | None = None, stream=None) -> dict[str, float]:
        """Fill arena ``slots`` with ``experts`` of ``layer_id``: pread into one
        pinned buffer, one host-to-device copy, device materializer (bit-exact
        bytes + scale atoms).  Returns the reference's stats keys."""
        buf, offs, read_s = self.read_blocks(layer_id, experts)
        t0 = time.monotonic()
        dev_slab = buf.to(arena.device, non_blocking=True)
        copied = arena.materialize(dev_slab, offs, slots, bf16_out=bf16_out, stream=stream)
        torch.cuda.current_stream(arena.device).synchronize()
        return {"packed_loads": len(experts), "packed_read_bytes": int(sum(
            self._expert_entry(layer_id, e)[2] for e in experts)), "packed_read_seconds": read_s,
            "materialize_seconds": time.monotonic() - t0, "copied_bytes": copied}


def _tensor_meta(name: str, dim: int, inter: int) -> tuple[str, list[int], str]:
    """(source_dtype, source_shape, transform) of a routed-expert tensor in the
    checkpoint manifest (results/spark-66c9/weight-manifest.csv:4731-4733,5510-5512)."""
    w, kind = name.split(".")
    rows, k = (dim, inter) if w == "w2" else (inter, dim)
    if kind == "scale":
        return "F8_E8M0", [rows, k // 32], "copy"
    return "I8", [rows, k // 2], "reinterpret_int8_as_fp4"


def write_packed_layout(out_dir: Path, blocks: dict[int, dict[int, np.ndarray]], dim: int, inter: int, *,
                        model_dir: str = "", manifest_csv: str = "", created_at: float | None = None) -> dict:
    """Write layer_XX.bin + layout.json for ``blocks[layer][expert]`` (packed
    blocks as uint8 arrays), byte-identical to the reference builder's output
    for the same tensors."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    sizes = {"w1.scale": inter * dim // 32, "w2.scale": dim * inter // 32, "w3.scale": inter * dim // 32,
             "w1.weight": inter * dim // 2, "w2.weight": dim * inter // 2, "w3.weight": inter * dim // 2}
    layout: dict[str, Any] = {"version": 1, "created_at_unix": time.time() if created_at is None else created_at,
                              "model_dir": model_dir, "manifest_csv": manifest_csv, "layers": {}}
    for layer in sorted(blocks):
        path = out_dir / f"layer_{layer:02d}.bin"
        entry: dict[str, Any] = {"path": path.name, "bytes": 0, "experts": {}}
        with path.open("wb") as f:
            for expert in sorted(blocks[layer]):
                blk = np.ascontiguousarray(blocks[layer][expert], dtype=np.uint8)
                start = f.tell()
                tensors, off = {}, 0
                for name in PACKED_ORDER:
                    dt, shape, transform = _tensor_meta(name, dim, inter)
                    tensors[f"layers.{layer}.ffn.experts.{expert}.{name}"] = {
                        "offset": off, "bytes": sizes[name], "source_dtype": dt, "source_shape": shape,
                        "transform": transform}
                    off += sizes[name]
                if blk.size != off:
                    raise ValueError(f"block of expert {expert} has {blk.size} bytes, expected {off}")
                f.write(blk.tobytes())
                entry["experts"][str(expert)] = {"offset": start, "bytes": f.tell() - start, "tensors": tensors}
        entry["bytes"] = path.stat().st_size
        layout["layers"][str(layer)] = entry
    tmp = out_dir / "layout.json.tmp"
    tmp.write_text(json.dumps(layout, indent=2, sort_keys=True), encoding="utf-8")
    tmp.replace(out_dir / "layout.json")
    return layout
