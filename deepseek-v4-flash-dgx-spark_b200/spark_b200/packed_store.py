"""Packed routed-expert slab: reader (drop-in for PackedExpertStore) and writer.

Format (scripts/build_packed_expert_layout.py:76-86,179-237): one
``layer_XX.bin`` per layer holding each expert's tensors contiguously in the
order w1.scale, w2.scale, w3.scale, w1.weight, w2.weight, w3.weight, plus a
``layout.json`` ``{version, created_at_unix, model_dir, manifest_csv,
layers: {L: {path, bytes, experts: {E: {offset, bytes, tensors: {name:
{offset, bytes, source_dtype, source_shape, transform}}}}}}}`` written
atomically (tmp + rename).

``PackedExpertStore`` answers the reference's interface (constructor,
``from_env``, ``tensors_for_expert``, ``native_plan_for_expert``,
``read_and_copy_with_plan``, ``copy_storage_to_tensors``,
``copy_storage_with_plan``, ``close``; spark_runtime/lazy_official_runtime.py:
49-338).  Inside, the layout is parsed once into a flat index (``SlabIndex``:
one row per expert with its file, offset and size, and the sub-offsets of its
tensors); every lookup, read and copy plan is derived from that index.

The B200 path is ``upload_experts``: experts move to the device in chunks
through two reused pinned staging buffers and two device slab buffers, so the
pread of chunk i+1 (host), the host-to-device copy of chunk i (a copy stream,
one ``cudaMemcpyAsync`` per chunk) and the device materializer of chunk i-1
(the caller's stream) overlap.
"""

from __future__ import annotations

import json
import os
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import native_packed_loader as _native
from .moe import PACKED_ORDER, ExpertArena

# environment switches the reference's store reads (values "1", "true", "yes")
_ENV_PINNED = "DEEPSEEK_SPARK_PACKED_NATIVE_PINNED_STAGING"
_ENV_CUDA_MEMCPY = "DEEPSEEK_SPARK_NATIVE_CUDA_MEMCPY"
_ENV_LAYOUT = "DEEPSEEK_SPARK_PACKED_EXPERT_LAYOUT"

# source_dtype names of the layout -> torch dtypes (lazy_official_runtime.py:341-353)
_DTYPES = {"BF16": torch.bfloat16, "F32": torch.float32, "F8_E8M0": torch.float8_e8m0fnu, "I8": torch.int8,
           "I32": torch.int32, "I64": torch.int64}


def _env_on(name: str) -> bool:
    return os.environ.get(name, "0").strip().lower() in ("1", "true", "yes")


def _torch_dtype(name: str) -> torch.dtype:
    dt = _DTYPES.get(name)
    if dt is None:
        raise ValueError(f"unsupported packed source dtype: {name}")
    return dt


@dataclass(frozen=True)
class PackedExpertBatch:
    """One expert block read into host memory: tensor views into ``_storage``."""

    tensors: dict[str, torch.Tensor]
    tensor_infos: dict[str, dict[str, Any]]
    read_seconds: float
    read_bytes: int
    _storage: Any


@dataclass(frozen=True)
class NativeExpertCopyPlan:
    """Copy plan of one expert's parameters: the loader plan over the
    parameters found in the block, and the indices of those found / missing."""

    plan: Any
    parameter_indices: tuple[int, ...]
    fallback_indices: tuple[int, ...]


class SlabIndex:
    """layout.json flattened: row r of the index is one (layer, expert) block,
    at ``offset[r]`` of file ``files[file_id[r]]``, ``nbytes[r]`` long, with its
    tensors' layout entries in ``tensors[r]`` (name -> info, offsets relative
    to the block)."""

    def __init__(self, layout: dict, base_dir: Path):
        self.files: list[Path] = []
        self.rows: dict[tuple[int, int], int] = {}
        file_id, offset, nbytes = [], [], []
        self.tensors: list[dict[str, dict[str, Any]]] = []
        for lkey in sorted(layout.get("layers", {}), key=int):
            lentry = layout["layers"][lkey]
            path = Path(lentry["path"])
            self.files.append(path if path.is_absolute() else base_dir / path)
            fid = len(self.files) - 1
            for ekey in sorted(lentry.get("experts", {}), key=int):
                e = lentry["experts"][ekey]
                self.rows[(int(lkey), int(ekey))] = len(offset)
                file_id.append(fid)
                offset.append(int(e["offset"]))
                nbytes.append(int(e["bytes"]))
                self.tensors.append(e["tensors"])
        self.file_id = np.asarray(file_id, dtype=np.int32)
        self.offset = np.asarray(offset, dtype=np.int64)
        self.nbytes = np.asarray(nbytes, dtype=np.int64)

    def row(self, layer_id: int, expert_id: int) -> int | None:
        return self.rows.get((int(layer_id), int(expert_id)))

    def rows_for(self, layer_id: int, experts: list[int]) -> np.ndarray:
        rows = [self.row(layer_id, e) for e in experts]
        missing = [e for e, r in zip(experts, rows) if r is None]
        if missing:
            raise KeyError(f"experts missing from the packed layout: layer={layer_id} experts={missing}")
        return np.asarray(rows, dtype=np.int64)


class _Staging:
    """Per-thread host staging buffer, grown to the largest request and
    reused; pinned when requested and CUDA is present."""

    def __init__(self, pinned: bool):
        self.pinned = pinned and torch.cuda.is_available()
        self._local = threading.local()

    def get(self, size: int) -> torch.Tensor:
        buf = getattr(self._local, "buf", None)
        if buf is None or buf.numel() < size:
            cap = max(size, 1 << 20)
            buf = torch.empty(cap, dtype=torch.uint8, pin_memory=self.pinned)
            self._local.buf = buf
        return buf[:size]


_READ_PIECE = 4 << 20  # bytes per pread piece of a block


class PackedExpertStore:
    def __init__(self, layout_path: Path):
        self.layout_path = Path(layout_path)
        self.base_dir = self.layout_path.parent
        self.layout = json.loads(self.layout_path.read_text())
        self.layers: dict[str, Any] = self.layout.get("layers", {})
        self.index = SlabIndex(self.layout, self.base_dir)
        # the native loader and its copy plans are always on here; the two
        # switches below keep their reference meaning
        self.native_pinned_staging = _env_on(_ENV_PINNED)
        self.native_cuda_memcpy = _env_on(_ENV_CUDA_MEMCPY)
        self.native_copy_plan = True
        self.native_fused_materializer = True
        self._native_module = _native.load_native_packed_loader()
        self._staging = _Staging(self.native_pinned_staging)
        self._fd_lock = threading.Lock()
        self._fd_of_file: list[int | None] = [None] * len(self.index.files)
        self._plans: dict[tuple[int, tuple[str, ...]], NativeExpertCopyPlan] = {}
        self._upload: dict[tuple[str, int], dict[str, Any]] = {}  # per device: pinned + device rings
        # blocks are pread in pieces of at most _READ_PIECE bytes by this many
        # threads at once (each piece is one native call that releases the
        # GIL); DSV4_READ_THREADS overrides
        self.read_threads = max(1, int(os.environ.get("DSV4_READ_THREADS", min(8, os.cpu_count() or 1))))
        self._read_pool: ThreadPoolExecutor | None = None

    @classmethod
    def from_env(cls) -> "PackedExpertStore | None":
        path = os.environ.get(_ENV_LAYOUT)
        return cls(Path(path)) if path else None

    def close(self) -> None:
        if self._read_pool is not None:
            self._read_pool.shutdown(wait=True)
            self._read_pool = None
        with self._fd_lock:
            for i, fd in enumerate(self._fd_of_file):
                if fd is not None:
                    os.close(fd)
                    self._fd_of_file[i] = None
        self._upload.clear()

    # ------------------------------------------------------------------ lookups
    def _descriptor(self, file_id: int) -> int:
        with self._fd_lock:
            fd = self._fd_of_file[file_id]
            if fd is None:
                fd = os.open(self.index.files[file_id], os.O_RDONLY)
                self._fd_of_file[file_id] = fd
            return fd

    def _block(self, layer_id: int, expert_id: int) -> tuple[int, int, int, dict] | None:
        """(descriptor, file offset, bytes, tensor infos) of one block, or None."""
        r = self.index.row(layer_id, expert_id)
        if r is None:
            return None
        return (self._descriptor(int(self.index.file_id[r])), int(self.index.offset[r]), int(self.index.nbytes[r]),
                self.index.tensors[r])

    # ---------------------------------------------------------- reference API
    def tensors_for_expert(self, layer_id: int, expert_id: int) -> PackedExpertBatch | None:
        blk = self._block(layer_id, expert_id)
        if blk is None:
            return None
        fd, off, size, infos = blk
        storage = self._staging.get(size)
        t0 = time.monotonic()
        got = self._native_module.read_into(fd, storage, size, off)
        seconds = time.monotonic() - t0
        if got != size:
            raise OSError(f"short packed expert read: layer={layer_id} expert={expert_id}")
        views = {}
        for name, info in infos.items():
            o, n = int(info["offset"]), int(info["bytes"])
            views[name] = storage[o:o + n].view(_torch_dtype(info["source_dtype"])).reshape(
                [int(d) for d in info["source_shape"]])
        return PackedExpertBatch(views, infos, seconds, size, storage)

    def native_plan_for_expert(self, layer_id: int, expert_id: int, prefix: str,
                               parameters: list[tuple[str, torch.nn.Parameter]]) -> NativeExpertCopyPlan | None:
        r = self.index.row(layer_id, expert_id)
        if r is None:
            return None
        key = (r, tuple(name for name, _ in parameters))
        cached = self._plans.get(key)
        if cached is not None:
            return cached
        infos = self.index.tensors[r]
        found = [(i, infos.get(f"{prefix}.{name}")) for i, (name, _) in enumerate(parameters)]
        have = [(i, info) for i, info in found if info is not None]
        plan = None
        if have:
            plan = self._native_module.ExpertCopyPlan(
                [int(info["offset"]) for _, info in have],
                [parameters[i][1].numel() * parameters[i][1].element_size() for i, _ in have])
        made = NativeExpertCopyPlan(plan, tuple(i for i, _ in have),
                                    tuple(i for i, info in found if info is None))
        self._plans[key] = made
        return made

    def read_and_copy_with_plan(self, layer_id: int, expert_id: int, plan, targets: list[torch.Tensor], *,
                                non_blocking: bool):
        blk = self._block(layer_id, expert_id)
        if blk is None:
            return None
        fd, off, size, _ = blk
        staging = self._staging.get(size)
        if self.native_cuda_memcpy:
            rb, cb, rs, cs = plan.read_into_and_copy_cuda(fd, staging, size, off, targets)
        else:
            rb, cb, rs, cs = plan.read_into_and_copy(fd, staging, size, off, targets, non_blocking)
        return int(rb), int(cb), float(rs), float(cs)

    def copy_storage_to_tensors(self, storage, targets, offsets, *, non_blocking: bool) -> int:
        return int(self._native_module.copy_storage_to_tensors(storage, targets, offsets, non_blocking))

    def copy_storage_with_plan(self, plan, storage, targets, *, non_blocking: bool) -> int:
        if self.native_cuda_memcpy:
            return int(plan.copy_storage_to_tensors_cuda(storage, targets))
        return int(plan.copy_storage_to_tensors(storage, targets, non_blocking))

    # --------------------------------------------------------- B200 bulk path
    def _pread_rows(self, rows: np.ndarray, dst: torch.Tensor, dst_off: np.ndarray) -> int:
        """pread the blocks of index ``rows`` into ``dst`` at ``dst_off`` in
        pieces of at most _READ_PIECE bytes, up to ``read_threads`` pieces at
        once (positional reads of distinct ranges into distinct destinations);
        raises on a short read.  Returns the bytes read."""
        jobs = []
        for r, o in zip(rows.tolist(), dst_off.tolist()):
            size, fd, offset = int(self.index.nbytes[r]), self._descriptor(int(self.index.file_id[r])), int(
                self.index.offset[r])
            for p0 in range(0, size, _READ_PIECE):
                jobs.append((min(_READ_PIECE, size - p0), fd, offset + p0, int(o) + p0))

        def one(job) -> int:
            size, fd, offset, o = job
            got = self._native_module.read_into(fd, dst[o:o + size], size, offset)
            if got != size:
                raise RuntimeError("short packed expert read")
            return size

        if len(jobs) > 1 and self.read_threads > 1:
            if self._read_pool is None:
                self._read_pool = ThreadPoolExecutor(max_workers=self.read_threads)
            return sum(self._read_pool.map(one, jobs))
        return sum(one(j) for j in jobs)

    def read_blocks(self, layer_id: int, experts: list[int]) -> tuple[torch.Tensor, list[int], float]:
        """All blocks of ``experts`` in one (pinned when CUDA is present) host
        buffer: returns (buffer, byte offset of each block, read seconds)."""
        rows = self.index.rows_for(layer_id, experts)
        sizes = self.index.nbytes[rows]
        offs = np.concatenate([[0], np.cumsum((sizes + 255) // 256 * 256)])
        buf = torch.empty(max(int(offs[-1]), 1), dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        t0 = time.monotonic()
        nbytes = self._pread_rows(rows, buf, offs[:-1])
        dt = time.monotonic() - t0
        from .telemetry import expert_telemetry

        expert_telemetry().record_packed_read(len(experts), nbytes, dt)
        return buf, [int(o) for o in offs[:-1]], dt

    def _rings(self, device: torch.device, chunk_bytes: int) -> dict[str, Any]:
        key = (str(device), chunk_bytes)
        ring = self._upload.get(key)
        if ring is None:
            ring = {"host": [torch.empty(chunk_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)],
                    "dev": [torch.empty(chunk_bytes, dtype=torch.uint8, device=device) for _ in range(2)],
                    "copy_stream": torch.cuda.Stream(device=device),
                    "h2d_done": [torch.cuda.Event() for _ in range(2)],
                    "mat_done": [torch.cuda.Event() for _ in range(2)]}
            self._upload[key] = ring  # kept: an unsynchronised upload may still be using an older ring
        return ring

    def upload_experts(self, layer_id: int, experts: list[int], arena: ExpertArena, slots: list[int], *,
                       bf16_out: torch.Tensor | None = None, stream=None, chunk_experts: int = 8,
                       synchronize: bool = True) -> dict[str, float]:
        """Fill arena ``slots`` with ``experts`` of ``layer_id`` (bit-exact bytes
        plus scale atoms, and optionally the exact bf16 decode).

        Pipelined in chunks of ``chunk_experts`` blocks: while the host preads
        chunk i+1 into one pinned buffer, the copy stream moves chunk i to one
        device buffer (one ``cudaMemcpyAsync``) and ``stream`` runs the device
        materializer over chunk i-1 from the other.  A buffer is refilled only
        after the work that reads it has finished (events), and the
        materializer of a chunk waits for its copy.  Returns the reference's
        stats keys plus the upload's wall time and rate."""
        if len(experts) != len(slots):
            raise RuntimeError("targets and offsets length mismatch")
        if not experts:
            return {"packed_loads": 0, "packed_read_bytes": 0, "packed_read_seconds": 0.0,
                    "materialize_seconds": 0.0, "copied_bytes": 0, "upload_seconds": 0.0, "upload_gbs": 0.0}
        dev = arena.device
        rows = self.index.rows_for(layer_id, experts)
        sizes = self.index.nbytes[rows]
        stride = int(((sizes.max() + 255) // 256) * 256)
        per = max(1, min(int(chunk_experts), len(experts)))
        ring = self._rings(dev, stride * per)
        compute = stream if stream is not None else torch.cuda.current_stream(dev)
        copy_stream = ring["copy_stream"]
        read_s = 0.0
        copied = 0
        t_start = time.monotonic()
        for c, first in enumerate(range(0, len(experts), per)):
            b = c % 2
            chunk_rows = rows[first:first + per]
            n = len(chunk_rows)
            host, dbuf = ring["host"][b], ring["dev"][b]
            if c >= 2:
                ring["h2d_done"][b].synchronize()  # the copy out of this pinned buffer has finished
            t0 = time.monotonic()
            self._pread_rows(chunk_rows, host, np.arange(n, dtype=np.int64) * stride)
            read_s += time.monotonic() - t0
            with torch.cuda.stream(copy_stream):
                if c >= 2:
                    copy_stream.wait_event(ring["mat_done"][b])  # the materializer read this device buffer
                dbuf[:n * stride].copy_(host[:n * stride], non_blocking=True)
                ring["h2d_done"][b].record(copy_stream)
            compute.wait_event(ring["h2d_done"][b])
            with torch.cuda.stream(compute):
                copied += arena.materialize(dbuf, [i * stride for i in range(n)], slots[first:first + n],
                                            bf16_out=bf16_out, stream=compute)
                ring["mat_done"][b].record(compute)
        if synchronize:
            compute.synchronize()
        total_s = time.monotonic() - t_start
        nbytes = int(sizes.sum())
        from .telemetry import expert_telemetry

        expert_telemetry().record_packed_read(len(experts), nbytes, read_s)
        return {"packed_loads": len(experts), "packed_read_bytes": nbytes, "packed_read_seconds": read_s,
                "materialize_seconds": total_s - read_s, "copied_bytes": copied, "upload_seconds": total_s,
                "upload_gbs": nbytes / max(total_s, 1e-9) / 1e9}


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
