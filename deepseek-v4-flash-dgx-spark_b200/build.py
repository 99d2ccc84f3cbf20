"""Build libdsv4moe.so (sm_100a) in-tree with nvcc.

    python deepseek-v4-flash-dgx-spark_b200/build.py [--force]

The shared libraries land in deepseek-v4-flash-dgx-spark_b200/lib/:
libdsv4moe.so (the C ABI, loaded by spark_b200._lib through ctypes) and
libdsv4moe_torch.so (the TORCH_LIBRARY(dsv4moe) op layer over it, loaded by
spark_b200.ops with torch.ops.load_library).  nvcc cross-compiles for sm_100a on
a machine without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "lib"
LIB = LIB_DIR / "libdsv4moe.so"
TORCH_OPS_LIB = LIB_DIR / "libdsv4moe_torch.so"
INCLUDE = REPO / "include"

SOURCES = ["dsv4moe.cu", "loader.cpp"]
DEPS = ["gate.cu", "route.cu", "expert_gemm.cu", "expert_gemm_pair.cu", "materialize.cu", "capi.cu", "no_alloc.cu", "gate_gemm.cu", "ep.cu", "sparse_attn.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + DEPS] + list(CSRC.glob("*.cuh")) + [INCLUDE / "dsv4moe.h", Path(__file__)]
    return any(p.stat().st_mtime > mtime for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = PKG_DIR / "_build"
    obj_dir.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in SOURCES:
        obj = obj_dir / (src + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(CSRC / src), "-o", str(obj)]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(str(obj))
    logs = []
    for src, p in procs:
        out, _ = p.communicate()
        logs.append(f"== {src}\n{out}")
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{out}")
    (obj_dir / "ptxas.log").write_text("\n".join(logs))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", str(tmp)]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print("\n".join(logs))
    return LIB


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    import torch.utils.cpp_extension as ext

    inc = [f"-I{p}" for p in ext.include_paths()] + [f"-I{Path(nvcc()).parent.parent / 'include'}"]
    libs = [f"-L{p}" for p in ext.library_paths()] + [f"-Wl,-rpath,{p}" for p in ext.library_paths()]
    abi = int(torch.compiled_with_cxx11_abi())
    return inc + [f"-D_GLIBCXX_USE_CXX11_ABI={abi}"], libs + ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
                                                              "-ltorch_cuda"]


def build_torch_ops(force: bool = False) -> Path:
    """libdsv4moe_torch.so: the TORCH_LIBRARY(dsv4moe) op layer (csrc/torch_ops.cpp)
    over libdsv4moe.so, compiled with g++ against the installed torch headers
    (no CUDA code of its own) and loaded with torch.ops.load_library."""
    src = CSRC / "torch_ops.cpp"
    lib = build(force)
    if not force and TORCH_OPS_LIB.exists() and TORCH_OPS_LIB.stat().st_mtime > max(
            src.stat().st_mtime, lib.stat().st_mtime, (INCLUDE / "dsv4moe.h").stat().st_mtime,
            Path(__file__).stat().st_mtime):
        return TORCH_OPS_LIB
    cflags, ldflags = _torch_flags()
    tmp = TORCH_OPS_LIB.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", *cflags, f"-I{INCLUDE}",
           str(src), "-o", str(tmp), f"-L{LIB_DIR}", "-ldsv4moe", "-Wl,-rpath,$ORIGIN", *ldflags]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed on torch_ops.cpp:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, TORCH_OPS_LIB)
    return TORCH_OPS_LIB


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
    print(build_torch_ops(force="--force" in sys.argv))
