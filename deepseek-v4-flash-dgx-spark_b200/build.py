"""Build libdsv4moe.so (sm_100a) in-tree with nvcc.

    python deepseek-v4-flash-dgx-spark_b200/build.py [--force]

The shared library lands in deepseek-v4-flash-dgx-spark_b200/lib/ and is
loaded by spark_b200._lib through ctypes.  nvcc cross-compiles for sm_100a on
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
INCLUDE = REPO / "include"

SOURCES = ["dsv4moe.cu", "loader.cpp"]
DEPS = ["gate.cu", "route.cu", "expert_gemm.cu", "expert_gemm_pair.cu", "materialize.cu", "capi.cu", "no_alloc.cu", "gate_gemm.cu", "ep.cu"]
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


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
