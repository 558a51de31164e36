"""Build libggmlc_b200.so in-tree (ggmlc_b200/libggmlc_b200.so) with nvcc for sm_100a.

    python -m ggmlc_b200.build [--force]

Objects go to ggmlc_b200/_build/; a source is recompiled when it or any header in csrc/ is
newer than its object.  The shared library links the CUDA runtime statically so it loads in
any process of this image (with or without torch).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libggmlc_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (CUDA 12.9 toolkit required to build ggmlc_b200)")
    return cand


def _flags(src: Path) -> list[str]:
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-lineinfo", "-I", str(CSRC),
              "-I", str(PKG.parent / "include")]
    if src.suffix == ".cu":
        return common + ARCH + ["--expt-relaxed-constexpr", "-Xptxas", "-O3"]
    return common + ARCH


def _compile(src: Path) -> Path:
    obj = BUILD / (src.name + ".o")
    cmd = [nvcc(), "-c", str(src), "-o", str(obj)] + _flags(src)
    if src.suffix != ".cu":
        cmd += ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted([p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp")])
    headers = [p for p in CSRC.iterdir() if p.suffix in (".h", ".cuh")]
    headers.append(PKG.parent / "include" / "ggmlc_b200.h")
    newest_header = max(h.stat().st_mtime for h in headers)
    todo = []
    for s in sources:
        obj = BUILD / (s.name + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, newest_header):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for obj in ex.map(_compile, todo):
                if verbose:
                    print("compiled", obj.name)
    objs = [BUILD / (s.name + ".o") for s in sources]
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), "-shared", "-o", str(tmp)] + [str(o) for o in objs] + ARCH + [
            "-Xlinker", "--no-undefined", "-lcuda", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    build_bench_tool(force)
    return LIB


TOOL_SRC = PKG / "tools" / "ggmlc_bench.cpp"
TOOL = PKG / "ggmlc-bench"


def build_bench_tool(force: bool = False) -> Path:
    """ggmlc_b200/ggmlc-bench: the reference's benchmark CLI over the C ABI (host C++ only)."""
    if not force and TOOL.exists() and TOOL.stat().st_mtime >= max(
            TOOL_SRC.stat().st_mtime, LIB.stat().st_mtime):
        return TOOL
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-o", str(TOOL), str(TOOL_SRC), "-I",
           str(PKG.parent / "include"), "-L", str(PKG), "-lggmlc_b200", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ggmlc-bench build failed:\n{r.stdout}\n{r.stderr}")
    return TOOL


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
