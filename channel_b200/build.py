"""Build libchannel_b200.so (sm_100a CUDA kernels + C-ABI) in-tree with nvcc.

The shared library lands next to this file so it travels with the source tree;
nothing is installed into site-packages.  Usage: ``python -m channel_b200.build``.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "libchannel_b200.so"
OBJ = PKG / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    "-I", str(ROOT / "include"),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def build(verbose: bool = False, force: bool = False, trace: bool = False) -> Path:
    """Compile every source and link the library.  trace=True builds the
    instrumented variant (-DCH_PHASE_TRACE: per-phase timeline of the decode-step
    kernel) as libchannel_b200_trace.so, in its own object folder."""
    nvcc = _nvcc()
    obj_dir = OBJ.with_name(OBJ.name + "_trace") if trace else OBJ
    out = OUT.with_name("libchannel_b200_trace.so") if trace else OUT
    extra = ["-DCH_PHASE_TRACE"] if trace else []
    obj_dir.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + [ROOT / "include" / "channel_cuda.h"]
    newest_hdr = max(h.stat().st_mtime for h in headers)
    objs, cmds = [], []
    for src in sources():
        obj = obj_dir / (src.name + ".o")
        objs.append(obj)
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_hdr):
            continue
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if src.suffix == ".cpp":
            cmd = [nvcc, "-x", "cu", *cmd[1:]]
        cmds.append(cmd)
    # independent translation units: compile them side by side
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for cmd in cmds:
            if verbose:
                print(" ".join(cmd), flush=True)
        for f in [ex.submit(subprocess.run, cmd, check=True) for cmd in cmds]:
            f.result()
    if force or not out.exists() or out.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs), "-o", str(out),
               "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return out


def build_oracle(verbose: bool = False) -> Path:
    """Compile the CPU oracle (test infrastructure) with its Makefile."""
    oracle = ROOT / "oracle"
    subprocess.run(["make", "-s", "-C", str(oracle)], check=True,
                   stdout=None if verbose else subprocess.DEVNULL)
    return oracle / "liboracle.so"


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build(verbose=v, force="--force" in sys.argv, trace="--trace" in sys.argv))
    print(build_oracle(verbose=v))
