"""Builds libmbp.so (the C-ABI CUDA library) in-tree for sm_100a.

    python muse-bf16-proj_b200/build.py            # incremental
    python muse-bf16-proj_b200/build.py --force    # rebuild everything

Each ``csrc/*.cu`` is compiled by nvcc with ``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into
``_build/`` (ptxas register/spill report in ``_build/<name>.ptxas.txt``), then linked against the shared CUDA
runtime (so the library shares the runtime -- current device, streams -- with PyTorch in the same process)
into ``mbp/libmbp.so``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "mbp", "libmbp.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr", "-Xptxas", "-v", f"-I{INCLUDE}", "-cudart", "shared"]


def nvcc() -> str:
    for cand in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def compile_one(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, src[:-3] + ".o")
    srcp = os.path.join(CSRC, src)
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(srcp), headers_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", srcp, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    with open(os.path.join(BUILD, src[:-3] + ".ptxas.txt"), "w") as f:
        f.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr[-6000:]}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force), srcs))
    if force or not os.path.exists(OUT) or os.path.getmtime(OUT) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-o", OUT, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr[-4000:]}")
    if verbose:
        print(OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    try:
        build(a.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
