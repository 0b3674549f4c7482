"""Build libmoe_fp4.so (the sm_100a CUDA library) in-tree.

    python -m moe_fused_inference_b200.build [--verbose] [--ptxas-v]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links them
into ``moe_fused_inference_b200/lib/libmoe_fp4.so``.  Objects are cached in
``moe_fused_inference_b200/_build`` and rebuilt when a source or header is
newer.  No flush-to-zero and no fast-math: the quantiser's sign rule for tiny
negatives depends on subnormal arithmetic.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(PKG, "_build")
LIB = os.path.join(LIBDIR, "libmoe_fp4.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# Shared cudart: one runtime instance per process, shared with torch (the
# same arrangement torch.utils.cpp_extension uses), so the current device and
# stream-capture state are common to both.
CUDA_LIB = os.path.join(os.path.dirname(os.path.dirname(shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")), "lib64")
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
              "-fmad=true"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libmoe_fp4.so")
    return cand


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def build(verbose: bool = False, ptxas_v: bool = False, force: bool = False) -> str:
    nvcc = _nvcc()
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_mtime = max([os.path.getmtime(h) for h in _headers()] + [0])
    objs = []
    for src in srcs:
        obj = os.path.join(OBJDIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if (not force and os.path.exists(obj)
                and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_mtime)):
            continue
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-cudart", "shared", "-I", CSRC, "-I", INCLUDE, "-c", src,
               "-o", obj]
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", "-o", LIB + ".tmp", *objs,
               "-Xlinker", f"-rpath,{CUDA_LIB}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(LIB + ".tmp", LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage per kernel")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    path = build(verbose=a.verbose, ptxas_v=a.ptxas_v, force=a.force)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
