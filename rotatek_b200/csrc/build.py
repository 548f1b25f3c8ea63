"""Build librotatek_b200.so (the C-ABI library) for sm_100a with nvcc.

    python -m rotatek_b200.csrc.build [--verbose]

The library lands next to the package (rotatek_b200/librotatek_b200.so) so a
snapshot of the source tree carries it.  The CUDA runtime is linked
statically: the library does not depend on which libcudart the host process
(e.g. torch) has loaded.  cuTensorMapEncodeTiled is resolved at run time
through cudaGetDriverEntryPointByVersion, so there is no -lcuda.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

CSRC = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(CSRC)
REPO = os.path.dirname(PKG)
LIB_NAME = "librotatek_b200.so"
SOURCES = ["capi.cu", "decode_tc.cu", "decode_simt.cu", "decode_static.cu", "quant_fp8.cu", "spark_pack.cu", "cov_tc.cu", "kproj_tc.cu", "eigen.cu",
           "rotate.cu", "selftest.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def build(verbose: bool = False, out_dir: str = PKG) -> str:
    out = os.path.join(out_dir, LIB_NAME)
    obj_dir = os.path.join(REPO, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                    "--expt-relaxed-constexpr", "-I", os.path.join(REPO, "include")]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        obj = os.path.join(obj_dir, src.replace(".cu", ".o"))
        cmd = [nvcc()] + flags + ["-c", os.path.join(CSRC, src), "-o", obj]
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = out + ".tmp"
    subprocess.run([nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs, check=True)
    os.replace(tmp, out)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="print ptxas register / smem usage")
    args = ap.parse_args()
    print(build(verbose=args.verbose))


if __name__ == "__main__":
    sys.exit(main())
