"""Build libasap.so (the sm_100a CUDA library behind asap_b200) in-tree with nvcc.

    python sgl-afd-plugin_b200/build.py [--debug]

The library is linked against the static CUDA runtime, so loading it needs no libcudart and no GPU (the
driver is resolved on the first CUDA call).  Output: sgl-afd-plugin_b200/asap_b200/libasap.so.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "asap_b200", "libasap.so")
SOURCES = ["transport.cu", "ffn.cu"]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: libasap needs the CUDA toolkit (12.8+) to build")


def build(debug: bool = False, verbose: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, n) for n in os.listdir(CSRC) if n.endswith(".cuh")]
    deps.append(os.path.join(HERE, "..", "include", "asap.h"))
    if os.path.exists(OUT) and not debug:
        newest = max(os.path.getmtime(p) for p in deps)
        if os.path.getmtime(OUT) >= newest:
            return OUT
    cmd = [nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-lineinfo",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-o", OUT + ".tmp"]
    cmd += ["-O0", "-G"] if debug else ["-O3"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += srcs
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.debug, a.verbose))
    sys.exit(0)
