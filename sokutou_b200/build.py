"""Build the sokutou_b200 shared library (sm_100a) in-tree: sokutou_b200/lib/libsokutou_b200.so, and
the bounds-checked variant sokutou_b200/lib/libsokutou_b200_checked.so (every guarded shared, tensor
and global memory index tested before its access; failures land in the device error word as
SK_DEVERR_BOUNDS — the sanitizer substitute for this pool).

    python -m sokutou_b200.build [--force] [--verbose] [--checked]

nvcc cross-compiles without a GPU. The library links only the CUDA runtime (static); the tensor-map
encoder of the driver is looked up at run time, so no libcuda is needed at link time.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
ROOT = os.path.dirname(PKG)
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libsokutou_b200.so")
LIB_CHECKED = os.path.join(LIB_DIR, "libsokutou_b200_checked.so")
SOURCES = ["api.cu", "decode_attn.cu", "dit_prologue.cu", "dit_attn_f32.cu", "dit_attn_tc.cu", "dit_gate.cu",
           "dit_linear.cu", "decode_block.cu"]
HEADERS = ["sk_common.cuh", "dit_qk_math.cuh", "dit_attn_tc.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def _stamp(extra: list[str]) -> str:
    h = hashlib.sha256()
    for f in SOURCES + HEADERS:
        with open(os.path.join(CSRC, f), "rb") as fh:
            h.update(fh.read())
    with open(os.path.join(ROOT, "include", "sokutou_b200.h"), "rb") as fh:
        h.update(fh.read())
    h.update(" ".join(FLAGS + extra).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False, checked: bool = False) -> str:
    """Compile (when sources changed) and return the library path; checked=True: the bounds-checked one."""
    os.makedirs(LIB_DIR, exist_ok=True)
    lib = LIB_CHECKED if checked else LIB
    extra = ["-DSK_BOUNDS_CHECK=1"] if checked else []
    stamp_file = lib + ".stamp"
    stamp = _stamp(extra)
    if not force and os.path.exists(lib) and os.path.exists(stamp_file):
        with open(stamp_file) as fh:
            if fh.read().strip() == stamp:
                return lib
    objs = []
    for src in SOURCES:
        obj = os.path.join(LIB_DIR, ("checked_" if checked else "") + src.replace(".cu", ".o"))
        cmd = [NVCC, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = lib + ".tmp"
    subprocess.run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static", *objs,
                    "-o", tmp], check=True)
    os.replace(tmp, lib)
    for o in objs:
        os.remove(o)
    with open(stamp_file, "w") as fh:
        fh.write(stamp)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--checked", action="store_true", help="build the bounds-checked variant")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.checked))
    sys.exit(0)
