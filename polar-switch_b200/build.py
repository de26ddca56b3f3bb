"""Build libpolarswitch_b200.so (sm_100a) in-tree with nvcc.

Usage: python polar-switch_b200/build.py [--force] [--verbose]

The library lands in polar-switch_b200/polar_switch/_lib/ so that it travels
with the source tree; nothing is installed into site-packages.
"""

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "polar_switch", "_lib")
LIB_NAME = "libpolarswitch_b200.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)
HEADER = os.path.join(ROOT, "include", "polar_switch_b200.h")
SOURCES = [os.path.join(CSRC, "ps_capi.cu")]
# Every header under csrc/ is included by ps_capi.cu; a change to any of them rebuilds.
DEPENDS = SOURCES + sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")) + [HEADER]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-Wall",
    "-shared", "--expt-relaxed-constexpr",
]


def nvcc_path():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or put CUDA 12.8+ on PATH")
    return cand


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(p) <= t for p in DEPENDS)


def build(force=False, verbose=False, extra_flags=()):
    """Compile the C-ABI library for sm_100a unless it is already current."""
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, *extra_flags, "-o", tmp, *SOURCES]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    flags = ["-Xptxas", "-v"] if a.ptxas_info else []
    path = build(force=a.force or a.ptxas_info, verbose=a.verbose, extra_flags=flags)
    print(path)
    sys.exit(0)
