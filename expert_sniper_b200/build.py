"""Build the CUDA library (libes_moe.so) in-tree with nvcc for sm_100a.

    python -m expert_sniper_b200.build          # build if sources changed
    python -m expert_sniper_b200.build --force  # rebuild

The library is a plain C-ABI shared object (include/es_moe.h) with no
dependency on torch; Python reaches it through ctypes.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_NAME = "libes_moe.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libes_moe.so")
    return p


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _inputs():
    files = sources()
    files += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    files += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    files.append(os.path.abspath(__file__))
    return files


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force: bool = False, verbose: bool = False, extra=None) -> str:
    if not force and not needs_build():
        return LIB_PATH
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr",
           "-DES_BUILD_LIB", *(extra or []), *sources(), "-o", LIB_PATH + ".tmp"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed building {LIB_NAME}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_v else None
    print(build(force=args.force or args.ptxas_v, verbose=True, extra=extra))
