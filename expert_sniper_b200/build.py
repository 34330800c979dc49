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


def _flags(extra=None):
    return [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
            "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}", f"-I{CSRC}",
            "--expt-relaxed-constexpr", "-DES_BUILD_LIB", *(extra or [])]


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed: {' '.join(cmd[-3:])}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)


def build(force: bool = False, verbose: bool = False, extra=None) -> str:
    """Compile every .cu file to an object (in parallel, under _build/) and
    link them into libes_moe.so."""
    if not force and not needs_build():
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor
    obj_dir = os.path.join(PKG_DIR, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = nvcc_path()
    objs = []
    cmds = []
    for src in sources():
        obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        cmds.append([nvcc, *_flags(extra), "-c", src, "-o", obj])
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for f in [ex.submit(_run, c, verbose) for c in cmds]:
            f.result()
    _run([nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs,
          "-o", LIB_PATH + ".tmp"], verbose)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_v else None
    print(build(force=args.force or args.ptxas_v, verbose=True, extra=extra))
