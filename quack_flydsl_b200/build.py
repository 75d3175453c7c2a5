"""Ahead-of-time build of libquack_b200.so with nvcc for sm_100a.

Replaces the reference's JIT compile + on-disk cache path (quack/cache/jit.py:160-341): there is
nothing to compile at run time.  Usage: ``python -m quack_flydsl_b200.build [--force]``.
The library is built in-tree (``quack_flydsl_b200/lib/libquack_b200.so``) so that it travels with
the source tree; objects go to ``quack_flydsl_b200/build/``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
OBJ_DIR = PKG_DIR / "build"
LIB_DIR = PKG_DIR / "lib"
LIB_NAME = "libquack_b200.so"

SOURCES = ["api.cu", "norm_fwd.cu", "norm_fwd_stream.cu", "norm_bwd.cu", "norm_bwd_ring.cu", "norm_bwd_static.cu",
           "softmax.cu", "softmax_ring.cu", "softmax_cluster.cu", "cross_entropy.cu", "rms_final_reduce.cu", "topk.cu", "peer_reduce.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC"]


def lib_path(tag: str = "") -> Path:
    """Path of the shared library; ``tag`` names an experimental variant (e.g. cache policy)."""
    name = LIB_NAME if not tag else LIB_NAME.replace(".so", f"_{tag}.so")
    return LIB_DIR / name


def _nvcc() -> str:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        raise RuntimeError("nvcc not found; CUDA 12.8+ with sm_100a support is required")
    return nvcc


def _newest_mtime(paths) -> float:
    return max(p.stat().st_mtime for p in paths)


def _deps() -> list:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _compile_one(nvcc: str, src: Path, obj: Path, defines: list, verbose: bool) -> str:
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *defines, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src),
           "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas")
        cmd.insert(2, "-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(force: bool = False, tag: str = "", defines: list | None = None, verbose: bool = False) -> Path:
    """Compiles every CUDA source for sm_100a and links the shared library.  Returns its path."""
    defines = list(defines or [])
    out = lib_path(tag)
    srcs = [CSRC / s for s in SOURCES]
    if not force and out.exists() and out.stat().st_mtime >= _newest_mtime(srcs + _deps()):
        return out
    nvcc = _nvcc()
    obj_dir = OBJ_DIR / (tag or "default")
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objs = [obj_dir / (s.stem + ".o") for s in srcs]
    dep_mtime = _newest_mtime(_deps())
    jobs = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        for src, obj in zip(srcs, objs):
            fresh = obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, dep_mtime)
            if force or not fresh:
                jobs.append(pool.submit(_compile_one, nvcc, src, obj, defines, verbose))
        for j in jobs:
            log = j.result()
            if verbose and log:
                print(log, file=sys.stderr)
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true", help="rebuild even if up to date")
    ap.add_argument("--tag", default="", help="suffix of an experimental library variant")
    ap.add_argument("-D", dest="defines", action="append", default=[],
                    help="extra preprocessor define, e.g. -D QB_LDG_MOD='\".L1::no_allocate\"'")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    args = ap.parse_args()
    defines = [f"-D{d}" for d in args.defines]
    print(build(force=args.force, tag=args.tag, defines=defines, verbose=args.verbose))


if __name__ == "__main__":
    main()
