"""Build libmsgl.so in-tree for sm_100a (B200).

    python mini-sglang-cpp_b200/build.py [--force] [--verbose]

Every CUDA source is compiled by nvcc with -gencode arch=compute_100a,code=sm_100a into
_build/, the C++ engine sources with the same nvcc (host compiler g++), and all objects are
linked into mini-sglang-cpp_b200/libmsgl.so (cudart linked statically; NCCL dynamically).
Objects are rebuilt when a source or any header is newer than the object.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
ENGINE = os.path.join(PKG, "engine")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libmsgl.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-I" + os.path.join(ROOT, "include")]
CUFLAGS = ARCH + COMMON + ["-lineinfo", "--expt-relaxed-constexpr"]


def _headers():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    hs += glob.glob(os.path.join(ENGINE, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _stale(obj, src, headers):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *headers])


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if src.endswith(".cu"):
        cmd = [NVCC, *CUFLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd += ["-Xptxas", "-v"]
    else:
        cmd = [NVCC, *ARCH, *COMMON, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, obj, r


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(ENGINE, "*.cpp")))
    headers = _headers()
    todo = [s for s in srcs if force or _stale(os.path.join(BUILD, os.path.basename(s) + ".o"), s, headers)]
    objs = [os.path.join(BUILD, os.path.basename(s) + ".o") for s in srcs]
    failed = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for src, obj, r in ex.map(lambda s: _compile(s, verbose), todo):
                if r.returncode != 0:
                    failed.append((src, r.stderr))
                elif verbose and r.stderr:
                    sys.stderr.write(r.stderr)
    if failed:
        for src, err in failed:
            sys.stderr.write(f"--- {src}\n{err}\n")
        raise RuntimeError(f"nvcc failed on {len(failed)} file(s)")
    if todo or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lnccl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
