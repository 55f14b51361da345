"""Build the sm_100a paged-KV libraries in-tree with nvcc.

Outputs (git-ignored, shipped with the source snapshot):
  flashengine.cpp_b200/lib/libfe_kv_b200.so          C ABI (include/fe_kv.h)
  flashengine.cpp_b200/lib/libfe_native_cuda_b200.so C++ shim with the
      reference's fe::cuda::{create_plan, destroy_plan, prepare_plan,
      attention, store} signatures (include/fe_native_cuda.hpp)

nvcc cross-compiles for sm_100a on a host without a GPU. Run directly:
``python flashengine.cpp_b200/build.py [--force] [--verbose]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(PKG, "_build")

LIB_KV = os.path.join(LIBDIR, "libfe_kv_b200.so")
LIB_SHIM = os.path.join(LIBDIR, "libfe_native_cuda_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-Xptxas", "-v"] + ARCH
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra"]

KV_SOURCES = ["fe_kv_ops.cu", "fe_attn.cu", "fe_decode.cu", "fe_prefill_tc.cu", "fe_rope_accept.cu",
              "fe_plan_device.cu", "fe_attn_plan.cpp", "fe_kv_fork.cpp"]
SHIM_SOURCES = ["fe_native_cuda_shim.cpp"]
HEADERS = ["fe_common.cuh", "fe_attn_common.cuh", "fe_attn_plan.h", "fe_tcgen05.cuh"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found")


def cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc())))


def _deps(src: str) -> list[str]:
    deps = [os.path.join(CSRC, src)] + [os.path.join(CSRC, h) for h in HEADERS]
    deps += [os.path.join(INCLUDE, h) for h in os.listdir(INCLUDE)]
    return deps


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.splitext(src)[0] + ".o")
    if not force and not _stale(obj, _deps(src)):
        return obj
    path = os.path.join(CSRC, src)
    if src.endswith(".cu"):
        cmd = [nvcc()] + NVCC_FLAGS + ["-I", INCLUDE, "-I", CSRC, "-c", path, "-o", obj]
    else:
        cmd = ["g++"] + CXX_FLAGS + ["-I", INCLUDE, "-I", CSRC,
                                     "-I", os.path.join(cuda_home(), "include"), "-c", path, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    log = os.path.join(OBJDIR, os.path.splitext(src)[0] + ".ptxas.txt")
    with open(log, "w") as f:
        f.write(res.stdout + res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> tuple[str, str]:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=4) as ex:
        kv_objs = list(ex.map(lambda s: _compile(s, force, verbose), KV_SOURCES))
        shim_objs = list(ex.map(lambda s: _compile(s, force, verbose), SHIM_SOURCES))
    if force or _stale(LIB_KV, kv_objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB_KV] + kv_objs + [
            "-Xlinker", "-soname=libfe_kv_b200.so"]
        subprocess.run(cmd, check=True)
    if force or _stale(LIB_SHIM, shim_objs + [LIB_KV]):
        cmd = ["g++", "-shared", "-o", LIB_SHIM] + shim_objs + [
            "-L", LIBDIR, "-lfe_kv_b200", "-Wl,-rpath,$ORIGIN"]
        subprocess.run(cmd, check=True)
    return LIB_KV, LIB_SHIM


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    for p in build(a.force, a.verbose):
        print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
