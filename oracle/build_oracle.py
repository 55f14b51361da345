"""Build recipe for the CPU checkers (test infrastructure only).

* ``oracle/libfe_oracle.so``  — the plain-C restatement, ``oracle/fe_oracle.c``.
* ``oracle/_ref/libfe_ref_aten.so`` — the reference's own ATen path
  (FlashEngine.cpp ``src/portable_gpu_ops.cpp``), compiled unmodified from the
  reference source tree through ``oracle/ref_aten_wrap.cpp`` and linked against
  the CPU LibTorch that ships with the PyTorch wheel. Built only where the
  reference tree exists (it is not present on the GPU box, which uses the
  prebuilt file that travels with the repository snapshot).
* ``oracle/_ref/libfe_ref_cuda.so`` — the reference's own CUDA kernels
  (``src/cuda_kernels.cu``: rope, store, accept) for sm_100a through
  ``oracle/ref_cuda_wrap.cu``; the GPU tests run them as the comparator for the
  fused RoPE+append and accept kernels. Built the same way (reference tree
  only; the GPU box uses the prebuilt file).
* ``oracle/_ref/libfe_ref_flashinfer.so`` — the reference's own CUDA attention
  (``src/flashinfer_attention.cu`` over the FlashInfer headers installed with
  the flashinfer wheel) for sm_100a through ``oracle/ref_flashinfer_wrap.cu``:
  the GPU comparator for decode and verify attention. Built the same way.

The reference tree is looked up in ``$FE_REFERENCE_ROOT``, else in a
``reference`` directory beside this repository's root.

Run directly: ``python oracle/build_oracle.py [--reference-root DIR]``.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(HERE)
DEFAULT_REFERENCE_ROOT = os.environ.get(
    "FE_REFERENCE_ROOT", os.path.join(os.path.dirname(REPO_ROOT), "reference"))

C_ORACLE_SRC = os.path.join(HERE, "fe_oracle.c")
C_ORACLE_LIB = os.path.join(HERE, "libfe_oracle.so")
REF_WRAP_SRC = os.path.join(HERE, "ref_aten_wrap.cpp")
REF_DIR = os.path.join(HERE, "_ref")
REF_LIB = os.path.join(REF_DIR, "libfe_ref_aten.so")
REF_CUDA_WRAP_SRC = os.path.join(HERE, "ref_cuda_wrap.cu")
REF_CUDA_LIB = os.path.join(REF_DIR, "libfe_ref_cuda.so")
REF_FI_WRAP_SRC = os.path.join(HERE, "ref_flashinfer_wrap.cu")
REF_FI_LIB = os.path.join(REF_DIR, "libfe_ref_flashinfer.so")


def _stale(target: str, *sources: str) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.exists(s))


def build_c_oracle(force: bool = False) -> str:
    if force or _stale(C_ORACLE_LIB, C_ORACLE_SRC):
        cmd = ["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fPIC", "-shared", "-Wall", "-Wextra",
               C_ORACLE_SRC, "-o", C_ORACLE_LIB, "-lm"]
        subprocess.run(cmd, check=True)
    return C_ORACLE_LIB


def reference_source(reference_root: str = DEFAULT_REFERENCE_ROOT) -> str:
    return os.path.join(reference_root, "src", "portable_gpu_ops.cpp")


def build_reference(reference_root: str = DEFAULT_REFERENCE_ROOT, force: bool = False) -> str | None:
    """Compile the reference ATen path for the CPU. Returns the library path,
    or None when the reference tree is absent (e.g. on the GPU box)."""
    src = reference_source(reference_root)
    if not os.path.exists(src):
        return REF_LIB if os.path.exists(REF_LIB) else None
    if not (force or _stale(REF_LIB, REF_WRAP_SRC, src)):
        return REF_LIB
    import torch  # only for its include and library paths

    troot = os.path.dirname(torch.__file__)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    os.makedirs(REF_DIR, exist_ok=True)
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", os.path.join(reference_root, "include"),
           "-I", os.path.join(troot, "include"),
           "-I", os.path.join(troot, "include", "torch", "csrc", "api", "include"),
           REF_WRAP_SRC, "-o", REF_LIB,
           "-L", os.path.join(troot, "lib"), "-ltorch_cpu", "-lc10",
           f"-Wl,-rpath,{os.path.join(troot, 'lib')}"]
    subprocess.run(cmd, check=True)
    return REF_LIB


def build_reference_cuda(reference_root: str = DEFAULT_REFERENCE_ROOT,
                         force: bool = False) -> str | None:
    """Compile the reference's CUDA kernels (src/cuda_kernels.cu) for sm_100a
    with nvcc (no GPU needed to build). None when the tree is absent."""
    src = os.path.join(reference_root, "src", "cuda_kernels.cu")
    if not os.path.exists(src):
        return REF_CUDA_LIB if os.path.exists(REF_CUDA_LIB) else None
    if not (force or _stale(REF_CUDA_LIB, REF_CUDA_WRAP_SRC, src)):
        return REF_CUDA_LIB
    os.makedirs(REF_DIR, exist_ok=True)
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
           "-Xcompiler", "-fPIC", "-shared", "-I", os.path.join(reference_root, "include"),
           REF_CUDA_WRAP_SRC, "-o", REF_CUDA_LIB]
    subprocess.run(cmd, check=True)
    return REF_CUDA_LIB


def flashinfer_include() -> str | None:
    """The C++ headers shipped inside the flashinfer wheel (flashinfer/data)."""
    try:
        import importlib.util

        spec = importlib.util.find_spec("flashinfer")
    except Exception:
        return None
    if spec is None or not spec.submodule_search_locations:
        return None
    data = os.path.join(list(spec.submodule_search_locations)[0], "data")
    ok = os.path.exists(os.path.join(data, "include", "flashinfer", "attention", "prefill.cuh"))
    return data if ok else None


def build_reference_flashinfer(reference_root: str = DEFAULT_REFERENCE_ROOT,
                               force: bool = False) -> str | None:
    """Compile the reference's FlashInfer attention (src/flashinfer_attention.cu)
    for sm_100a. None when the tree or the FlashInfer headers are absent."""
    src = os.path.join(reference_root, "src", "flashinfer_attention.cu")
    data = flashinfer_include()
    if not os.path.exists(src) or data is None:
        return REF_FI_LIB if os.path.exists(REF_FI_LIB) else None
    if not (force or _stale(REF_FI_LIB, REF_FI_WRAP_SRC, src)):
        return REF_FI_LIB
    os.makedirs(REF_DIR, exist_ok=True)
    # the reference's own CUDA flags (CMakeLists.txt: --expt-relaxed-constexpr,
    # --extended-lambda, C++17), for sm_100a
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
           "--expt-relaxed-constexpr", "--extended-lambda", "-Xcompiler", "-fPIC", "-shared",
           "-I", os.path.join(reference_root, "include"), "-I", os.path.join(data, "include"),
           "-I", os.path.join(data, "cutlass", "include"), "-I", os.path.join(data, "spdlog", "include"),
           REF_FI_WRAP_SRC, "-o", REF_FI_LIB, "-Xlinker", "-Bsymbolic"]
    subprocess.run(cmd, check=True)
    return REF_FI_LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=DEFAULT_REFERENCE_ROOT)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    print(build_c_oracle(a.force))
    print(build_reference(a.reference_root, a.force))
    print(build_reference_cuda(a.reference_root, a.force))
    print(build_reference_flashinfer(a.reference_root, a.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
