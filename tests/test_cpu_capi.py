"""The C-ABI libraries load on a host without a GPU, export every entry point
the headers declare, and reject bad arguments before touching CUDA."""
import ctypes
import os
import re
import subprocess

import pytest

import fekv
from fekv import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fe_kv.h")
SHIM_HEADER = os.path.join(ROOT, "include", "fe_native_cuda.hpp")


def declared_c_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(fe_\w+)\s*\(", text, flags=re.M)))


def exported(path, demangle=False):
    args = ["nm", "-D", "--defined-only"] + (["-C"] if demangle else []) + [path]
    return subprocess.run(args, capture_output=True, text=True, check=True).stdout


def test_library_loads_and_reports_version():
    lib = fekv.load()
    assert lib.fe_abi_version() == 1
    assert _lib.status_string(0) == "ok"
    assert _lib.status_string(_lib.FE_ERR_CAPACITY) == "capacity exceeded"


def test_every_declared_function_is_exported():
    decl = declared_c_functions()
    assert len(decl) >= 15, decl
    syms = exported(_lib.LIB_PATH)
    for name in decl:
        assert re.search(rf"\bT {name}$", syms, flags=re.M), f"{name} not exported"
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes binding"
    lib = fekv.load()
    for name in decl:
        getattr(lib, name)


def test_shim_exports_reference_signatures():
    """The C++ shim keeps the reference's fe::cuda signatures
    (include/fe/native_cuda.hpp:7-10,13-15) so src/cuda_model.cpp links unchanged."""
    syms = exported(_lib.SHIM_PATH, demangle=True)
    for sig in [
        "fe::cuda::create_plan(int, int, int, int, int, int, bool, int)",
        "fe::cuda::destroy_plan(fe::cuda::AttentionPlan*)",
        "fe::cuda::prepare_plan(fe::cuda::AttentionPlan*, int const*, int const*, int const*, "
        "int const*, int, int, bool, void*)",
        "fe::cuda::attention(fe::cuda::AttentionPlan*, void*, void*, void*, void*, bool, void*)",
        "fe::cuda::store(void const*, void const*, void*, void*, long const*, int, int, bool, "
        "void*, int)",
        "fe::cuda::rope(void*, void*, long const*, float const*, int, int, int, int, bool, void*, "
        "int)",
        "fe::cuda::accept(long const*, long const*, long*, int, int, void*)",
    ]:
        assert sig in syms, sig
    ctypes.CDLL(_lib.SHIM_PATH)


def test_shim_header_compiles_standalone(tmp_path):
    src = tmp_path / "use.cpp"
    src.write_text('#include "fe_native_cuda.hpp"\n#include "fe_kv.h"\n'
                   "int main(){ return fe::cuda::create_plan == nullptr; }\n")
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                    str(src)], check=True)
    subprocess.run(["gcc", "-std=c99", "-fsyntax-only", "-x", "c", HEADER], check=True)


def test_argument_errors_without_gpu():
    lib = fekv.load()
    p = ctypes.c_void_p(16)
    # bad dtype, bad width: rejected before any CUDA call
    assert lib.fe_kv_append(p, p, p, p, p, 1, 1024, 7, 16, None) == _lib.FE_ERR_INVALID_ARGUMENT
    assert lib.fe_kv_append(p, p, p, p, p, 1, 1020, 1, 16, None) == _lib.FE_ERR_UNSUPPORTED
    assert lib.fe_kv_append(None, p, p, p, p, 1, 1024, 1, 16, None) == _lib.FE_ERR_INVALID_ARGUMENT
    assert lib.fe_kv_append(p, p, p, p, p, 0, 1024, 1, 16, None) == _lib.FE_OK  # nothing to do
    assert "null" in _lib.last_error() or _lib.last_error() != ""
    arr = (ctypes.c_void_p * 1)(16)
    assert lib.fe_kv_copy_blocks(arr, arr, 129, p, p, p, 1, 16, 1024, 4, 1, None) == \
        _lib.FE_ERR_INVALID_ARGUMENT
    out = ctypes.c_void_p()
    assert lib.fe_attn_plan_create(8, 2, 64, 16, 4, 4, 1, 8, ctypes.byref(out)) == \
        _lib.FE_ERR_UNSUPPORTED
    assert lib.fe_attn_plan_create(8, 3, 128, 16, 4, 4, 1, 8, ctypes.byref(out)) == \
        _lib.FE_ERR_UNSUPPORTED
    assert lib.fe_attn_plan_create(8, 2, 128, 8, 4, 4, 1, 8, ctypes.byref(out)) == \
        _lib.FE_ERR_UNSUPPORTED


def test_plan_create_without_gpu_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    with pytest.raises(fekv.FeError) as e:
        fekv.AttentionPlan(8, 2, 128, 16, 4, 4, True, 8)
    assert e.value.status in (_lib.FE_ERR_CUDA, _lib.FE_ERR_NO_DEVICE)
