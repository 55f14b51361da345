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


REFERENCE_ROOT = os.environ.get("FE_REFERENCE_ROOT",
                                os.path.join(os.path.dirname(ROOT), "reference"))


def _torch_includes():
    torch = pytest.importorskip("torch")
    troot = os.path.dirname(torch.__file__)
    return troot, int(torch._C._GLIBCXX_USE_CXX11_ABI)


@pytest.mark.skipif(not os.path.exists(os.path.join(REFERENCE_ROOT, "src", "cuda_model.cpp")),
                    reason="reference source tree not present")
def test_reference_cuda_model_compiles_against_shim_header(tmp_path):
    """The reference's CUDA DeviceModel (src/cuda_model.cpp), unmodified,
    type-checks against this library's fe::cuda header. Its own
    include/fe/native_cuda.hpp is replaced by a stand-in that includes
    include/fe_native_cuda.hpp and declares the two operators that stay in
    the reference's src/cuda_kernels.cu (norm and silu_mul, copied from
    include/fe/native_cuda.hpp:11-12)."""
    troot, abi = _torch_includes()
    stand_in = tmp_path / "fe"
    stand_in.mkdir()
    (stand_in / "native_cuda.hpp").write_text(
        "#pragma once\n#include \"fe_native_cuda.hpp\"\nnamespace fe::cuda {\n"
        "void norm(const void* x,const void* residual,const void* weight,void* output,"
        "void* new_residual,int rows,int width,float eps,bool bf16,void* stream);\n"
        "void silu_mul(const void* gu,void* output,int rows,int width,bool bf16,void* stream);\n}\n")
    # the reference's headers need nlohmann/json; the wheel's cuDNN frontend
    # carries a copy of it
    json_dir = os.path.join(os.path.dirname(troot), "include", "cudnn_frontend", "thirdparty")
    if not os.path.exists(os.path.join(json_dir, "nlohmann", "json.hpp")):
        pytest.skip("no nlohmann/json.hpp for the reference's headers")
    cmd = ["g++", "-std=c++20", "-fsyntax-only", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", str(tmp_path), "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(REFERENCE_ROOT, "include"), "-I", json_dir,
           "-I", os.path.join(troot, "include"),
           "-I", os.path.join(troot, "include", "torch", "csrc", "api", "include"),
           "-I", "/usr/local/cuda/include", os.path.join(REFERENCE_ROOT, "src", "cuda_model.cpp")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]


@pytest.mark.skipif(not os.path.exists(os.path.join(REFERENCE_ROOT, "include", "fe",
                                                    "native_cuda.hpp")),
                    reason="reference source tree not present")
def test_reference_header_links_against_shim(tmp_path):
    """A caller compiled against the reference's own include/fe/native_cuda.hpp
    links against the shim: every operator of this path it declares
    (create_plan, destroy_plan, prepare_plan, attention, rope, store, accept)
    resolves to a shim symbol."""
    src = tmp_path / "caller.cpp"
    src.write_text(
        "#include \"fe/native_cuda.hpp\"\n"
        "int main(int argc, char**){\n"
        "  if (argc < 100) return 0;\n"
        "  auto* p = fe::cuda::create_plan(8,2,128,16,1,2,true,4);\n"
        "  fe::cuda::prepare_plan(p,nullptr,nullptr,nullptr,nullptr,0,0,false,nullptr);\n"
        "  fe::cuda::attention(p,nullptr,nullptr,nullptr,nullptr,true,nullptr);\n"
        "  fe::cuda::rope(nullptr,nullptr,nullptr,nullptr,0,0,0,0,true,nullptr,0);\n"
        "  fe::cuda::store(nullptr,nullptr,nullptr,nullptr,nullptr,0,0,true,nullptr,0);\n"
        "  fe::cuda::accept(nullptr,nullptr,nullptr,0,0,nullptr);\n"
        "  fe::cuda::destroy_plan(p);\n  return 1;\n}\n")
    libdir = os.path.dirname(_lib.SHIM_PATH)
    cmd = ["g++", "-std=c++17", "-I", os.path.join(REFERENCE_ROOT, "include"), str(src),
           "-o", str(tmp_path / "caller"), "-L", libdir, "-lfe_native_cuda_b200",
           "-lfe_kv_b200", f"-Wl,-rpath,{libdir}", "-Wl,--no-undefined"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
