"""The C++ drop-in shim (libfe_native_cuda_b200.so, include/fe_native_cuda.hpp)
on the GPU: the reference DeviceModel's operator sequence (create_plan,
prepare_plan with host metadata, rope, store, attention, accept,
destroy_plan: Cambridgebit/FlashEngine.cpp src/cuda_model.cpp:94-96,118-140,184)
run through the shim's fe::cuda functions, checked against the CPU oracle:

* in this process, through the shim's exported C++ symbols (no exception can
  be raised on this path);
* in a small C++ program (tests/shim/shim_step.cpp) built against the shim
  header, which also checks that invalid calls raise std::runtime_error as
  the reference's check() does (src/cuda_kernels.cu:10).

Cases: C1 (hq16/hkv8 fp16, 4 sequences) and one C2 layer (hq32/hkv8 bf16,
64 sequences, contexts 512-4096)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import oracle
from fe_testutil import compare_attention

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER_SRC = os.path.join(ROOT, "tests", "shim", "shim_step.cpp")


def _rope_cache(max_positions, dim, theta=1.0e6):
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
    ang = np.arange(max_positions, dtype=np.float64)[:, None] * inv[None, :]
    return np.concatenate([np.cos(ang), np.sin(ang)], 1).astype(np.float32)


def _case(name):
    from fekv import workloads
    w = workloads.c1(seed=0) if name == "c1" else workloads.c2(seed=0)
    md = w.metadata()
    rng = np.random.default_rng(21)
    inp = {
        "kpool": workloads.random_bits(rng, (w.cache_slots, w.width), w.bf16, w.scale),
        "vpool": workloads.random_bits(rng, (w.cache_slots, w.width), w.bf16, w.scale),
        "knew": workloads.random_bits(rng, (md.rows, w.width), w.bf16, w.scale),
        "vnew": workloads.random_bits(rng, (md.rows, w.width), w.bf16, w.scale),
        "q": workloads.random_bits(rng, (md.rows, w.hq, w.dim), w.bf16, w.scale),
    }
    max_positions = int(md.lengths(w.page).max()) + 16
    cache = _rope_cache(max_positions, w.dim)
    kdraft = 7
    draft = rng.integers(0, 4, size=(md.batch, kdraft)).astype(np.int64)
    verify = rng.integers(0, 4, size=(md.batch, kdraft + 1)).astype(np.int64)
    verify[:, :kdraft] = np.where(rng.random((md.batch, kdraft)) < 0.7, draft, verify[:, :kdraft])
    return w, md, inp, cache, draft, verify, kdraft


def _expected(w, md, inp, cache, draft, verify):
    dt = w.dtype_code
    q_rot, k_rot = oracle.rope(inp["q"], inp["knew"].reshape(md.rows, w.hkv, w.dim), md.positions,
                               cache, dt)
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(k_rot.reshape(md.rows, w.width), inp["vnew"], ko, vo, md.slots, w.cache_slots)
    want, want32 = oracle.attention(q_rot, ko, vo, md.qo, md.kv, md.pages, md.last, w.hq, w.hkv,
                                    w.dim, w.page, True, dt)
    return q_rot, k_rot, ko, vo, want, want32, oracle.accept(draft, verify)


@pytest.fixture(scope="module")
def shim():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from fekv import _lib
    _lib.load()
    return ctypes.CDLL(_lib.SHIM_PATH)


def _fn(lib, name, args, res=None):
    f = getattr(lib, name)
    f.argtypes = args
    f.restype = res
    return f


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_shim_in_process(shim, name):
    """The DeviceModel's operator sequence through the shim's C++ entry points."""
    import torch
    P, I, B = ctypes.c_void_p, ctypes.c_int, ctypes.c_bool
    create = _fn(shim, "_ZN2fe4cuda11create_planEiiiiiibi", [I, I, I, I, I, I, B, I], P)
    destroy = _fn(shim, "_ZN2fe4cuda12destroy_planEPNS0_13AttentionPlanE", [P])
    prepare = _fn(shim, "_ZN2fe4cuda12prepare_planEPNS0_13AttentionPlanEPKiS4_S4_S4_iibPv",
                  [P, P, P, P, P, I, I, B, P])
    rope = _fn(shim, "_ZN2fe4cuda4ropeEPvS1_PKlPKfiiiibS1_i", [P, P, P, P, I, I, I, I, B, P, I])
    store = _fn(shim, "_ZN2fe4cuda5storeEPKvS2_PvS3_PKliibS3_i", [P, P, P, P, P, I, I, B, P, I])
    attention = _fn(shim, "_ZN2fe4cuda9attentionEPNS0_13AttentionPlanEPvS3_S3_S3_bS3_",
                    [P, P, P, P, P, B, P])
    accept = _fn(shim, "_ZN2fe4cuda6acceptEPKlS2_PliiPv", [P, P, P, I, I, P])

    w, md, inp, cache, draft, verify, kdraft = _case(name)
    # A C++ exception cannot cross ctypes (it would end the process), so the
    # same plan is first created and prepared through the C ABI, which
    # reports a failure as a Python error instead.
    import fekv
    pre = fekv.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(), w.bf16,
                             w.num_blocks)
    pre.prepare(md.qo, md.kv, md.pages, md.last)
    pre.close()
    torch.cuda.synchronize()
    assert fekv.device_errors() == 0
    dev = {k: torch.from_numpy(v.view(np.int16)).cuda() for k, v in inp.items()}
    slots = torch.from_numpy(md.slots).cuda()
    pos = torch.from_numpy(md.positions).cuda()
    cache_d = torch.from_numpy(cache).cuda()
    draft_d, verify_d = torch.from_numpy(draft).cuda(), torch.from_numpy(verify).cuda()
    committed = torch.full((md.batch, kdraft + 2), -1, dtype=torch.int64, device="cuda")
    out = torch.empty_like(dev["q"])
    stream = torch.cuda.current_stream().cuda_stream
    host = [np.ascontiguousarray(a, np.int32) for a in (md.qo, md.kv, md.pages, md.last)]
    plan = create(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(), w.bf16, w.num_blocks)
    assert plan
    prepare(plan, *[a.ctypes.data for a in host], md.batch, md.rows, False, stream)
    rope(dev["q"].data_ptr(), dev["knew"].data_ptr(), pos.data_ptr(), cache_d.data_ptr(), md.rows,
         w.hq, w.hkv, w.dim, w.bf16, stream, cache.shape[0])
    store(dev["knew"].data_ptr(), dev["vnew"].data_ptr(), dev["kpool"].data_ptr(),
          dev["vpool"].data_ptr(), slots.data_ptr(), md.rows, w.width, w.bf16, stream,
          w.cache_slots)
    attention(plan, dev["q"].data_ptr(), dev["kpool"].data_ptr(), dev["vpool"].data_ptr(),
              out.data_ptr(), True, stream)
    accept(draft_d.data_ptr(), verify_d.data_ptr(), committed.data_ptr(), md.batch, kdraft, stream)
    torch.cuda.synchronize()
    destroy(plan)

    def bits(t):
        return t.cpu().numpy().view(np.uint16)

    q_rot, k_rot, ko, vo, want, want32, acc = _expected(w, md, inp, cache, draft, verify)
    np.testing.assert_array_equal(bits(dev["q"]).reshape(q_rot.shape), q_rot)
    np.testing.assert_array_equal(bits(dev["knew"]).reshape(-1), k_rot.reshape(-1))
    np.testing.assert_array_equal(bits(dev["kpool"]).reshape(ko.shape), ko)
    np.testing.assert_array_equal(bits(dev["vpool"]).reshape(vo.shape), vo)
    res = compare_attention(bits(out).reshape(want.shape), want, w.bf16, ref_f32=want32)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    np.testing.assert_array_equal(committed.cpu().numpy(), acc)


def _build_driver(tmp_path):
    from fekv import _lib
    libdir = os.path.dirname(_lib.SHIM_PATH)
    exe = str(tmp_path / "shim_step")
    cuda_lib = "/usr/local/cuda/lib64"
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
           "-I", "/usr/local/cuda/include", DRIVER_SRC, "-o", exe, "-L", libdir,
           "-lfe_native_cuda_b200", "-lfe_kv_b200", "-L", cuda_lib, "-lcudart",
           f"-Wl,-rpath,{libdir}:{cuda_lib}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_shim_cpp_program(shim, tmp_path, name):
    """A C++ caller of the shim header: the same sequence, then the error
    behaviour (capacity, context, page id, head_dim, width, null plan)."""
    exe = _build_driver(tmp_path)
    w, md, inp, cache, draft, verify, kdraft = _case(name)
    d = tmp_path / "io"
    d.mkdir()
    (d / "dims.txt").write_text(" ".join(str(x) for x in (
        w.hq, w.hkv, w.dim, w.page, md.batch, md.rows, w.max_pages(), w.num_blocks, int(w.bf16),
        cache.shape[0], kdraft)))
    arrays = {"kpool": inp["kpool"], "vpool": inp["vpool"], "knew": inp["knew"],
              "vnew": inp["vnew"], "q": inp["q"], "slots": md.slots.astype(np.int64),
              "pos": md.positions.astype(np.int64), "draft": draft, "verify": verify,
              "qo": md.qo.astype(np.int32), "kv": md.kv.astype(np.int32),
              "pages": md.pages.astype(np.int32), "last": md.last.astype(np.int32),
              "cache": cache}
    for k, a in arrays.items():
        np.ascontiguousarray(a).tofile(str(d / k))
    r = subprocess.run([exe, str(d)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "shim_step ok" in r.stdout
    assert "errors capacity=1 context=1 page=1 dim=1 width=1 null_plan=1" in r.stdout, r.stdout

    def load(fname, dtype, shape):
        return np.fromfile(str(d / fname), dtype=dtype).reshape(shape)

    q_rot, k_rot, ko, vo, want, want32, acc = _expected(w, md, inp, cache, draft, verify)
    np.testing.assert_array_equal(load("q.out", np.uint16, q_rot.shape), q_rot)
    np.testing.assert_array_equal(load("knew.out", np.uint16, (-1,)), k_rot.reshape(-1))
    np.testing.assert_array_equal(load("kpool.out", np.uint16, ko.shape), ko)
    np.testing.assert_array_equal(load("vpool.out", np.uint16, vo.shape), vo)
    got = load("attn.out", np.uint16, want.shape)
    res = compare_attention(got, want, w.bf16, ref_f32=want32)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    np.testing.assert_array_equal(load("accept.out", np.int64, acc.shape), acc)
