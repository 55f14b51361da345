"""CPU checkers for the paged-KV hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg / reference arm may import this package. The product library
(``flashengine.cpp_b200``) never imports, links or calls it.

Checkers, reached through ctypes:

* :func:`c_oracle` — the plain-C restatement in ``oracle/fe_oracle.c``
  (append: ``src/cuda_kernels.cu:24``; attention: ``src/portable_gpu_ops.cpp:27-44``;
  block copy: memcpy, as the reference has no block-copy op).
* :class:`RefAten` — the reference's own ATen path, ``src/portable_gpu_ops.cpp``,
  compiled for the CPU by ``oracle/build_oracle.py`` into ``oracle/_ref``.
* :func:`ref_cuda` — the reference's own CUDA rope / store / accept kernels
  (``src/cuda_kernels.cu``) for sm_100a, run beside this repository's kernels.
* :class:`RefFlashInfer` — the reference's own CUDA attention
  (``src/flashinfer_attention.cu``, FlashInfer FA2) for sm_100a: the GPU
  comparator for attention outputs and timings.

16-bit values travel as ``numpy.uint16`` bit patterns; ``dtype`` is 0 for
fp16 and 1 for bf16, as in the product C-ABI.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build_oracle

_P = ctypes.c_void_p
_I = ctypes.c_int
_c_lib = None
_ref_lib = None


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def c_oracle():
    """Load (building if needed) the C restatement."""
    global _c_lib
    if _c_lib is None:
        path = build_oracle.C_ORACLE_LIB
        if not os.path.exists(path):
            build_oracle.build_c_oracle()
        lib = ctypes.CDLL(path)
        lib.fe_oracle_append.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I]
        lib.fe_oracle_copy_blocks.argtypes = [_P, _P, _I, _P, _P, _P, _I, _I, _I]
        lib.fe_oracle_gather.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
        lib.fe_oracle_attention.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P,
                                            _I, _I, _I, _I, _I, _I, _I]
        lib.fe_oracle_attention.restype = _I
        lib.fe_oracle_rope.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I]
        lib.fe_oracle_float_to_half.argtypes = [ctypes.c_float]
        lib.fe_oracle_float_to_half.restype = ctypes.c_uint16
        lib.fe_oracle_float_to_bf16.argtypes = [ctypes.c_float]
        lib.fe_oracle_float_to_bf16.restype = ctypes.c_uint16
        lib.fe_oracle_half_to_float.argtypes = [ctypes.c_uint16]
        lib.fe_oracle_half_to_float.restype = ctypes.c_float
        lib.fe_oracle_bf16_to_float.argtypes = [ctypes.c_uint16]
        lib.fe_oracle_bf16_to_float.restype = ctypes.c_float
        _c_lib = lib
    return _c_lib


def _u16(a: np.ndarray) -> np.ndarray:
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def append(k, v, kc, vc, slots, cache_slots, redirect_negative=False):
    """In place on kc/vc. Rows: k/v [rows, width]; pools [cache_slots, width]."""
    k, v, kc, vc = _u16(k), _u16(v), _u16(kc), _u16(vc)
    slots = _i64(slots)
    rows = slots.shape[0]
    width = k.size // max(rows, 1) if rows else 0
    c_oracle().fe_oracle_append(_ptr(k), _ptr(v), _ptr(kc), _ptr(vc), _ptr(slots), rows, width,
                                int(cache_slots), int(bool(redirect_negative)))


def copy_blocks(k_pools, v_pools, src, dst, ntok, page, width):
    """In place on every pool. k_pools/v_pools: lists of uint16 arrays."""
    n = len(k_pools)
    kp = (ctypes.c_void_p * n)(*[_u16(p).ctypes.data for p in k_pools])
    vp = (ctypes.c_void_p * n)(*[_u16(p).ctypes.data for p in v_pools])
    src, dst, ntok = _i32(src), _i32(dst), _i32(ntok)
    c_oracle().fe_oracle_copy_blocks(kp, vp, n, _ptr(src), _ptr(dst), _ptr(ntok), src.shape[0],
                                     int(page), int(width))


def rope(q, k, pos, cache, dtype):
    """RoPE restated (src/cuda_kernels.cu:19-23) on uint16 bit arrays
    q [rows, hq, dim] and k [rows, hkv, dim] (returned rotated copies);
    cache: float32 [max_positions, rotary_dim] (cos | sin), rotary_dim <= dim."""
    q = np.ascontiguousarray(q, dtype=np.uint16).copy()
    k = np.ascontiguousarray(k, dtype=np.uint16).copy()
    pos = _i64(pos)
    cache = np.ascontiguousarray(cache, dtype=np.float32)
    rows, hkv, dim = k.shape
    hq = q.shape[1] if q.ndim == 3 else 0
    c_oracle().fe_oracle_rope(_ptr(q), _ptr(k), _ptr(pos), _ptr(cache), rows, hq, hkv, dim,
                              cache.shape[1], cache.shape[0], dtype)
    return q, k


def accept(draft, verify):
    """Greedy acceptance restated (src/cuda_kernels.cu:25): returns the
    [batch, k+2] rows the kernel writes (entries it leaves untouched are -1)."""
    draft = np.asarray(draft, np.int64)
    verify = np.asarray(verify, np.int64)
    batch, k1 = verify.shape
    k = k1 - 1
    out = np.full((batch, k + 2), -1, np.int64)
    for b in range(batch):
        m = 0
        while m < k and draft[b, m] == verify[b, m]:
            out[b, m] = draft[b, m]
            m += 1
        out[b, m] = verify[b, m]
        out[b, k + 1] = m + 1
    return out


def seq_lengths(kv, last, page):
    kv, last = np.asarray(kv, dtype=np.int64), np.asarray(last, dtype=np.int64)
    return (kv[1:] - kv[:-1] - 1) * page + last


def gather(pool, kv, pages, last, page, width):
    pool = _u16(pool)
    kv, pages, last = _i32(kv), _i32(pages), _i32(last)
    total = int(seq_lengths(kv, last, page).sum())
    out = np.zeros((total, width), dtype=np.uint16)
    c_oracle().fe_oracle_gather(_ptr(pool), _ptr(out), _ptr(kv), _ptr(pages), _ptr(last),
                                kv.shape[0] - 1, int(page), int(width))
    return out


def attention(q, kpool, vpool, qo, kv, pages, last, hq, hkv, dim, page, causal, dtype):
    """Returns (out_bits uint16 [rows, hq, dim], out_f32 float32 [rows, hq, dim])."""
    q, kpool, vpool = _u16(q), _u16(kpool), _u16(vpool)
    qo, kv, pages, last = _i32(qo), _i32(kv), _i32(pages), _i32(last)
    rows = int(qo[-1])
    out = np.zeros((rows, hq, dim), dtype=np.uint16)
    out32 = np.zeros((rows, hq, dim), dtype=np.float32)
    rc = c_oracle().fe_oracle_attention(_ptr(q), _ptr(kpool), _ptr(vpool), _ptr(out), _ptr(out32),
                                        _ptr(qo), _ptr(kv), _ptr(pages), _ptr(last),
                                        kv.shape[0] - 1, hq, hkv, dim, page, int(bool(causal)),
                                        int(dtype))
    if rc != 0:
        raise MemoryError("fe_oracle_attention: allocation failed")
    return out, out32


def to_float(bits: np.ndarray, dtype: int) -> np.ndarray:
    """uint16 bit patterns -> float32 (exact)."""
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def from_float(x: np.ndarray, dtype: int) -> np.ndarray:
    """float32 -> uint16 bit patterns, round to nearest even (numpy for fp16)."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    if dtype:
        u = x.view(np.uint32).astype(np.uint64)
        nan = (u & 0x7FFFFFFF) > 0x7F800000
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
        return r
    return x.astype(np.float16).view(np.uint16)


# ---------------------------------------------------------------------------
# The reference's own ATen path, compiled for the CPU.
# ---------------------------------------------------------------------------

_ref_cuda_lib = None


def ref_cuda_available() -> bool:
    return os.path.exists(build_oracle.REF_CUDA_LIB)


def ref_cuda():
    """The reference's own CUDA kernels (src/cuda_kernels.cu) compiled from its
    source: ref_cuda_rope / ref_cuda_store / ref_cuda_accept, device pointers.
    GPU tests only."""
    global _ref_cuda_lib
    if _ref_cuda_lib is None:
        path = build_oracle.REF_CUDA_LIB
        if not os.path.exists(path):
            built = build_oracle.build_reference_cuda()
            if built is None:
                raise FileNotFoundError("oracle/_ref/libfe_ref_cuda.so is not built and the "
                                        "reference source tree is absent")
        lib = ctypes.CDLL(path)
        lib.ref_cuda_rope.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I]
        lib.ref_cuda_store.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _P, _I]
        lib.ref_cuda_accept.argtypes = [_P, _P, _P, _I, _I, _P]
        for f in (lib.ref_cuda_rope, lib.ref_cuda_store, lib.ref_cuda_accept):
            f.restype = _I
        _ref_cuda_lib = lib
    return _ref_cuda_lib


def ref_library_path() -> str:
    return build_oracle.REF_LIB


def ref_available() -> bool:
    return os.path.exists(build_oracle.REF_LIB)


def _ref():
    global _ref_lib
    if _ref_lib is None:
        path = build_oracle.REF_LIB
        if not os.path.exists(path):
            built = build_oracle.build_reference()
            if built is None:
                raise FileNotFoundError("oracle/_ref/libfe_ref_aten.so is not built and the "
                                        "reference source tree is absent")
        lib = ctypes.CDLL(path)
        lib.fe_ref_last_error.restype = ctypes.c_char_p
        lib.fe_ref_set_threads.argtypes = [_I]
        lib.fe_ref_get_threads.restype = _I
        lib.fe_ref_create_plan.argtypes = [_I, _I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_P)]
        lib.fe_ref_destroy_plan.argtypes = [_P]
        lib.fe_ref_prepare_plan.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
        lib.fe_ref_attention.argtypes = [_P, _P, _P, _P, _P, _I]
        lib.fe_ref_store.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I]
        for f in ("fe_ref_create_plan", "fe_ref_prepare_plan", "fe_ref_attention", "fe_ref_store"):
            getattr(lib, f).restype = _I
        _ref_lib = lib
    return _ref_lib


class RefError(RuntimeError):
    pass


def _check_ref(rc: int):
    if rc != 0:
        raise RefError(_ref().fe_ref_last_error().decode("utf-8", "replace"))


def ref_set_threads(n: int):
    _ref().fe_ref_set_threads(int(n))


def ref_get_threads() -> int:
    return _ref().fe_ref_get_threads()


class RefAten:
    """The reference's ``fe::cuda`` AttentionPlan / attention / store, on the CPU."""

    def __init__(self, hq, hkv, dim, page, max_batch, max_pages, bf16, blocks):
        self.lib = _ref()
        h = ctypes.c_void_p()
        _check_ref(self.lib.fe_ref_create_plan(hq, hkv, dim, page, max_batch, max_pages, int(bf16),
                                               blocks, ctypes.byref(h)))
        self.handle = h
        self.hq, self.hkv, self.dim, self.page, self.bf16 = hq, hkv, dim, page, bool(bf16)
        self.cache_slots = (blocks + 1) * page
        self._keep = []

    def prepare(self, qo, kv, pages, last, graph=False):
        qo, kv, pages, last = _i32(qo), _i32(kv), _i32(pages), _i32(last)
        if pages.size == 0:
            pages = np.zeros(1, np.int32)
        self._keep = [qo, kv, pages, last]
        _check_ref(self.lib.fe_ref_prepare_plan(self.handle, _ptr(qo), _ptr(kv), _ptr(pages),
                                                _ptr(last), kv.shape[0] - 1, int(qo[-1]),
                                                int(bool(graph))))
        self.rows = int(qo[-1])

    def attention(self, q, kpool, vpool, causal):
        q, kpool, vpool = _u16(q), _u16(kpool), _u16(vpool)
        out = np.zeros((self.rows, self.hq, self.dim), dtype=np.uint16)
        _check_ref(self.lib.fe_ref_attention(self.handle, _ptr(q), _ptr(kpool), _ptr(vpool),
                                             _ptr(out), int(bool(causal))))
        return out

    def store(self, k, v, kc, vc, slots):
        k, v, kc, vc = _u16(k), _u16(v), _u16(kc), _u16(vc)
        slots = _i64(slots)
        rows = slots.shape[0]
        width = k.size // max(rows, 1) if rows else 0
        _check_ref(self.lib.fe_ref_store(_ptr(k), _ptr(v), _ptr(kc), _ptr(vc), _ptr(slots), rows,
                                         width, int(self.bf16), self.cache_slots))

    def close(self):
        if self.handle:
            self.lib.fe_ref_destroy_plan(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# The reference's own CUDA attention (src/flashinfer_attention.cu over
# FlashInfer), built for sm_100a: the GPU comparator. Device pointers; GPU
# tests and bench.py's reference arm only.
# ---------------------------------------------------------------------------

_ref_fi_lib = None


def ref_flashinfer_available() -> bool:
    return os.path.exists(build_oracle.REF_FI_LIB)


def _ref_fi():
    global _ref_fi_lib
    if _ref_fi_lib is None:
        path = build_oracle.REF_FI_LIB
        if not os.path.exists(path):
            built = build_oracle.build_reference_flashinfer()
            if built is None:
                raise FileNotFoundError("oracle/_ref/libfe_ref_flashinfer.so is not built and "
                                        "the reference source tree is absent")
        lib = ctypes.CDLL(path)
        lib.fe_ref_fi_last_error.restype = ctypes.c_char_p
        lib.fe_ref_fi_create_plan.argtypes = [_I, _I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_P)]
        lib.fe_ref_fi_destroy_plan.argtypes = [_P]
        lib.fe_ref_fi_prepare_plan.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _P]
        lib.fe_ref_fi_attention.argtypes = [_P, _P, _P, _P, _P, _I, _P]
        for f in ("fe_ref_fi_create_plan", "fe_ref_fi_prepare_plan", "fe_ref_fi_attention"):
            getattr(lib, f).restype = _I
        _ref_fi_lib = lib
    return _ref_fi_lib


class RefFlashInfer:
    """The reference's fe::cuda AttentionPlan / prepare_plan / attention on the
    GPU (FlashInfer FA2 paged prefill kernel, split-KV disabled). Tensors are
    torch CUDA tensors; metadata are host int32 arrays."""

    def __init__(self, hq, hkv, dim, page, max_batch, max_pages, bf16, blocks):
        self.lib = _ref_fi()
        h = ctypes.c_void_p()
        self._check(self.lib.fe_ref_fi_create_plan(hq, hkv, dim, page, max_batch, max_pages,
                                                   int(bf16), blocks, ctypes.byref(h)))
        self.handle = h
        self._keep = []

    def _check(self, rc):
        if rc != 0:
            raise RefError(self.lib.fe_ref_fi_last_error().decode("utf-8", "replace"))

    def prepare(self, qo, kv, pages, last, stream=0, graph=False):
        qo, kv, pages, last = _i32(qo), _i32(kv), _i32(pages), _i32(last)
        if pages.size == 0:
            pages = np.zeros(1, np.int32)
        self._keep = [qo, kv, pages, last]
        self._check(self.lib.fe_ref_fi_prepare_plan(self.handle, _ptr(qo), _ptr(kv), _ptr(pages),
                                                    _ptr(last), kv.shape[0] - 1, int(qo[-1]),
                                                    int(bool(graph)), ctypes.c_void_p(stream)))

    def attention(self, q, k, v, out, causal, stream=0):
        self._check(self.lib.fe_ref_fi_attention(
            self.handle, ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
            ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(out.data_ptr()), int(bool(causal)),
            ctypes.c_void_p(stream)))

    def close(self):
        if self.handle:
            self.lib.fe_ref_fi_destroy_plan(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
