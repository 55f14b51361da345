"""Python mirror of the reference's ``fe::cuda`` KV/attention operator
interface (Cambridgebit/FlashEngine.cpp include/fe/native_cuda.hpp:6-14), over
the fe_kv C ABI. Device buffers are torch CUDA tensors (PyTorch is only the
allocator and stream provider here); per-step plan metadata are host arrays.

Names, argument meaning and error behaviour follow the reference:
``create_plan``/``AttentionPlan``, ``prepare_plan``, ``attention``, ``store``;
a failing call raises (the reference throws std::runtime_error).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import FE_DTYPE_BF16, FE_DTYPE_F16, FeError, check

_P = ctypes.c_void_p


def _torch():
    import torch

    return torch


def _ptr(t):
    if t is None:
        return None
    return _P(t.data_ptr())


def _stream(stream):
    if stream is None:
        torch = _torch()
        return _P(torch.cuda.current_stream().cuda_stream)
    if hasattr(stream, "cuda_stream"):
        return _P(stream.cuda_stream)
    return _P(int(stream))


def dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.bfloat16:
        return FE_DTYPE_BF16
    if t.dtype == torch.float16:
        return FE_DTYPE_F16
    raise TypeError(f"unsupported dtype {t.dtype}; expected float16 or bfloat16")


def _host_i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _require_device_i32(t):
    torch = _torch()
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.int32 and
            t.is_contiguous()):
        raise ValueError("expected a contiguous int32 CUDA tensor")


# ---------------------------------------------------------------------------
# fe::cuda::store  (include/fe/native_cuda.hpp:14)
# ---------------------------------------------------------------------------

def store(k, v, kc, vc, slots, rows=None, width=None, bf16=None, stream=None, cache_slots=None):
    """Scatter rows of k/v into the pools through `slots` (int64, device).
    Rows with a negative slot are skipped, as in the reference CUDA kernel."""
    lib = _lib.load()
    rows = int(slots.shape[0]) if rows is None else int(rows)
    width = int(k.numel() // max(rows, 1)) if width is None else int(width)
    dtype = dtype_code(kc) if bf16 is None else (FE_DTYPE_BF16 if bf16 else FE_DTYPE_F16)
    cache_slots = int(kc.numel() // width) if cache_slots is None else int(cache_slots)
    check(lib.fe_kv_append(_ptr(k), _ptr(v), _ptr(kc), _ptr(vc), _ptr(slots), rows, width, dtype,
                           cache_slots, _stream(stream)), "store")


# ---------------------------------------------------------------------------
# fe::cuda::rope / accept  (include/fe/native_cuda.hpp:13,15) and the fused
# rope + store (no reference counterpart)
# ---------------------------------------------------------------------------

def rope(q, k, pos, cache, stream=None):
    """Rotate q [rows, hq, dim] and k [rows, hkv, dim] in place with the fp32
    cache [max_positions, rotary_dim] (cos | sin); rotary_dim = the cache's
    width (dim for full rotary, less for partial rotary); pos: int64 [rows]."""
    lib = _lib.load()
    rows, hkv, dim = (int(x) for x in k.shape)
    hq = int(q.shape[1]) if q is not None else 0
    check(lib.fe_rope(_ptr(q) if q is not None else None, _ptr(k), _ptr(pos), _ptr(cache), rows,
                      hq, hkv, dim, int(cache.shape[1]), int(cache.shape[0]), dtype_code(k),
                      _stream(stream)), "rope")


def rope_append(q, k, v, kc, vc, slots, pos, cache, k_out=None, stream=None):
    """rope + store in one launch: q rotated in place, rotated k (and v) written
    to the pools [cache_slots, hkv*dim] through `slots`; the rotated keys also
    go to `k_out` when given (it may be `k`). The rotary width is the cache's
    width, as in rope()."""
    lib = _lib.load()
    rows, hkv, dim = (int(x) for x in k.shape)
    hq = int(q.shape[1])
    cache_slots = int(kc.numel() // (hkv * dim))
    check(lib.fe_rope_append(_ptr(q), _ptr(k), _ptr(v), _ptr(k_out) if k_out is not None else None,
                             _ptr(kc), _ptr(vc), _ptr(slots), _ptr(pos), _ptr(cache), rows, hq, hkv,
                             dim, int(cache.shape[1]), int(cache.shape[0]), dtype_code(k),
                             cache_slots, _stream(stream)), "rope_append")


def accept(draft, verify, out, stream=None):
    """Greedy acceptance: draft int64 [batch, k], verify [batch, k+1],
    out [batch, k+2] (device)."""
    lib = _lib.load()
    batch = int(verify.shape[0])
    k = int(verify.shape[1]) - 1
    check(lib.fe_accept(_ptr(draft), _ptr(verify), _ptr(out), batch, k, _stream(stream)),
          "accept")


# ---------------------------------------------------------------------------
# block copy / copy-on-write and page clearing (no reference counterpart)
# ---------------------------------------------------------------------------

def copy_blocks(k_pools, v_pools, src, dst, ntok, page, width, num_pages_total, dtype=None,
                stream=None):
    """Copy token rows [0, ntok[c]) of page src[c] onto page dst[c] in every
    layer's K and V pool. src/dst/ntok: int32 device tensors."""
    lib = _lib.load()
    n = len(k_pools)
    if n != len(v_pools):
        raise ValueError("k_pools and v_pools differ in length")
    kp = (_P * max(n, 1))(*[t.data_ptr() for t in k_pools])
    vp = (_P * max(n, 1))(*[t.data_ptr() for t in v_pools])
    dtype = dtype_code(k_pools[0]) if dtype is None else int(dtype)
    check(lib.fe_kv_copy_blocks(kp, vp, n, _ptr(src), _ptr(dst), _ptr(ntok), int(src.shape[0]),
                                int(page), int(width), int(num_pages_total), dtype,
                                _stream(stream)), "copy_blocks")


def fork_copies(parent_tables, child_tables, fork_lens, page):
    """Copy-on-write lists for forked sequences (host only): for fork f, the
    pages of the first fork_lens[f] tokens that child_tables[f] does not share
    with parent_tables[f] become (src, dst, ntok) entries for copy_blocks.
    Returns three int32 numpy arrays. Raises FeError on tables that would let
    one sequence write a page the other reads (a shared partial tail)."""
    lib = _lib.load()
    n = len(parent_tables)
    if len(child_tables) != n or len(fork_lens) != n:
        raise ValueError("one parent table, child table and fork length per fork")
    pt = [np.asarray(t, np.int32) for t in parent_tables]
    ct = [np.asarray(t, np.int32) for t in child_tables]
    poff = _host_i32(np.concatenate([[0], np.cumsum([len(t) for t in pt])]))
    coff = _host_i32(np.concatenate([[0], np.cumsum([len(t) for t in ct])]))
    pcat = _host_i32(np.concatenate(pt) if n else np.zeros(1, np.int32))
    ccat = _host_i32(np.concatenate(ct) if n else np.zeros(1, np.int32))
    lens = np.ascontiguousarray(np.asarray(fork_lens, np.int64))
    cap = int(sum(-(-int(L) // int(page)) for L in lens)) if n else 0
    src, dst, ntok = (np.zeros(max(cap, 1), np.int32) for _ in range(3))
    count = ctypes.c_int(0)
    hp = lambda a: a.ctypes.data_as(_P)  # noqa: E731
    check(lib.fe_kv_fork_copies(n, hp(pcat), hp(poff), hp(ccat), hp(coff), hp(lens), int(page),
                                hp(src), hp(dst), hp(ntok), cap, ctypes.byref(count)),
          "fork_copies")
    k = count.value
    return src[:k].copy(), dst[:k].copy(), ntok[:k].copy()


def clear_pages(pools, pages, page, width, num_pages_total, dtype=None, stream=None):
    """Zero whole pages (int32 device tensor `pages`) of every pool."""
    lib = _lib.load()
    n = len(pools)
    arr = (_P * max(n, 1))(*[t.data_ptr() for t in pools])
    dtype = dtype_code(pools[0]) if dtype is None else int(dtype)
    check(lib.fe_kv_clear_pages(arr, n, _ptr(pages), int(pages.shape[0]), int(page), int(width),
                                int(num_pages_total), dtype, _stream(stream)), "clear_pages")


def gather(pool, out, kv, pages, last, row_offset, batch, max_len, page, width, dtype=None,
           stream=None):
    """Dense copy of whole sequences' KV rows (device int32 metadata)."""
    lib = _lib.load()
    dtype = dtype_code(pool) if dtype is None else int(dtype)
    check(lib.fe_kv_gather(_ptr(pool), _ptr(out), _ptr(kv), _ptr(pages), _ptr(last),
                           _ptr(row_offset), int(batch), int(max_len), int(page), int(width), dtype,
                           _stream(stream)), "gather")


def paged_decode_noalloc(q, k_pool, v_pool, out, kv, pages, last, batch, hq, hkv, page,
                        num_blocks, max_pages, dtype=None, stream=None):
    """Decode attention through fe_paged_decode_noalloc: no plan and no
    device allocation (split-K scratch is a fixed array inside the library).
    kv/pages/last are int32 DEVICE tensors; one query row per sequence."""
    lib = _lib.load()
    dtype = dtype_code(q) if dtype is None else int(dtype)
    check(lib.fe_paged_decode_noalloc(_ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(out), _ptr(kv),
                                      _ptr(pages), _ptr(last), int(batch), int(hq), int(hkv),
                                      int(page), int(num_blocks), int(max_pages), dtype,
                                      _stream(stream)), "paged_decode_noalloc")


def device_errors(stream=None) -> int:
    """Read and clear the device-side error bits (FE_DEVERR_*)."""
    lib = _lib.load()
    bits = ctypes.c_uint32(0)
    check(lib.fe_device_errors(_stream(stream), ctypes.byref(bits)), "device_errors")
    return int(bits.value)


# ---------------------------------------------------------------------------
# fe::cuda::create_plan / destroy_plan / prepare_plan / attention
# (include/fe/native_cuda.hpp:7-10)
# ---------------------------------------------------------------------------

class AttentionPlan:
    """Owns an fe_attn_plan. `prepare` takes host metadata (as
    fe::cuda::prepare_plan); `attention` takes device tensors."""

    def __init__(self, hq, hkv, dim, page, max_batch, max_pages, bf16, blocks):
        self.lib = _lib.load()
        h = _P()
        dtype = FE_DTYPE_BF16 if bf16 else FE_DTYPE_F16
        check(self.lib.fe_attn_plan_create(int(hq), int(hkv), int(dim), int(page), int(max_batch),
                                           int(max_pages), dtype, int(blocks), ctypes.byref(h)),
              "create_plan")
        self.handle = h
        self.hq, self.hkv, self.dim, self.page = hq, hkv, dim, page
        self.bf16, self.blocks = bool(bf16), blocks

    def prepare(self, qo, kv, pages, last, batch=None, rows=None, graph=False, stream=None):
        qo, kv, pages, last = _host_i32(qo), _host_i32(kv), _host_i32(pages), _host_i32(last)
        batch = kv.shape[0] - 1 if batch is None else int(batch)
        rows = int(qo[batch]) if rows is None else int(rows)
        check(self.lib.fe_attn_plan_prepare(self.handle, qo.ctypes.data_as(_P),
                                            kv.ctypes.data_as(_P), pages.ctypes.data_as(_P),
                                            last.ctypes.data_as(_P), batch, rows, int(bool(graph)),
                                            _stream(stream)), "prepare_plan")

    def prepare_device(self, qo, kv, pages, last, batch, rows, stream=None):
        """fe_attn_plan_prepare_device: the same metadata as `prepare`, as
        int32 DEVICE tensors; the work lists are built on the GPU (graph mode,
        nothing read back, capturable in a CUDA graph)."""
        for t in (qo, kv, pages, last):
            _require_device_i32(t)
        check(self.lib.fe_attn_plan_prepare_device(self.handle, _ptr(qo), _ptr(kv), _ptr(pages),
                                                   _ptr(last), int(batch), int(rows),
                                                   _stream(stream)), "prepare_plan_device")

    def step_prepare_device(self, block_tables, starts, rows_per_seq, slots, positions,
                            stream=None):
        """fe_step_prepare_device: slot mapping and work lists on the GPU from
        int32 block tables [batch, stride] and start positions [batch] (< 0:
        graph padding entry); writes int64 slots / positions [batch *
        rows_per_seq]."""
        _require_device_i32(block_tables)
        _require_device_i32(starts)
        batch, stride = int(block_tables.shape[0]), int(block_tables.shape[1])
        if int(starts.shape[0]) != batch:
            raise ValueError("starts must have one entry per block-table row")
        torch = _torch()
        for t in (slots, positions):
            if t.dtype != torch.int64 or not t.is_cuda or t.numel() < batch * rows_per_seq:
                raise ValueError("slots / positions: int64 CUDA tensors of batch*rows_per_seq")
        check(self.lib.fe_step_prepare_device(self.handle, _ptr(block_tables), stride, _ptr(starts),
                                              batch, int(rows_per_seq), _ptr(slots),
                                              _ptr(positions), _stream(stream)),
              "step_prepare_device")

    def device_meta(self, total_pages=None, nbytes=1 << 22, stream=None) -> dict:
        """The plan's device metadata (what the kernels read), copied back and
        unpacked (parse_meta)."""
        buf = np.zeros(int(nbytes), np.uint8)
        check(self.lib.fe_attn_plan_debug_device_meta(self.handle, buf.ctypes.data_as(_P),
                                                      int(nbytes), _stream(stream)),
              "debug_device_meta")
        return parse_meta(buf, total_pages)

    def host_meta(self) -> dict:
        """The host copy of the last host-side prepare's metadata."""
        return _host_meta(self.lib, self.handle)

    def attention(self, q, k, v, out, causal=True, stream=None, lists=None):
        """fe_attn_run; `lists` (FE_ATTN_LISTS_DECODE / _ROWS) runs only part
        of the prepared work (fe_attn_run_lists)."""
        if lists is None:
            check(self.lib.fe_attn_run(self.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                       int(bool(causal)), _stream(stream)), "attention")
        else:
            check(self.lib.fe_attn_run_lists(self.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                             int(bool(causal)), int(lists), _stream(stream)),
                  "attention")

    def info(self) -> dict:
        inf = _lib.PlanInfo()
        check(self.lib.fe_attn_plan_get_info(self.handle, ctypes.byref(inf)), "plan_info")
        return {name: getattr(inf, name) for name, _ in _lib.PlanInfo._fields_}

    def close(self):
        if getattr(self, "handle", None):
            self.lib.fe_attn_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def create_plan(hq, hkv, dim, page, max_batch, max_pages, bf16, blocks) -> AttentionPlan:
    return AttentionPlan(hq, hkv, dim, page, max_batch, max_pages, bf16, blocks)


def destroy_plan(plan: AttentionPlan):
    plan.close()


def prepare_plan(plan: AttentionPlan, qo, kv, pages, last, batch, rows, graph=False, stream=None):
    plan.prepare(qo, kv, pages, last, batch, rows, graph, stream)


def attention(plan: AttentionPlan, q, k, v, output, causal=True, stream=None):
    plan.attention(q, k, v, output, causal, stream)


# ---------------------------------------------------------------------------
# host-only planner (test hook): inspect the work list without a GPU
# ---------------------------------------------------------------------------

ITEM_DTYPE = np.dtype([("seq", "<i4"), ("kvh", "<i2"), ("key_mode", "<i2"), ("rb0", "<i4"),
                       ("nrb", "<i4"), ("kt0", "<i4"), ("kt1", "<i4"), ("part", "<i4"),
                       ("group", "<i4")])
GROUP_DTYPE = np.dtype([("nsplit", "<i4"), ("part0", "<i4"), ("rec_floats", "<i4"),
                        ("rows", "<i4"), ("seq", "<i4"), ("kvh", "<i4"), ("row0", "<i4"),
                        ("rows_per_head", "<i4")])
SEQ_DTYPE = np.dtype([("q_row0", "<i4"), ("qrows", "<i4"), ("length", "<i4"),
                      ("page_off", "<i4")])


def _host_meta(lib, handle) -> dict:
    """The host copy of the last host-side prepare's metadata, unpacked."""
    n = ctypes.c_int64(0)
    check(lib.fe_attn_plan_debug_meta(handle, None, 0, ctypes.byref(n)), "meta")
    buf = np.zeros(n.value, dtype=np.uint8)
    check(lib.fe_attn_plan_debug_meta(handle, buf.ctypes.data_as(_P), n.value, ctypes.byref(n)),
          "meta")
    return parse_meta(buf)


def parse_meta(buf: np.ndarray, total_pages: int | None = None) -> dict:
    """Unpack a plan's metadata blob (fe_attn_plan.h layout; section order
    from the header's offsets). `total_pages` defaults to everything between
    the pages offset and the end (the host planner puts the pages last)."""
    h = buf[:128].view(np.int32)
    out = {"batch": int(h[18]), "rows": int(h[19]), "chunk_tiles": int(h[23]),
           "dec_heads": int(h[24]), "views": []}
    seqs_off, pages_off = int(h[20]), int(h[21])
    batch = out["batch"]
    out["seqs"] = buf[seqs_off:seqs_off + SEQ_DTYPE.itemsize * batch].view(SEQ_DTYPE)
    # lists: 0 = row work (non-causal), 1 = row work (causal), 2 = decode work
    for c in range(3):
        n_items, n_groups, grid = int(h[0 + c]), int(h[3 + c]), int(h[6 + c])
        co, io, go = int(h[9 + c]), int(h[12 + c]), int(h[15 + c])
        view = {
            "grid": grid,
            "n_items": n_items,
            "cta_off": (buf[co:co + 4 * (grid + 1)].view(np.int32) if grid
                        else np.zeros(1, np.int32)),
            "items": buf[io:io + ITEM_DTYPE.itemsize * n_items].view(ITEM_DTYPE),
            "groups": buf[go:go + GROUP_DTYPE.itemsize * n_groups].view(GROUP_DTYPE),
        }
        out["views"].append(view)
    end = int(h[22]) if total_pages is None else pages_off + 4 * int(total_pages)
    out["pages"] = buf[pages_off:end].view(np.int32)
    out["buf"] = buf
    return out


class HostPlan:
    """fe_attn_plan_create_host: validates metadata and builds the work list
    on the host for `grid_cap` CTAs, without touching a GPU."""

    def __init__(self, hq, hkv, dim, page, max_batch, max_pages, bf16, blocks, grid_cap=296):
        self.lib = _lib.load()
        h = _P()
        dtype = FE_DTYPE_BF16 if bf16 else FE_DTYPE_F16
        check(self.lib.fe_attn_plan_create_host(int(hq), int(hkv), int(dim), int(page),
                                                int(max_batch), int(max_pages), dtype, int(blocks),
                                                int(grid_cap), ctypes.byref(h)), "create_host")
        self.handle = h
        self.G = hq // hkv

    def prepare(self, qo, kv, pages, last, batch=None, rows=None, graph=False):
        qo, kv, pages, last = _host_i32(qo), _host_i32(kv), _host_i32(pages), _host_i32(last)
        batch = kv.shape[0] - 1 if batch is None else int(batch)
        rows = int(qo[batch]) if rows is None else int(rows)
        check(self.lib.fe_attn_plan_prepare(self.handle, qo.ctypes.data_as(_P),
                                            kv.ctypes.data_as(_P), pages.ctypes.data_as(_P),
                                            last.ctypes.data_as(_P), batch, int(rows),
                                            int(bool(graph)), None), "prepare_plan")
        return self.meta()

    def meta(self) -> dict:
        return _host_meta(self.lib, self.handle)

    def close(self):
        if getattr(self, "handle", None):
            self.lib.fe_attn_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["store", "copy_blocks", "paged_decode_noalloc", "clear_pages", "gather", "device_errors", "AttentionPlan",
           "create_plan", "destroy_plan", "prepare_plan", "attention", "HostPlan", "FeError",
           "dtype_code", "ITEM_DTYPE", "GROUP_DTYPE", "SEQ_DTYPE", "parse_meta"]
