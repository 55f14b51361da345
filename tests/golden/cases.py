"""Golden parity cases for the paged-KV path (test infrastructure).

Each case is a small paged-KV step: pool contents, new K/V rows with their
slot mapping, query rows and the attention metadata. ``make_golden.py`` runs
the reference's own ATen implementation (FlashEngine.cpp
src/portable_gpu_ops.cpp, compiled for the CPU by oracle/build_oracle.py) on
each case and stores its outputs under tests/golden/*.npz.

Inputs are regenerated from the case's seed with numpy's PCG64 generator; the
fixture records a sha256 of the generated inputs so a drift in the generator
is detected instead of silently comparing different data. Small cases also
store their inputs outright.
"""
from __future__ import annotations

import hashlib
import os
import sys
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "flashengine.cpp_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

from fekv import workloads  # noqa: E402
from fekv.metadata import build_step_metadata  # noqa: E402


@dataclass
class Case:
    name: str
    hq: int
    hkv: int
    page: int
    bf16: bool
    num_blocks: int
    block_tables: list
    cached: np.ndarray
    rows: np.ndarray
    causal: bool
    seed: int
    scale: float = 1.0
    pad_to: int | None = None     # graph padding (slot -1 rows, dummy page)
    store_inputs: bool = False

    dim: int = 128

    @property
    def width(self):
        return self.hkv * self.dim

    @property
    def cache_slots(self):
        return (self.num_blocks + 1) * self.page

    @property
    def dtype_code(self):
        return 1 if self.bf16 else 0

    def metadata(self):
        return build_step_metadata(self.block_tables, self.cached, self.rows, self.page,
                                   pad_to=self.pad_to, pad_rows=1, dummy_page=self.num_blocks)

    def max_pages(self):
        md = self.metadata()
        return int((md.kv[1:] - md.kv[:-1]).max()) + 1

    def inputs(self):
        """Pools (every slot of every page seeded, padding page zero), new
        K/V rows and q, as uint16 bit patterns."""
        rng = np.random.default_rng(self.seed)
        md = self.metadata()
        kpool = workloads.random_bits(rng, (self.cache_slots, self.width), self.bf16, self.scale)
        vpool = workloads.random_bits(rng, (self.cache_slots, self.width), self.bf16, self.scale)
        pad0 = self.num_blocks * self.page
        kpool[pad0:] = 0
        vpool[pad0:] = 0
        knew = workloads.random_bits(rng, (md.rows, self.width), self.bf16, self.scale)
        vnew = workloads.random_bits(rng, (md.rows, self.width), self.bf16, self.scale)
        q = workloads.random_bits(rng, (md.rows, self.hq, self.dim), self.bf16, self.scale)
        return {"kpool": kpool, "vpool": vpool, "knew": knew, "vnew": vnew, "q": q}


def input_digest(inp: dict) -> str:
    h = hashlib.sha256()
    for k in ("kpool", "vpool", "knew", "vnew", "q"):
        h.update(np.ascontiguousarray(inp[k]).tobytes())
    return h.hexdigest()


def _tables(rng, blocks, lengths, page):
    perm = rng.permutation(blocks).astype(np.int32)
    out, off = [], 0
    for n in lengths:
        k = -(-int(n) // page)
        out.append(perm[off:off + k])
        off += k
    assert off <= blocks
    return out


def _case(name, hq, hkv, cached, rows, bf16, causal, seed, page=16, spare=2, **kw):
    cached = np.asarray(cached, np.int64)
    rows = np.asarray(rows, np.int64)
    lengths = cached + rows
    blocks = int(sum(-(-int(n) // page) for n in lengths)) + spare
    rng = np.random.default_rng(seed ^ 0x5EED)
    return Case(name, hq, hkv, page, bf16, blocks, _tables(rng, blocks, lengths, page), cached,
                rows, causal, seed, **kw)


def all_cases():
    w = workloads.c1(seed=0)
    c1 = Case("c1_decode", w.hq, w.hkv, w.page, w.bf16, w.num_blocks, w.block_tables, w.cached,
              w.rows, True, seed=1, store_inputs=False)
    return [
        c1,
        # decode, GQA 4, lengths around page boundaries (after the append: 1,16,17,32,33,101)
        _case("decode_g4_bf16", 8, 2, [0, 15, 16, 31, 32, 100], [1] * 6, True, True, 11),
        # chunked prefill, causal, with and without cached prefix, mixed with decode
        _case("prefill_causal_bf16", 8, 2, [0, 7, 40, 300], [20, 33, 1, 64], True, True, 12),
        _case("prefill_causal_f16", 8, 2, [0, 7, 40, 300], [20, 33, 1, 64], False, True, 13),
        # speculative verify, non-causal block over cached context, GQA 8
        _case("verify_full_f16", 16, 2, [30, 70, 1], [16, 16, 16], False, False, 14),
        _case("verify_full_bf16", 16, 2, [30, 70, 1], [16, 16, 16], True, False, 15),
        # GQA 1 (MHA) and GQA 16
        _case("mha_prefill_bf16", 2, 2, [5, 0, 64], [3, 17, 1], True, True, 16),
        _case("g16_mixed_f16", 16, 1, [9, 40, 200], [1, 2, 5], False, True, 17),
        # long contexts that the planner splits across CTAs (split-K)
        _case("decode_split_bf16", 8, 1, [3000, 5000, 700], [1, 1, 1], True, True, 18),
        # graph padding: batch 3 padded to 5 with slot -1 rows on the dummy page
        _case("graph_padding_f16", 4, 2, [10, 33, 64], [1, 1, 1], False, True, 19, pad_to=5,
              store_inputs=True),
        # page size 32
        _case("page32_prefill_bf16", 4, 2, [0, 31, 64], [40, 2, 1], True, True, 20, page=32),
        # value scale of the decode configs (0.5)
        _case("decode_scale05_bf16", 8, 2, [511, 1000, 2047], [1, 1, 1], True, True, 21, scale=0.5),
    ]


def case_by_name(name):
    for c in all_cases():
        if c.name == name:
            return c
    raise KeyError(name)


def fixture_path(name):
    return os.path.join(HERE, f"{name}.npz")
