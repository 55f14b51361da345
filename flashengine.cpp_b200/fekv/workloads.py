"""Seeded synthetic paged-KV workloads with the shapes of the five configs the
path is measured on (attention shapes of Qwen3-0.6B / 8B / 30B-A3B / 32B; no
model weights or datasets are involved, only K/V/q values drawn from
N(0,1) x scale). Everything is derived from ``numpy.random.default_rng(seed)``.

C1 ``c1``: hq16/hkv8/d128 fp16, page 16, 256-page pool; contexts
    {17,128,511,1000}; block tables are slices of one seeded permutation of
    the pool; 1 appended token per sequence; decode attention.
C2 ``c2``: hq32/hkv8 bf16, 36 layers; 64 sequences, contexts U[512,4096];
    random non-contiguous pages; x0.5; 1 appended token + decode per step.
C3 ``c3``: hq32/hkv8 bf16; 4 prefill chunks of 512 rows over cached prefixes
    drawn from {0,512,1024,2048} + 60 decode rows with contexts U[256,2048];
    causal; 2108 rows.
C4 ``c4``: hq32/hkv4 bf16, 48 layers; 128 sequences over one shared
    2048-token prefix (refcounted pages); each adds 1..256 divergent tokens;
    every odd sequence is forked from its even neighbour after that one's
    divergent tokens, so a partial shared tail page is copied on write; then
    a 16-row verify block per sequence, non-causal.
C5 ``c5``: hq64/hkv8 bf16, 64 layers; 1024 sequences, 128 per GPU, contexts
    LogNormal(ln 8192, 0.5) clipped to [2048, 32768]; split-K decode. The
    1024 sequences are split into 8 shards of nearly equal KV bytes.
``c2_shard``: C2 for sequence-sharded runs (one seeded list of 8 x 64
    contexts split into balanced shards of 64).

Two head_dim 256 workloads cover the hybrid and draft models' full-attention
layers (the reference serves them through ATen with any head_dim):
Q35 ``q35``: hq16/hkv2/d256 bf16 (the full-attention layer shape of the
    public Qwen3-Next hybrid configuration), 12 layers (one full-attention
    layer in four of a 48-layer stack); 64 sequences, contexts U[512,4096];
    x0.5; 1 appended token + decode per step.
DFL ``draft``: hq16/hkv2/d256 bf16, 4 layers; 32 sequences, contexts
    U[512,4096], each appending a 16-row block attended with the full
    (non-causal) mask, as a block draft model's step does.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .metadata import StepMetadata, build_step_metadata


@dataclass
class PagedWorkload:
    name: str
    hq: int
    hkv: int
    dim: int
    page: int
    bf16: bool
    num_blocks: int                 # request pages; page `num_blocks` is the padding page
    block_tables: list              # per sequence, int32 page ids
    cached: np.ndarray              # tokens in the cache before the step
    rows: np.ndarray                # tokens appended (= query rows) by the step
    causal: bool
    scale: float
    layers: int
    seed: int
    cow: tuple | None = None        # (src, dst, ntok) page copies applied before the step
    notes: dict = field(default_factory=dict)

    @property
    def G(self) -> int:
        return self.hq // self.hkv

    @property
    def width(self) -> int:
        return self.hkv * self.dim

    @property
    def cache_slots(self) -> int:
        return (self.num_blocks + 1) * self.page

    @property
    def batch(self) -> int:
        return len(self.block_tables)

    @property
    def dtype_code(self) -> int:
        return 1 if self.bf16 else 0

    def max_pages(self, steps: int = 1) -> int:
        most = int((self.cached + self.rows * steps).max()) if self.batch else 0
        return -(-most // self.page) + 1

    def metadata(self, step: int = 0) -> StepMetadata:
        starts = self.cached + self.rows * step
        return build_step_metadata(self.block_tables, starts, self.rows, self.page)

    def kv_bytes(self, step: int = 0) -> int:
        """Algorithmic decode bytes: K and V of every visible key, read once
        per KV head, plus q and o."""
        md = self.metadata(step)
        keys = int(md.lengths(self.page).sum())
        return keys * 2 * self.width * 2 + 2 * md.rows * self.hq * self.dim * 2


def _tables_from_permutation(perm, npages):
    out, off = [], 0
    for n in npages:
        out.append(np.asarray(perm[off:off + n], dtype=np.int32))
        off += n
    return out


def c1(seed: int = 0) -> PagedWorkload:
    rng = np.random.default_rng(seed)
    page, blocks = 16, 256
    ctx = np.array([17, 128, 511, 1000], dtype=np.int64)
    rows = np.ones(4, dtype=np.int64)
    npages = [-(-(int(c) + 1) // page) for c in ctx]
    perm = rng.permutation(blocks)
    return PagedWorkload("C1", 16, 8, 128, page, False, blocks,
                         _tables_from_permutation(perm, npages), ctx, rows, True, 1.0, 1, seed)


def decode_workload(name, hq, hkv, ctx, bf16, seed, steps=1, scale=1.0, layers=1, page=16,
                    spare_pages=0, dim=128) -> PagedWorkload:
    """Batched decode: 1 appended token per sequence per step, with block
    tables drawn as a seeded random permutation of a pool sized to the sum of
    contexts (+ steps) plus `spare_pages`."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, dtype=np.int64)
    npages = [-(-(int(c) + steps) // page) for c in ctx]
    blocks = int(sum(npages)) + int(spare_pages)
    perm = rng.permutation(blocks)
    return PagedWorkload(name, hq, hkv, dim, page, bf16, blocks,
                         _tables_from_permutation(perm, npages), ctx,
                         np.ones(ctx.shape[0], dtype=np.int64), True, scale, layers, seed)


def c2(seed: int = 0, steps: int = 1, batch: int = 64) -> PagedWorkload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(512, 4097, size=batch)
    w = decode_workload("C2", 32, 8, ctx, True, seed + 1, steps=steps, scale=0.5, layers=36)
    return w


def c3(seed: int = 0) -> PagedWorkload:
    rng = np.random.default_rng(seed)
    page = 16
    prefixes = rng.choice(np.array([0, 512, 1024, 2048]), size=4)
    dctx = rng.integers(256, 2049, size=60)
    cached = np.concatenate([prefixes, dctx]).astype(np.int64)
    rows = np.concatenate([np.full(4, 512), np.ones(60)]).astype(np.int64)
    npages = [-(-int(c + r) // page) for c, r in zip(cached, rows)]
    blocks = int(sum(npages))
    perm = rng.permutation(blocks)
    w = PagedWorkload("C3", 32, 8, 128, page, True, blocks, _tables_from_permutation(perm, npages),
                      cached, rows, True, 1.0, 36, seed)
    w.notes["prefixes"] = prefixes.tolist()
    return w


def c4(seed: int = 0, batch: int = 128, prefix: int = 2048, verify_rows: int = 16) -> PagedWorkload:
    """Shared prefix + copy-on-write forks + non-causal verify."""
    rng = np.random.default_rng(seed)
    page = 16
    div = rng.integers(1, 257, size=batch)
    prefix_pages = prefix // page
    next_page = [prefix_pages]  # pages [0, prefix_pages) hold the shared prefix

    def alloc(n):
        out = list(range(next_page[0], next_page[0] + n))
        next_page[0] += n
        return out

    tables, cached, forks = [None] * batch, np.zeros(batch, np.int64), []
    shared = list(range(prefix_pages))
    for e in range(0, batch, 2):
        # even sequence: prefix + its own divergent tokens (+ room for verify)
        le = prefix + int(div[e])
        own = alloc(-(-(le + verify_rows) // page) - prefix_pages)
        tables[e] = shared + own
        cached[e] = le
        if e + 1 < batch:
            # odd sequence: forked from `e` at length le; shares e's full pages,
            # copies e's partial tail page on write, then adds div[e+1] tokens.
            o = e + 1
            full = le // page
            tail = le % page
            lo = le + int(div[o])
            table = tables[e][:full]
            need = -(-(lo + verify_rows) // page) - full
            fresh = alloc(need)
            tables[o] = table + fresh
            cached[o] = lo
            if tail:
                forks.append((e, o, le))
    blocks = next_page[0]
    # Scatter the logical page ids over a random physical permutation.
    perm = rng.permutation(blocks).astype(np.int32)
    tables = [perm[np.asarray(t, dtype=np.int64)] for t in tables]
    cow = None
    if forks:
        # the copy-on-write lists come from the library's fork helper
        from .ops import fork_copies

        cow = fork_copies([tables[e] for e, _, _ in forks], [tables[o] for _, o, _ in forks],
                          [le for _, _, le in forks], page)
    w = PagedWorkload("C4", 32, 4, 128, page, True, blocks, tables, cached,
                      np.full(batch, verify_rows, np.int64), False, 1.0, 48, seed, cow=cow)
    w.notes["prefix_pages"] = perm[:0].tolist()
    w.notes["shared_prefix_pages"] = [int(x) for x in perm[:prefix_pages]]
    w.notes["divergent"] = div.tolist()
    return w


def c2_shard(shard: int = 0, nshards: int = 8, seed: int = 0, steps: int = 1,
             per_shard: int = 64) -> PagedWorkload:
    """C2 for sequence-sharded runs: one seeded list of nshards x 64 contexts
    U[512, 4096], split into shards of 64 sequences with nearly equal KV
    bytes (fekv.dist.balanced_shards); GPU `shard` runs one of them."""
    from .dist import balanced_shards

    rng = np.random.default_rng(seed)
    ctx_all = rng.integers(512, 4097, size=per_shard * nshards)
    own = balanced_shards(ctx_all, nshards, per_shard)[shard]
    w = decode_workload("C2", 32, 8, ctx_all[own], True, seed + 1 + shard, steps=steps, scale=0.5,
                        layers=36)
    w.notes["shard"] = f"{shard} of {nshards} balanced shards of {per_shard} (seed {seed})"
    return w


def c5_contexts(seed: int = 0, total: int = 1024, median: float = 8192.0, sigma: float = 0.5):
    rng = np.random.default_rng(seed)
    ctx = rng.lognormal(np.log(median), sigma, size=total)
    return np.clip(np.round(ctx), 2048, 32768).astype(np.int64)


def c5(rank: int = 0, world: int = 1, seed: int = 0, steps: int = 32, per_gpu: int = 128):
    """C5: the 1024 contexts of the config, split into 8 shards of 128
    sequences with nearly equal KV bytes; GPU `rank` runs shard `rank`."""
    from .dist import balanced_shards

    nshards = max(world, 8)
    ctx_all = c5_contexts(seed, per_gpu * nshards)
    own = balanced_shards(ctx_all, nshards, per_gpu)[rank]
    w = decode_workload("C5", 64, 8, ctx_all[own], True, seed + 1000 + rank, steps=steps,
                        scale=0.5, layers=64)
    w.notes["sigma"] = 0.5
    w.notes["shard"] = f"{rank} of {nshards} balanced shards of {per_gpu}"
    return w


def q35(seed: int = 0, steps: int = 1, batch: int = 64) -> PagedWorkload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(512, 4097, size=batch)
    return decode_workload("Q35", 16, 2, ctx, True, seed + 1, steps=steps, scale=0.5, layers=12,
                           dim=256)


def draft(seed: int = 0, batch: int = 32, block: int = 16) -> PagedWorkload:
    rng = np.random.default_rng(seed)
    page = 16
    cached = rng.integers(512, 4097, size=batch).astype(np.int64)
    rows = np.full(batch, block, dtype=np.int64)
    npages = [-(-int(c + r) // page) for c, r in zip(cached, rows)]
    blocks = int(sum(npages))
    perm = rng.permutation(blocks)
    return PagedWorkload("DFL", 16, 2, 256, page, True, blocks,
                         _tables_from_permutation(perm, npages), cached, rows, False, 0.5, 4, seed)


def random_bits(rng, shape, bf16: bool, scale: float = 1.0) -> np.ndarray:
    """N(0,1) x scale rounded to fp16/bf16, as uint16 bit patterns."""
    x = (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(scale))
    if bf16:
        u = x.view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return x.astype(np.float16).view(np.uint16)
