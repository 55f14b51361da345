"""fe_kv_fork_copies (the copy-on-write trigger for forked sequences) against
the reference's block-sharing rules, on the CPU.

RefBlockManager restates the reference's BlockManager (src/scheduler.cpp:6-36):
a FIFO free deque, per-page reference counts, prefix pages published under
their token prefix, probe() sharing only whole published pages and keeping at
least one token to recompute, eviction of a published page when it is
reallocated. It is pinned by the reference's own host assertions
(tests/host_tests.cpp:33-37). A fork then runs through it exactly as the
scheduler would (probe, then ensure), and the helper turns the fork into
copies: applied with the oracle's block copy, the child's prefix KV equals
the parent's bit for bit, later appends of either sequence never touch a page
the other reads, and every page returns to the free list once all holders
release it.
"""
from collections import deque

import numpy as np
import pytest

import fekv
import oracle

PAGE = 16


class Seq:
    def __init__(self, tokens):
        self.tokens = list(tokens)
        self.blocks = []
        self.cached = 0


class RefBlockManager:
    """src/scheduler.cpp:6-36 (ensure, release, probe, publish)."""

    def __init__(self, total, size, caching=False):
        self.size, self.caching = size, caching
        self.free = deque(range(total))
        self.refs = [0] * total
        self.used = set()
        self.cached = {}   # token prefix -> page
        self.keys = {}     # page -> token prefix
        self.evictions = 0

    def ensure(self, s, target):
        needed = -(-target // self.size)
        if needed <= len(s.blocks):
            return True
        if needed - len(s.blocks) > len(self.free):
            return False
        while len(s.blocks) < needed:
            pid = self.free.popleft()
            if pid in self.keys:  # a published page is evicted when reallocated
                del self.cached[self.keys.pop(pid)]
                self.evictions += 1
            assert self.refs[pid] == 0 and pid not in self.used, "page allocated twice"
            self.used.add(pid)
            self.refs[pid] = 1
            s.blocks.append(pid)
        return True

    def release(self, s):
        for pid in s.blocks:
            assert self.refs[pid] > 0, "page released twice"
            self.refs[pid] -= 1
            if self.refs[pid] == 0:
                self.used.remove(pid)
                self.free.append(pid)
        s.blocks = []
        s.cached = 0

    def probe(self, s):
        if not self.caching:
            return
        assert not s.blocks and s.cached == 0
        end = self.size
        while end < len(s.tokens):  # keeps at least one token to recompute
            pid = self.cached.get(tuple(s.tokens[:end]))
            if pid is None:
                break
            if self.refs[pid] == 0:
                self.free.remove(pid)
                self.used.add(pid)
            self.refs[pid] += 1
            s.blocks.append(pid)
            s.cached = end
            end += self.size

    def publish(self, s, computed):
        if not self.caching:
            return
        computed = min(computed, len(s.tokens))
        for end in range(self.size, computed + 1, self.size):
            pid = s.blocks[(end - 1) // self.size]
            key = tuple(s.tokens[:end])
            if key in self.cached:
                continue
            assert pid not in self.keys, "a published page may not change"
            self.cached[key] = pid
            self.keys[pid] = key


def test_restatement_matches_reference_host_assertions():
    """tests/host_tests.cpp:33-37, restated."""
    blocks = RefBlockManager(2, 16)
    a, b = Seq([1]), Seq([2])
    assert blocks.ensure(a, 17)
    assert not blocks.ensure(b, 1) and b.blocks == []
    blocks.release(a)
    assert len(blocks.used) == 0
    assert blocks.ensure(b, 1)
    blocks.release(b)
    cache = RefBlockManager(4, 16, True)
    first, same, different = Seq([7] * 33), Seq([7] * 33), Seq([7] * 33)
    assert cache.ensure(first, 33)
    cache.publish(first, 32)
    cache.probe(same)
    assert same.cached == 32 and len(same.blocks) == 2 and same.blocks[0] == first.blocks[0]
    assert cache.ensure(same, 33)
    different.tokens[1] = 9
    cache.probe(different)
    assert different.cached == 0
    cache.release(first)
    assert len(cache.used) == 3
    cache.release(same)
    assert len(cache.used) == 0 and len(cache.cached) == 2
    exact = Seq([7] * 32)
    cache.probe(exact)
    assert exact.cached == 16 and len(exact.blocks) == 1
    cache.release(exact)
    assert cache.ensure(different, 64)
    assert len(cache.cached) == 0 and cache.evictions == 2
    cache.release(different)


def _slots(blocks, positions):
    blocks = np.asarray(blocks, np.int64)
    positions = np.asarray(positions, np.int64)
    return blocks[positions // PAGE] * PAGE + positions % PAGE


def _prefix_kv(pool, blocks, length, width):
    npages = -(-length // PAGE)
    kv = np.array([0, npages], np.int32)
    last = np.array([(length - 1) % PAGE + 1], np.int32)
    return oracle.gather(pool, kv, np.asarray(blocks[:npages], np.int32), last, PAGE, width)


@pytest.mark.parametrize("seed", range(6))
def test_forks_through_block_manager(seed):
    rng = np.random.default_rng(seed)
    total, width, layers = 96, 64, 2
    mgr = RefBlockManager(total, PAGE, caching=True)
    pools_k = [oracle.from_float(rng.standard_normal(((total + 1) * PAGE, width)), 1)
               for _ in range(layers)]
    pools_v = [oracle.from_float(rng.standard_normal(((total + 1) * PAGE, width)), 1)
               for _ in range(layers)]
    plen = int(rng.integers(20, 200))
    parent = Seq(rng.integers(0, 50, size=plen))
    assert mgr.ensure(parent, plen)
    # only part of the parent's prefix may be published yet: probe() shares
    # those pages, the child copies the other full pages as well as its tail
    mgr.publish(parent, plen if seed % 2 == 0 else int(rng.integers(0, plen + 1)))
    children = []
    for _ in range(4):
        L = int(rng.integers(1, plen + 1))
        if rng.random() < 0.3:
            L = max(PAGE, (L // PAGE) * PAGE)  # page-aligned forks too
        extra = int(rng.integers(1, 40))
        child = Seq(list(parent.tokens[:L]) + list(rng.integers(100, 150, size=extra)))
        mgr.probe(child)  # shares published full pages, as the scheduler does
        assert mgr.ensure(child, len(child.tokens))
        children.append((child, L))
    src, dst, ntok = fekv.fork_copies([parent.blocks] * len(children),
                                      [c.blocks for c, _ in children],
                                      [L for _, L in children], PAGE)
    # one copy per prefix page the child does not share (the partial tail,
    # and full pages probe() left to recompute)
    want = sum(sum(1 for j in range(-(-L // PAGE)) if c.blocks[j] != parent.blocks[j])
               for c, L in children)
    assert len(src) == want
    assert (ntok >= 1).all() and (ntok <= PAGE).all()
    if seed % 2 == 0:  # everything published: only partial tails are copied
        assert (ntok < PAGE).all()
    oracle.copy_blocks(pools_k, pools_v, src, dst, ntok, PAGE, width)
    for c, L in children:
        for pool in pools_k + pools_v:
            np.testing.assert_array_equal(_prefix_kv(pool, np.asarray(c.blocks), L, width),
                                          _prefix_kv(pool, np.asarray(parent.blocks), L, width))
    # later appends: each sequence writes its next positions; nothing any
    # other sequence reads as its prefix changes
    before = [[_prefix_kv(p, np.asarray(c.blocks), L, width) for p in pools_k]
              for c, L in children]
    before_parent = [_prefix_kv(p, np.asarray(parent.blocks), plen, width) for p in pools_k]
    for c, L in children:
        pos = np.arange(L, len(c.tokens))
        rows = oracle.from_float(rng.standard_normal((len(pos), width)), 1)
        for k, v in zip(pools_k, pools_v):
            oracle.append(rows, rows, k, v, _slots(c.blocks, pos), k.shape[0])
    for (c, L), b in zip(children, before):
        for p, want_kv in zip(pools_k, b):
            np.testing.assert_array_equal(_prefix_kv(p, np.asarray(c.blocks), L, width), want_kv)
    for p, want_kv in zip(pools_k, before_parent):
        np.testing.assert_array_equal(_prefix_kv(p, np.asarray(parent.blocks), plen, width),
                                      want_kv)
    # reference counts: shared pages stay allocated until their last holder
    # releases them; everything returns to the free list exactly once
    shared = set(parent.blocks) & set().union(*[set(c.blocks) for c, _ in children])
    mgr.release(parent)
    assert shared <= mgr.used
    for c, _ in children:
        mgr.release(c)
    assert not mgr.used and sorted(mgr.free) == list(range(total))


def test_shared_partial_tail_is_rejected():
    parent = np.arange(5, dtype=np.int32)
    with pytest.raises(fekv.FeError) as e:  # fork at 40 tokens sharing page 2 (8 tokens)
        fekv.fork_copies([parent], [np.array([0, 1, 2, 9], np.int32)], [40], PAGE)
    assert e.value.status == fekv._lib.FE_ERR_INVALID_ARGUMENT and "partial tail" in str(e.value)
    with pytest.raises(fekv.FeError):  # a child page that is the parent's page 4
        fekv.fork_copies([parent], [np.array([0, 1, 4], np.int32)], [40], PAGE)
    with pytest.raises(fekv.FeError):  # fork length beyond the child's table
        fekv.fork_copies([parent], [np.array([0, 1], np.int32)], [40], PAGE)
    # page-aligned fork: everything shared, nothing to copy
    src, _, _ = fekv.fork_copies([parent], [np.array([0, 1, 7], np.int32)], [32], PAGE)
    assert len(src) == 0


def test_c4_workload_uses_the_helper():
    """C4's copy-on-write lists are the helper's output for its forks."""
    from fekv import workloads
    w = workloads.c4(seed=0)
    src, dst, ntok = w.cow
    assert len(src) > 0 and (ntok < PAGE).all() and (ntok > 0).all()
    assert not set(dst.tolist()) & set(src.tolist())
