"""KV append / block copy / page clear / gather on the GPU through the C ABI,
bit-exact against the CPU oracle and the reference fixtures."""
import hashlib

import numpy as np
import pytest

import cases
import oracle
from fe_testutil import to_device, to_host_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fk():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import fekv
    fekv.load()
    return fekv


def _i64(a):
    import torch
    return torch.from_numpy(np.asarray(a, np.int64)).cuda()


def _i32(a):
    import torch
    return torch.from_numpy(np.asarray(a, np.int32)).cuda()


@pytest.mark.parametrize("name", [c.name for c in cases.all_cases()])
def test_append_matches_reference(fk, name):
    case = cases.case_by_name(name)
    fx = dict(np.load(cases.fixture_path(name)))
    inp = case.inputs()
    md = case.metadata()
    kc, vc = to_device(inp["kpool"], case.bf16), to_device(inp["vpool"], case.bf16)
    fk.store(to_device(inp["knew"], case.bf16), to_device(inp["vnew"], case.bf16), kc, vc,
             _i64(md.slots), md.rows, case.width, case.bf16, None, case.cache_slots)
    k, v = to_host_bits(kc).reshape(inp["kpool"].shape), to_host_bits(vc).reshape(inp["vpool"].shape)
    assert fk.device_errors() == 0
    # skip semantics (src/cuda_kernels.cu:24): equal to the CPU oracle everywhere
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    np.testing.assert_array_equal(k, ko)
    np.testing.assert_array_equal(v, vo)
    # and equal to the reference's ATen store on every non-padding row written
    ok = md.slots >= 0
    np.testing.assert_array_equal(k[md.slots[ok]], fx["ref_k_rows"][ok])
    np.testing.assert_array_equal(v[md.slots[ok]], fx["ref_v_rows"][ok])
    if ok.all():
        assert hashlib.sha256(k.tobytes()).hexdigest() == str(fx["ref_k_sha256"])


@pytest.mark.parametrize("rows,hkv,bf16", [(1, 8, True), (64, 8, True), (2108, 8, True),
                                            (37, 4, False), (5000, 1, False)])
def test_append_random_bit_exact(fk, rows, hkv, bf16):
    rng = np.random.default_rng(rows * 7 + hkv)
    width, page, blocks = hkv * 128, 16, max(8, rows // 8 + 4)
    cache_slots = (blocks + 1) * page
    pool_k = rng.integers(0, 65535, size=(cache_slots, width), dtype=np.uint16)
    pool_v = rng.integers(0, 65535, size=(cache_slots, width), dtype=np.uint16)
    knew = rng.integers(0, 65535, size=(rows, width), dtype=np.uint16)
    vnew = rng.integers(0, 65535, size=(rows, width), dtype=np.uint16)
    slots = rng.permutation(blocks * page)[:rows].astype(np.int64)
    slots[rng.random(rows) < 0.1] = -1  # graph padding rows are skipped
    kc, vc = to_device(pool_k, bf16), to_device(pool_v, bf16)
    fk.store(to_device(knew, bf16), to_device(vnew, bf16), kc, vc, _i64(slots), rows, width, bf16,
             None, cache_slots)
    oracle.append(knew, vnew, pool_k, pool_v, slots, cache_slots)
    np.testing.assert_array_equal(to_host_bits(kc).reshape(pool_k.shape), pool_k)
    np.testing.assert_array_equal(to_host_bits(vc).reshape(pool_v.shape), pool_v)
    assert fk.device_errors() == 0


def test_append_out_of_range_slot_is_reported_not_written(fk):
    rng = np.random.default_rng(5)
    width, cache_slots = 256, 64
    pool = rng.integers(0, 65535, size=(cache_slots, width), dtype=np.uint16)
    new = rng.integers(0, 65535, size=(3, width), dtype=np.uint16)
    kc, vc = to_device(pool, True), to_device(pool, True)
    fk.device_errors()  # clear
    fk.store(to_device(new, True), to_device(new, True), kc, vc, _i64([3, cache_slots, 5]), 3, width,
             True, None, cache_slots)
    bits = fk.device_errors()
    assert bits & fk._lib.FE_DEVERR_SLOT_RANGE
    want = pool.copy()
    want[3], want[5] = new[0], new[2]
    np.testing.assert_array_equal(to_host_bits(kc).reshape(pool.shape), want)


def test_append_rejects_bad_arguments(fk):
    import torch
    x = torch.zeros(16, 1024, dtype=torch.bfloat16, device="cuda")
    s = _i64([0])
    with pytest.raises(fk.FeError):
        fk.store(x, x, x, x, s, 1, 1004, True, None, 16)   # width not a multiple of 8
    with pytest.raises(fk.FeError):
        fk.store(x[:, 1:], x, x, x, s, 1, 1024, True, None, 16)  # misaligned source


def test_copy_blocks_cow_matches_oracle(fk):
    """Copy-on-write of partial tail pages plus whole-block copies over
    several layers (C4 shape, fewer layers)."""
    import fekv.workloads as wl
    w = wl.c4(seed=0)
    src, dst, ntok = w.cow
    # add whole-block copies of prefix pages too
    extra_src = np.array(w.notes["shared_prefix_pages"][:2], np.int32)
    used = set(src.tolist()) | set(dst.tolist()) | set(extra_src.tolist())
    extra_dst = [int(t[-1]) for t in w.block_tables[1::2] if int(t[-1]) not in used][:2]
    assert len(extra_dst) == 2
    src = np.concatenate([src, extra_src])
    dst = np.concatenate([dst, np.array(extra_dst, np.int32)])
    ntok = np.concatenate([ntok, [16, 16]]).astype(np.int32)
    layers = 3
    rng = np.random.default_rng(9)
    host = [rng.integers(0, 65535, size=(w.cache_slots, w.width), dtype=np.uint16)
            for _ in range(2 * layers)]
    dev = [to_device(h, True) for h in host]
    fk.copy_blocks(dev[:layers], dev[layers:], _i32(src), _i32(dst), _i32(ntok), w.page, w.width,
                   w.num_blocks + 1)
    oracle.copy_blocks(host[:layers], host[layers:], src, dst, ntok, w.page, w.width)
    for h, d in zip(host, dev):
        np.testing.assert_array_equal(to_host_bits(d).reshape(h.shape), h)
    assert fk.device_errors() == 0


def test_copy_blocks_bad_page_is_reported(fk):
    import torch
    pool = torch.zeros(4 * 16, 256, dtype=torch.float16, device="cuda")
    fk.device_errors()
    fk.copy_blocks([pool], [pool], _i32([0, 9]), _i32([1, 2]), _i32([16, 16]), 16, 256, 4)
    assert fk.device_errors() & fk._lib.FE_DEVERR_PAGE_RANGE
    fk.copy_blocks([pool], [pool], _i32([0]), _i32([1]), _i32([17]), 16, 256, 4)
    assert fk.device_errors() & fk._lib.FE_DEVERR_NTOK_RANGE


def test_clear_padding_page(fk):
    rng = np.random.default_rng(2)
    blocks, page, width = 10, 16, 512
    host = rng.integers(1, 65535, size=((blocks + 1) * page, width), dtype=np.uint16)
    pools = [to_device(host, True), to_device(host, True)]
    fk.clear_pages(pools, _i32([blocks]), page, width, blocks + 1)
    for p in pools:
        got = to_host_bits(p).reshape(host.shape)
        np.testing.assert_array_equal(got[:blocks * page], host[:blocks * page])
        assert (got[blocks * page:] == 0).all()


@pytest.mark.parametrize("name", ["c1_decode", "prefill_causal_bf16", "page32_prefill_bf16"])
def test_gather_bit_exact(fk, name):
    import torch
    case = cases.case_by_name(name)
    inp = case.inputs()
    md = case.metadata()
    lengths = md.lengths(case.page)
    offs = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
    pool = to_device(inp["kpool"], case.bf16)
    out = torch.empty(int(lengths.sum()), case.width, dtype=pool.dtype, device="cuda")
    fk.gather(pool, out, _i32(md.kv), _i32(md.pages), _i32(md.last), _i32(offs), md.batch,
              int(lengths.max()), case.page, case.width)
    want = oracle.gather(inp["kpool"], md.kv, md.pages, md.last, case.page, case.width)
    np.testing.assert_array_equal(to_host_bits(out).reshape(want.shape), want)


@pytest.mark.parametrize("fork_len", [37, 48, 1000, 1])
def test_fork_copy_on_write_then_attention(fk, fork_len):
    """A child forked from a parent at `fork_len` tokens: fe_kv_fork_copies
    turns the fork into copies, fe_kv_copy_blocks applies them on the GPU,
    and decode attention of the child over the shared prefix equals the
    parent's bit for bit (same keys in the same order, the same plan shape).
    Both then append different tokens: neither changes the other's prefix."""
    import torch
    from fekv.metadata import build_step_metadata
    rng = np.random.default_rng(fork_len)
    hq, hkv, page = 32, 8, 16
    width = hkv * 128
    nblocks = 200
    parent_len = fork_len + 20
    perm = rng.permutation(nblocks).astype(np.int32)
    parent = perm[:-(-parent_len // page)]
    full = fork_len // page
    child_pages = -(-(fork_len + 30) // page)
    child = np.concatenate([parent[:full], perm[100:100 + child_pages - full]]).astype(np.int32)
    src, dst, ntok = fk.fork_copies([parent], [child], [fork_len], page)
    assert len(src) == (1 if fork_len % page else 0)
    g = torch.Generator(device="cuda")
    g.manual_seed(fork_len)
    kc = torch.randn((nblocks + 1) * page, width, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn((nblocks + 1) * page, width, generator=g, device="cuda").to(torch.bfloat16)
    if len(src):
        fk.copy_blocks([kc], [vc], _i32(src), _i32(dst), _i32(ntok), page, width, nblocks + 1)
    q = torch.randn(1, hq, 128, generator=g, device="cuda").to(torch.bfloat16)

    def attend(table, length):
        md = build_step_metadata([table], [length - 1], [1], page)
        plan = fk.AttentionPlan(hq, hkv, 128, page, 1, len(table) + 1, True, nblocks)
        plan.prepare(md.qo, md.kv, md.pages, md.last)
        out = torch.empty_like(q)
        plan.attention(q, kc, vc, out, True)
        torch.cuda.synchronize()
        plan.close()
        return to_host_bits(out)

    want = attend(parent, fork_len)
    np.testing.assert_array_equal(attend(child, fork_len), want)
    # each appends its own next tokens; the other's prefix is unchanged
    for table, start in ((parent, fork_len), (child, fork_len)):
        pos = np.arange(start, start + 10)
        slots = table[pos // page].astype(np.int64) * page + pos % page
        rows = torch.randn(10, width, generator=g, device="cuda").to(torch.bfloat16)
        fk.store(rows, rows, kc, vc, _i64(slots), 10, width, True, None,
                 (nblocks + 1) * page)
    np.testing.assert_array_equal(attend(parent, fork_len), want)
    np.testing.assert_array_equal(attend(child, fork_len), want)
    assert fk.device_errors() == 0
