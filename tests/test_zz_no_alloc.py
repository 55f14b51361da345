"""fe_paged_decode_noalloc — the decode entry point that allocates nothing.

Some callers cannot make a device allocation where they call attention: an
engine that handed all free HBM to its own KV-page pool at start-up (a later
cudaMalloc fails), or a hot loop in which an allocation, which may
synchronise the device, is not allowed. This entry point takes the step
metadata as device arrays and keeps its split-K scratch in a fixed array
inside the library, so it needs no plan and no cudaMalloc. These tests check,
through the C ABI, that two calls in a row give the same results as the
plan-based fe_attn_run within the attention tolerance used by every parity
test here, that small cases also match the CPU oracle, and that device memory
does not move while it runs.

This file is collected last on purpose (name order).
"""
import numpy as np
import pytest

import oracle
from fe_testutil import compare_attention, to_host_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fk():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import fekv
    fekv.load()
    return fekv


def _run_pair(fk, hq, hkv, ctx, bf16, seed, with_oracle=False):
    import torch
    from fekv import workloads
    w = workloads.decode_workload("noalloc", hq, hkv, ctx, bf16, seed, steps=1)
    md = w.metadata()
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    kc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    vc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    qs = [torch.randn(md.rows, hq, 128, generator=g, device="cuda").to(dt) for _ in range(2)]
    kv_d = torch.from_numpy(md.kv).cuda()
    pages_d = torch.from_numpy(md.pages).cuda()
    last_d = torch.from_numpy(md.last).cuda()
    outs_plan = [torch.empty_like(q) for q in qs]
    outs_static = [torch.full_like(q, float("nan")) for q in qs]
    max_pages = w.max_pages()

    plan = fk.AttentionPlan(hq, hkv, 128, w.page, md.batch, max_pages, bf16, w.num_blocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last)
    for q, o in zip(qs, outs_plan):
        plan.attention(q, kc, vc, o, True)
    torch.cuda.synchronize()

    # first call on this device resolves the scratch array; then measure
    fk.paged_decode_noalloc(qs[0], kc, vc, outs_static[0], kv_d, pages_d, last_d, md.batch, hq,
                            hkv, w.page, w.num_blocks, max_pages)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for q, o in zip(qs, outs_static):  # two calls in a row
        fk.paged_decode_noalloc(q, kc, vc, o, kv_d, pages_d, last_d, md.batch, hq, hkv, w.page,
                                w.num_blocks, max_pages)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, "device memory changed during allocation-free calls"
    assert fk.device_errors() == 0
    plan.close()
    plan_bits = [to_host_bits(o) for o in outs_plan]
    static_bits = [to_host_bits(o) for o in outs_static]
    if with_oracle:
        kb, vb = to_host_bits(kc), to_host_bits(vc)
        for q, got in zip(qs, static_bits):
            want, want32 = oracle.attention(to_host_bits(q), kb, vb, md.qo, md.kv, md.pages,
                                            md.last, hq, hkv, 128, w.page, True, 1 if bf16 else 0)
            res = compare_attention(got, want, bf16, ref_f32=want32)
            assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    return plan_bits, static_bits


@pytest.mark.parametrize("hq,hkv,ctx,bf16", [
    (32, 8, [600, 3000, 4096, 17, 1, 2200, 900, 3500] * 3, True),   # C2 shape, split-K
    (16, 8, [17, 128, 511, 1000], False),                            # C1 shape, fp16
    (32, 4, [2049, 2304, 40, 700], True),                            # 4 heads per item
    (32, 2, [5000, 12, 1700, 300, 2600], True),                      # G = 16: 2-row-block items
    (16, 1, [3100, 1, 800, 2222], False),                            # H = 1, G = 16
    (8, 2, [1025, 64, 4000], True),                                  # H = 2, G = 4
])
def test_noalloc_matches_plan_path(fk, hq, hkv, ctx, bf16):
    small = sum(ctx) <= 6000
    plan_outs, static_outs = _run_pair(fk, hq, hkv, ctx, bf16, seed=hq + hkv + len(ctx),
                                       with_oracle=small)
    for call, (want, got) in enumerate(zip(plan_outs, static_outs)):
        res = compare_attention(got, want, bf16)
        assert res["excess"] <= 0, (call, res)
        assert np.isfinite(oracle.to_float(got, 1 if bf16 else 0)).all()


@pytest.mark.parametrize("hq,batch", [(32, 4096), (128, 200)])
def test_noalloc_large_batch_runs_unsplit(fk, hq, batch):
    """Batches whose split-K records cannot share the fixed scratch run every
    sequence unsplit: 4096 sequences (more head groups than twice the SMs, so
    no split is wanted) and 200 sequences of 128-row head groups (hq128 /
    hkv8), whose two-way split would need 26.6 MB of records, more than the
    16 MiB scratch. The results still equal the plan path's."""
    rng = np.random.default_rng(11 + hq)
    hi = 300 if batch > 1000 else 2000
    ctx = [int(c) for c in rng.integers(1, hi, size=batch)]
    ctx[7] = 2500  # one long context, which the plan path splits
    plan_outs, static_outs = _run_pair(fk, hq, 8, ctx, True, seed=12)
    for call, (want, got) in enumerate(zip(plan_outs, static_outs)):
        res = compare_attention(got, want, True)
        assert res["excess"] <= 0, (call, res)


def test_noalloc_rejects_oversized_batch(fk):
    import torch
    x = torch.zeros(16, 128, dtype=torch.bfloat16, device="cuda")
    i = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(fk.FeError) as e:
        fk.paged_decode_noalloc(x, x, x, x, i, i, i, 20000, 8, 1, 16, 4, 2)
    assert e.value.status == fk._lib.FE_ERR_CAPACITY
