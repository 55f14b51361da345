"""head_dim 256 (tcgen05 rows in fe_prefill_tc.cu, decode rows in fe_decode.cu)
through the same plan / attention calls, against the reference's own ATen
attention (src/portable_gpu_ops.cpp:27-44, which takes any head_dim; compiled
for the host as oracle/_ref) on small cases, and against the fp32 torch
restatement of it (pinned on the CPU by test_cpu_torch_restatement.py) on
every case. Tolerance as for head_dim 128: fe_testutil.ATOL widened by one
output ulp."""
import numpy as np
import pytest

from fe_testutil import (compare_attention, ref_aten_attention, to_host_bits,
                         torch_reference_attention)

pytestmark = pytest.mark.gpu

DIM = 256
PAGE = 16


@pytest.fixture(scope="module")
def fk():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import fekv
    fekv.load()
    return fekv


def _case(fk, hq, hkv, cached, rows, bf16, causal, seed, graph=False, ref_aten=False):
    import torch
    import fekv.workloads as wl
    from fekv.metadata import build_step_metadata
    rng = np.random.default_rng(seed)
    npg = [-(-int(c + r) // PAGE) for c, r in zip(cached, rows)]
    tables = wl._tables_from_permutation(rng.permutation(sum(npg) + 5), npg)
    nblocks = sum(npg) + 5
    md = build_step_metadata(tables, cached, rows, PAGE)
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    slots_total = (nblocks + 1) * PAGE
    kc = torch.randn(slots_total, hkv * DIM, generator=g, device="cuda").to(dt)
    vc = torch.randn(slots_total, hkv * DIM, generator=g, device="cuda").to(dt)
    q = torch.randn(md.rows, hq, DIM, generator=g, device="cuda").to(dt)
    plan = fk.AttentionPlan(hq, hkv, DIM, PAGE, md.batch, int(np.diff(md.kv).max()) + 1, bf16,
                            nblocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last, graph=graph)
    out = torch.full_like(q, float("nan"))
    plan.attention(q, kc, vc, out, causal)
    ref = torch_reference_attention(q, kc, vc, md.qo, md.kv, md.pages, md.last, hq, hkv, PAGE,
                                    causal)
    torch.cuda.synchronize()
    assert fk.device_errors() == 0
    out_bits = to_host_bits(out)
    res = compare_attention(out_bits, to_host_bits(ref.to(dt)), bf16, ref_f32=ref.cpu().numpy())
    if ref_aten:
        want = ref_aten_attention(to_host_bits(q), to_host_bits(kc), to_host_bits(vc), md, hq, hkv,
                                  DIM, PAGE, causal, bf16, nblocks)
        res["vs_reference"] = compare_attention(out_bits, want, bf16)
    plan.close()
    return res


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("hq,hkv", [(16, 2), (24, 4), (8, 8), (32, 2)])
def test_decode_rows(fk, bf16, hq, hkv):
    rng = np.random.default_rng(hq + hkv)
    cached = rng.integers(1, 3000, 12)
    res = _case(fk, hq, hkv, cached, np.ones(12, int), bf16, True, hq * 7 + hkv)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("seed", range(4))
def test_mixed_rows_random(fk, causal, seed):
    """Decode rows, draft / verify blocks and prefill chunks in one step."""
    rng = np.random.default_rng(50 + seed)
    hkv = int(rng.choice([1, 2, 4]))
    G = int(rng.choice([1, 2, 3, 4, 6, 8]))
    batch = int(rng.integers(1, 7))
    cached = rng.integers(0, 1500, batch)
    rows = np.where(rng.random(batch) < 0.4, 1, rng.integers(1, 160, batch))
    res = _case(fk, hkv * G, hkv, cached, rows, bool(seed % 2), causal, 900 + seed)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res


def test_graph_mode_plan(fk):
    res = _case(fk, 16, 2, [100, 2000, 7], [33, 1, 5], True, True, 3, graph=True)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("bf16", [True, False])
def test_draft_blocks_split_across_ctas(fk, causal, bf16):
    """DFlash-style 16-row blocks over long contexts: too few 64-row items to
    fill the GPU, so their key ranges are split into pieces whose records the
    merge kernel combines; checked against the fp32 reference, and the plan
    is checked to have split them."""
    from fekv.metadata import build_step_metadata
    cached, rows = [3000, 2500, 1800], [16, 16, 16]
    res = _case(fk, 16, 2, cached, rows, bf16, causal, 77 + causal)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    tables = [np.arange(i * 200, i * 200 + 200) for i in range(3)]
    md = build_step_metadata(tables, cached, rows, PAGE)
    hp = fk.HostPlan(16, 2, DIM, PAGE, 3, 200, True, 600, grid_cap=148)
    meta = hp.prepare(md.qo, md.kv, md.pages, md.last)
    assert (meta["views"][1 if causal else 0]["groups"]["nsplit"] >= 2).any()
    hp.close()


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("hq,hkv", [(16, 2), (8, 1), (32, 4)])
def test_decode_rows_vs_reference(fk, parity_record, bf16, hq, hkv):
    """Decode rows at head_dim 256 against the reference's ATen path itself,
    contexts long enough that the planner splits them."""
    cached = [2999, 17, 1500, 640, 2047, 1]
    res = _case(fk, hq, hkv, cached, np.ones(6, int), bf16, True, 300 + hq + hkv, ref_aten=True)
    parity_record(f"head_dim 256 decode hq{hq}/hkv{hkv} {'bf16' if bf16 else 'f16'} "
                  "(reference ATen path)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    assert res["vs_reference"]["excess"] <= 0, res


@pytest.mark.parametrize("causal", [True, False])
def test_draft_blocks_vs_reference(fk, parity_record, causal):
    """16-row draft / verify blocks at head_dim 256 (split into pieces over
    long contexts) and a prefill chunk, against the reference's ATen path."""
    cached, rows = [3000, 2500, 1800, 40], [16, 16, 16, 130]
    res = _case(fk, 16, 2, cached, rows, True, causal, 400 + causal, ref_aten=True)
    parity_record(f"head_dim 256 draft blocks + chunk, {'causal' if causal else 'full'} mask "
                  "(reference ATen path)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    assert res["vs_reference"]["excess"] <= 0, res


def test_q35_layer_full_size(fk, parity_record):
    """One full layer of the bench's q35 step (64 sequences, contexts
    512-4096, hq16/hkv2/d256)."""
    import fekv.workloads as wl
    w = wl.q35(seed=0)
    res = _case(fk, w.hq, w.hkv, w.cached, w.rows, w.bf16, w.causal, 31)
    parity_record("q35 layer (64 seqs, head_dim 256, torch fp32 restatement)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res


def test_draft_layer_full_size(fk, parity_record):
    """One full layer of the bench's draft step (32 sequences x 16-row blocks,
    full mask, head_dim 256)."""
    import fekv.workloads as wl
    w = wl.draft(seed=0)
    res = _case(fk, w.hq, w.hkv, w.cached, w.rows, w.bf16, w.causal, 32)
    parity_record("draft layer (32 x 16-row blocks, head_dim 256, torch fp32 restatement)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
