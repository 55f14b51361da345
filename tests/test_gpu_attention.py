"""Paged attention on the GPU through the C ABI against the reference's own
outputs (golden fixtures from src/portable_gpu_ops.cpp), the CPU oracle, and
— at full config sizes the CPU cannot finish quickly — an fp32 torch
restatement of the same ATen algorithm. Tolerance: fe_testutil.ATOL (2e-3)
widened by one output ulp (see fe_testutil)."""
import numpy as np
import pytest

import cases
import oracle
from fe_testutil import (compare_attention, ref_aten_attention, to_device, to_host_bits,
                         torch_reference_attention)

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


def run_case(fk, case, inp, md, causal=None, graph=False):
    import torch
    causal = case.causal if causal is None else causal
    kc, vc = to_device(inp["kpool"], case.bf16), to_device(inp["vpool"], case.bf16)
    fk.store(to_device(inp["knew"], case.bf16), to_device(inp["vnew"], case.bf16), kc, vc,
             _i64(md.slots), md.rows, case.width, case.bf16, None, case.cache_slots)
    plan = fk.AttentionPlan(case.hq, case.hkv, case.dim, case.page, md.batch, case.max_pages(),
                            case.bf16, case.num_blocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last, md.batch, md.rows, graph)
    q = to_device(inp["q"], case.bf16)
    out = torch.full_like(q, float("nan"))
    plan.attention(q, kc, vc, out, causal)
    torch.cuda.synchronize()
    assert fk.device_errors() == 0
    info = plan.info()
    plan.close()
    return to_host_bits(out).reshape(inp["q"].shape), info


@pytest.mark.parametrize("name", [c.name for c in cases.all_cases()])
def test_attention_matches_reference_fixture(fk, parity_record, name):
    case = cases.case_by_name(name)
    fx = dict(np.load(cases.fixture_path(name)))
    inp = case.inputs()
    md = case.metadata()
    out, info = run_case(fk, case, inp, md)
    real = np.arange(md.rows) < int(md.qo[len(case.block_tables)])  # graph-padding rows excluded
    # CPU oracle (float64) for the unrounded comparison
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    _, ref32 = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq,
                                case.hkv, case.dim, case.page, case.causal, case.dtype_code)
    res = compare_attention(out, fx["ref_out"], case.bf16, rows=real, ref_f32=ref32)
    parity_record(f"fixture {name} (reference ATen output)", res)
    assert res["excess"] <= 0, (res, info)
    assert res["excess_vs_f32"] <= 0, (res, info)
    assert np.isfinite(oracle.to_float(out[real], case.dtype_code)).all()


@pytest.mark.parametrize("causal", [True, False])
def test_attention_both_masks_vs_oracle(fk, causal):
    """The same metadata run with either mask (the plan serves both)."""
    case = cases.case_by_name("prefill_causal_bf16")
    inp = case.inputs()
    md = case.metadata()
    out, _ = run_case(fk, case, inp, md, causal=causal)
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    want, want32 = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq,
                                    case.hkv, case.dim, case.page, causal, case.dtype_code)
    res = compare_attention(out, want, case.bf16, ref_f32=want32)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res


@pytest.mark.parametrize("seed", range(10))
def test_attention_random_shapes_vs_oracle(fk, seed):
    rng = np.random.default_rng(1000 + seed)
    hkv = int(rng.choice([1, 2, 4, 8]))
    G = int(rng.choice([1, 2, 3, 4, 6, 8, 16]))
    batch = int(rng.integers(1, 7))
    cached = rng.integers(0, 1200, size=batch)
    rows = np.where(rng.random(batch) < 0.5, 1, rng.integers(1, 40, size=batch))
    bf16, causal = bool(seed % 2), bool(seed % 3 != 0)
    case = cases._case("rand", hkv * G, hkv, cached, rows, bf16, causal, 2000 + seed,
                       page=int(rng.choice([16, 32, 64])))
    inp = case.inputs()
    md = case.metadata()
    out, info = run_case(fk, case, inp, md)
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    want, want32 = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq,
                                    case.hkv, case.dim, case.page, causal, case.dtype_code)
    res = compare_attention(out, want, bf16, ref_f32=want32)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (res, info)


def _full_size(fk, w, layer_seed=0, ref_aten=False):
    """One layer of a BASELINE config at full size, against the fp32 torch
    restatement of the ATen algorithm (pinned on the CPU by
    test_cpu_torch_restatement.py) and, with `ref_aten`, against the
    reference's own ATen path run on the host (oracle/_ref)."""
    import torch
    md = w.metadata()
    g = torch.Generator(device="cuda")
    g.manual_seed(layer_seed)
    dt = torch.bfloat16 if w.bf16 else torch.float16
    kc = (torch.randn(w.cache_slots, w.width, generator=g, device="cuda") * w.scale).to(dt)
    vc = (torch.randn(w.cache_slots, w.width, generator=g, device="cuda") * w.scale).to(dt)
    q = (torch.randn(md.rows, w.hq, w.dim, generator=g, device="cuda") * w.scale).to(dt)
    knew = (torch.randn(md.rows, w.width, generator=g, device="cuda") * w.scale).to(dt)
    vnew = (torch.randn(md.rows, w.width, generator=g, device="cuda") * w.scale).to(dt)
    if w.cow is not None:
        src, dst, ntok = (torch.from_numpy(np.asarray(a, np.int32)).cuda() for a in w.cow)
        fk.copy_blocks([kc], [vc], src, dst, ntok, w.page, w.width, w.num_blocks + 1)
    fk.store(knew, vnew, kc, vc, _i64(md.slots), md.rows, w.width, w.bf16, None, w.cache_slots)
    plan = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(), w.bf16,
                            w.num_blocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last)
    out = torch.empty_like(q)
    plan.attention(q, kc, vc, out, w.causal)
    ref = torch_reference_attention(q, kc, vc, md.qo, md.kv, md.pages, md.last, w.hq, w.hkv,
                                    w.page, w.causal)
    torch.cuda.synchronize()
    assert fk.device_errors() == 0
    ref16 = ref.to(dt)
    out_bits = to_host_bits(out)
    res = compare_attention(out_bits, to_host_bits(ref16), w.bf16, ref_f32=ref.cpu().numpy())
    if ref_aten:
        want = ref_aten_attention(to_host_bits(q), to_host_bits(kc), to_host_bits(vc), md, w.hq,
                                  w.hkv, w.dim, w.page, w.causal, w.bf16, w.num_blocks)
        res["vs_reference"] = compare_attention(out_bits, want, w.bf16)
    info = plan.info()
    plan.close()
    return res, info


def test_c2_layer_full_size(fk, parity_record):
    import fekv.workloads as wl
    res, info = _full_size(fk, wl.c2(seed=0))
    parity_record("C2 layer (64 seqs, torch fp32 restatement)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (res, info)
    assert res["n_over_2e-3"] == 0, res  # |o| is small at this scale: the flat bar holds


def test_c3_layer_full_size(fk, parity_record):
    import fekv.workloads as wl
    res, info = _full_size(fk, wl.c3(seed=0))
    parity_record("C3 layer (4 prefill chunks + 60 decode rows)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (res, info)


def test_c5_long_contexts_vs_reference(fk, parity_record):
    """BASELINE config 5's attention shape (hq64/hkv8, bf16, x0.5) over
    contexts from 2,048 to exactly 32,768 keys (the config's clip range),
    eight sequences over 148 CTAs so every sequence is split-K; checked
    against the reference's own ATen path on the host and the fp32
    restatement."""
    import fekv.workloads as wl
    cached = [2047, 32767, 8191, 5000, 12000, 2048, 20000, 9273]
    w = wl.decode_workload("C5", 64, 8, cached, True, 55, steps=1, scale=0.5, layers=1)
    res, info = _full_size(fk, w, layer_seed=5, ref_aten=True)
    parity_record("C5 shape, 8 seqs, contexts 2,048-32,768 (reference ATen path)", res)
    assert info["split_sequences"] == len(cached), info
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (res, info)
    assert res["vs_reference"]["excess"] <= 0, res
    assert res["n_over_2e-3"] == 0 and res["vs_reference"]["n_over_2e-3"] == 0, res


def test_c5_layer_full_size(fk, parity_record):
    """One layer of a full C5 shard: 128 sequences, log-normal contexts."""
    import fekv.workloads as wl
    w = wl.c5(rank=0, world=1, steps=1)
    res, info = _full_size(fk, w, layer_seed=6)
    parity_record("C5 layer (128 seqs, torch fp32 restatement)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (res, info)
    assert res["n_over_2e-3"] == 0, res


def test_run_lists_parts_equal_one_call(fk):
    """fe_attn_run_lists(decode) then (rows) writes exactly what one fe_attn_run
    does (C3: decode rows and prefill chunks in one step)."""
    import torch
    import fekv.workloads as wl
    w = wl.c3(seed=1)
    md = w.metadata()
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    kc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn(md.rows, w.hq, w.dim, generator=g, device="cuda").to(torch.bfloat16)
    plan = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(), True,
                            w.num_blocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last)
    one, parts = torch.empty_like(q), torch.full_like(q, float("nan"))
    plan.attention(q, kc, vc, one, w.causal)
    plan.attention(q, kc, vc, parts, w.causal, lists=fk._lib.FE_ATTN_LISTS_DECODE)
    plan.attention(q, kc, vc, parts, w.causal, lists=fk._lib.FE_ATTN_LISTS_ROWS)
    torch.cuda.synchronize()
    plan.close()
    assert torch.equal(one.view(torch.int16), parts.view(torch.int16))


def test_c4_layer_full_size(fk, parity_record):
    import fekv.workloads as wl
    res, info = _full_size(fk, wl.c4(seed=0))
    parity_record("C4 layer (128 verify blocks, full mask, CoW tails)", res)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (res, info)


def test_graph_replay_follows_new_metadata(fk):
    """Capture append + attention in a CUDA graph once, then re-prepare with
    different metadata (lengths, splits) and replay: the output tracks the new
    step, as the reference's graph path requires (src/cuda_model.cpp:150-157)."""
    import torch
    import fekv.workloads as wl
    w = wl.decode_workload("g", 16, 4, [100, 900, 2500, 40], True, 7, steps=8)
    dt = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    kc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    vc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    plan = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, w.batch, w.max_pages(8), True,
                            w.num_blocks)
    rows = w.batch
    q = torch.randn(rows, w.hq, w.dim, generator=g, device="cuda").to(dt)
    knew = torch.randn(rows, w.width, generator=g, device="cuda").to(dt)
    vnew = torch.randn(rows, w.width, generator=g, device="cuda").to(dt)
    slots = torch.zeros(rows, dtype=torch.int64, device="cuda")
    out = torch.empty_like(q)
    md0 = w.metadata(0)
    slots.copy_(_i64(md0.slots))
    plan.prepare(md0.qo, md0.kv, md0.pages, md0.last, graph=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fk.store(knew, vnew, kc, vc, slots, rows, w.width, True, s, w.cache_slots)
        plan.attention(q, kc, vc, out, True, s)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        st = torch.cuda.current_stream()
        fk.store(knew, vnew, kc, vc, slots, rows, w.width, True, st, w.cache_slots)
        plan.attention(q, kc, vc, out, True, st)
    for step in range(1, 6):
        md = w.metadata(step)
        slots.copy_(_i64(md.slots))
        q.copy_(torch.randn(rows, w.hq, w.dim, generator=g, device="cuda").to(dt))
        plan.prepare(md.qo, md.kv, md.pages, md.last, graph=True)
        graph.replay()
        ref = torch_reference_attention(q, kc, vc, md.qo, md.kv, md.pages, md.last, w.hq, w.hkv,
                                        w.page, True)
        torch.cuda.synchronize()
        res = compare_attention(to_host_bits(out), to_host_bits(ref.to(dt)), True,
                                ref_f32=ref.cpu().numpy())
        assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (step, res)
    del graph
    plan.close()
    assert fk.device_errors() == 0


def test_graph_replay_prefill_rows_follow_new_split(fk):
    """Prefill rows in a captured graph: the row kernel's Q tensor map is
    encoded once at capture over the step's (fixed) total rows; replays that
    move the sequence boundaries inside those rows and change the contexts
    must follow the new metadata."""
    import torch
    from fekv.metadata import build_step_metadata
    hq, hkv, page, nblocks = 32, 8, 16, 300
    width = hkv * 128
    cache_slots = (nblocks + 1) * page
    rng = np.random.default_rng(5)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    dt = torch.bfloat16
    kc = torch.randn(cache_slots, width, generator=g, device="cuda").to(dt)
    vc = torch.randn(cache_slots, width, generator=g, device="cuda").to(dt)
    tables = [rng.permutation(nblocks)[:100], rng.permutation(nblocks)[:100]]
    cap_rows = 256
    q = torch.randn(cap_rows, hq, 128, generator=g, device="cuda").to(dt)
    out = torch.zeros_like(q)
    plan = fk.AttentionPlan(hq, hkv, 128, page, 2, 100, True, nblocks)
    steps = [([300, 50], [100, 100]), ([700, 120], [190, 10]), ([1000, 5], [37, 163]),
             ([40, 1400], [198, 2]), ([0, 0], [1, 199])]
    md = build_step_metadata(tables, *steps[0], page)
    plan.prepare(md.qo, md.kv, md.pages, md.last, graph=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        plan.attention(q, kc, vc, out, True, s)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        plan.attention(q, kc, vc, out, True, torch.cuda.current_stream())
    for starts, rows in steps:
        md = build_step_metadata(tables, starts, rows, page)
        plan.prepare(md.qo, md.kv, md.pages, md.last, graph=True)
        out.zero_()
        graph.replay()
        n = md.rows
        ref = torch_reference_attention(q[:n], kc, vc, md.qo, md.kv, md.pages, md.last, hq, hkv,
                                         page, True)
        torch.cuda.synchronize()
        res = compare_attention(to_host_bits(out[:n]), to_host_bits(ref.to(dt)), True,
                                ref_f32=ref.cpu().numpy())
        assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (rows, res)
    del graph
    plan.close()
    assert fk.device_errors() == 0


def test_plan_validation_errors(fk):
    plan = fk.AttentionPlan(8, 2, 128, 16, 2, 4, True, 10)
    with pytest.raises(fk.FeError) as e:
        plan.prepare([0, 5], [0, 1], [0], [3])          # 3 keys < 5 query rows
    assert e.value.status == fk._lib.FE_ERR_CONTEXT
    with pytest.raises(fk.FeError) as e:
        plan.prepare([0, 1, 2, 3], [0, 1, 2, 3], [0, 1, 2], [1, 1, 1])  # batch 3 > 2
    assert e.value.status == fk._lib.FE_ERR_CAPACITY
    with pytest.raises(fk.FeError) as e:
        plan.prepare([0, 1], [0, 1], [11], [1])         # page id > num_blocks
    assert e.value.status == fk._lib.FE_ERR_INVALID_ARGUMENT
    with pytest.raises(fk.FeError):
        fk.AttentionPlan(8, 2, 64, 16, 2, 4, True, 10)  # head_dim 64 not compiled
    plan.close()


def test_mixed_step_side_by_side_matches_serial(fk, parity_record):
    """A C3 step (chunked prefill + decode rows) outside graph mode runs the
    decode kernel and the tcgen05 kernel side by side on disjoint SMs (the
    row kernel on the plan's side stream). Its output equals the serial
    full-width run's (a graph-mode prepare): prefill rows bit for bit, decode
    rows within the tolerance (their split points differ). The same call
    captured in a CUDA graph replays to the same bits."""
    import torch
    import fekv.workloads as wl
    w = wl.c3(seed=1000)
    md = w.metadata()
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    dt = torch.bfloat16
    kc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    vc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    q = torch.randn(md.rows, w.hq, w.dim, generator=g, device="cuda").to(dt)
    side = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(), True,
                            w.num_blocks)
    side.prepare(md.qo, md.kv, md.pages, md.last)
    serial = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(), True,
                              w.num_blocks)
    serial.prepare(md.qo, md.kv, md.pages, md.last, graph=True)
    info = side.info()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert info["decode_items"] > 0 and info["prefill_items"] > 0
    assert info["grid_ctas"] <= sms, info  # the two grids share the SMs
    o_side = torch.full_like(q, float("nan"))
    o_serial = torch.full_like(q, float("nan"))
    side.attention(q, kc, vc, o_side, True)
    serial.attention(q, kc, vc, o_serial, True)
    torch.cuda.synchronize()
    qrows = md.qo[1:] - md.qo[:-1]
    is_dec = torch.from_numpy(np.repeat(qrows == 1, qrows)).cuda()
    assert torch.equal(o_side[~is_dec].view(torch.int16), o_serial[~is_dec].view(torch.int16))
    res = compare_attention(to_host_bits(o_side[is_dec]), to_host_bits(o_serial[is_dec]), True)
    parity_record("C3 decode rows: side by side vs serial full width", res)
    assert res["excess"] <= 0, res
    # captured: the fork onto the side stream and the join are part of the graph
    o_graph = torch.full_like(q, float("nan"))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        side.attention(q, kc, vc, o_graph, True, s)
    torch.cuda.current_stream().wait_stream(s)
    o_graph.fill_(float("nan"))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        side.attention(q, kc, vc, o_graph, True, torch.cuda.current_stream())
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(o_graph.view(torch.int16), o_side.view(torch.int16))
    del graph
    side.close()
    serial.close()
    assert fk.device_errors() == 0


def test_empty_step_launches_nothing(fk):
    """batch 0 (an idle step): prepare and attention succeed and write nothing."""
    import torch
    plan = fk.AttentionPlan(8, 2, 128, 16, 4, 8, True, 32)
    plan.prepare([0], [0], [], [])
    q = torch.zeros(4, 8, 128, dtype=torch.bfloat16, device="cuda")
    pool = torch.zeros(33 * 16, 2 * 128, dtype=torch.bfloat16, device="cuda")
    out = torch.full_like(q, 7.0)
    plan.attention(q, pool, pool, out, True)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    assert plan.info()["grid_ctas"] == 0
    plan.close()
    assert fk.device_errors() == 0


@pytest.mark.parametrize("bf16", [True, False])
def test_ragged_batch_with_zero_row_sequences(fk, bf16):
    """Sequences scheduled with no query rows this step (qo[b] == qo[b+1])
    between decode rows and prefill chunks: they are skipped, every other
    row matches the oracle."""
    case = cases._case("ragged", 16, 4, [300, 50, 700, 9, 1200], [1, 0, 33, 0, 1], bf16, True, 77)
    inp = case.inputs()
    md = case.metadata()
    out, info = run_case(fk, case, inp, md)
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    want, want32 = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq,
                                    case.hkv, case.dim, case.page, True, case.dtype_code)
    res = compare_attention(out, want, bf16, ref_f32=want32)
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, (res, info)


def test_step_at_plan_capacity(fk):
    """A step that fills the plan exactly: batch = max_batch and every
    sequence at max_pages pages (the reference's capacity check,
    src/flashinfer_attention.cu:30, accepts it; one more page is refused)."""
    import torch
    from fekv.metadata import build_step_metadata
    batch, max_pages, page = 6, 40, 16
    nblocks = batch * max_pages + 4
    rng = np.random.default_rng(3)
    perm = rng.permutation(nblocks).astype(np.int32)
    tables = [perm[b * max_pages:(b + 1) * max_pages] for b in range(batch)]
    starts = [max_pages * page - 1 - b for b in range(batch)]  # last page, 1..16 tokens
    md = build_step_metadata(tables, starts, [1] * batch, page)
    assert int(md.kv[-1]) == batch * max_pages
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    kc = torch.randn((nblocks + 1) * page, 8 * 128, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn((nblocks + 1) * page, 8 * 128, generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn(batch, 32, 128, generator=g, device="cuda").to(torch.bfloat16)
    plan = fk.AttentionPlan(32, 8, 128, page, batch, max_pages, True, nblocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last)
    out = torch.empty_like(q)
    plan.attention(q, kc, vc, out, True)
    ref = torch_reference_attention(q, kc, vc, md.qo, md.kv, md.pages, md.last, 32, 8, page, True)
    torch.cuda.synchronize()
    res = compare_attention(to_host_bits(out), to_host_bits(ref.to(torch.bfloat16)), True,
                            ref_f32=ref.cpu().numpy())
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    # one page more than a sequence may hold is refused with the capacity status
    big = build_step_metadata([np.concatenate([tables[0], perm[-1:]])] + tables[1:],
                              [max_pages * page] + starts[1:], [1] * batch, page)
    with pytest.raises(fk.FeError) as e:
        plan.prepare(big.qo, big.kv, big.pages, big.last)
    assert e.value.status == fk._lib.FE_ERR_CAPACITY
    plan.close()
    assert fk.device_errors() == 0
