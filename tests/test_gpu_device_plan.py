"""Device-side step preparation (fe_attn_plan_prepare_device,
fe_step_prepare_device) against the host path it replaces.

* The slot mapping is the reference's CudaModel::prepare
  (src/cuda_model.cpp:131-142, padding entries at :138), restated in
  `_host_step` below: slots, positions, qo / kv / pages / last must be equal.
* The decode work list must be the host planner's list item for item (the
  same exact cut), so decode outputs are bit-identical.
* Prefill / verify units are dealt differently (snake order instead of the
  host's least-loaded choice) but each is computed whole by one CTA, so the
  lists hold the same items and the outputs are bit-identical too.
* A captured CUDA graph of device prepare + append + attention replays later
  steps with no host work and matches the eager host-planned path.
"""
import numpy as np
import pytest

from fe_testutil import compare_attention, to_host_bits, torch_reference_attention

pytestmark = pytest.mark.gpu

PAGE = 16


@pytest.fixture(scope="module")
def fk():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import fekv
    fekv.load()
    return fekv


def _dev_i32(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.int32))).cuda()


def _host_step(tables, starts, rps, page, dummy):
    """CudaModel::prepare (src/cuda_model.cpp:131-142) for a graph bucket
    whose entries with start < 0 are padding (:138)."""
    slots, pos, pages, qo, kv, last = [], [], [], [0], [0], []
    for b, st in enumerate(starts):
        st = int(st)
        if st < 0:
            slots += [-1] * rps
            pos += list(range(rps))
            pages.append(dummy)
            last.append(rps)
        else:
            length = st + rps
            for j in range(rps):
                p = st + j
                pos.append(p)
                slots.append(int(tables[b][p // page]) * page + p % page)
            n = -(-length // page)
            pages += [int(x) for x in tables[b][:n]]
            last.append((length - 1) % page + 1)
        qo.append(qo[-1] + rps)
        kv.append(len(pages))
    return (np.array(slots, np.int64), np.array(pos, np.int64), np.array(qo, np.int32),
            np.array(kv, np.int32), np.array(pages, np.int32), np.array(last, np.int32))


GROUP_FIELDS = ["nsplit", "part0", "rec_floats", "rows", "seq", "kvh"]


def _same_list(a, b):
    for key in ("grid", "n_items"):
        assert a[key] == b[key], key
    np.testing.assert_array_equal(a["cta_off"], b["cta_off"])
    np.testing.assert_array_equal(a["items"], b["items"])
    np.testing.assert_array_equal(a["groups"][GROUP_FIELDS], b["groups"][GROUP_FIELDS])


def _same_row_list(dev, host, grid_cap):
    """The same units with the same key ranges (the host may split a unit into
    pieces, the device never does), every CTA range inside the list, balanced."""
    units = {}
    for it in host["items"]:
        units.setdefault((int(it["seq"]), int(it["kvh"]), int(it["rb0"]), int(it["nrb"])), []).append(
            (int(it["kt0"]), int(it["kt1"])))
    assert dev["n_items"] == len(units)
    if not units:
        return
    assert dev["grid"] == grid_cap and host["grid"] == grid_cap
    for it in dev["items"]:
        ranges = sorted(units.pop((int(it["seq"]), int(it["kvh"]), int(it["rb0"]), int(it["nrb"]))))
        assert ranges[0][0] == 0 and ranges[-1][1] == int(it["kt1"]) and int(it["kt0"]) == 0
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert it["part"] == -1 and it["group"] == -1
    assert not units
    off = dev["cta_off"]
    assert off[0] == 0 and off[-1] == dev["n_items"] and np.all(np.diff(off) >= 0)
    # dealt by cost, longest first, in snake order: no CTA exceeds the mean
    # load by more than the largest item (per round the spread is at most the
    # round's first minus last cost, and those telescope)
    cost = ((dev["items"]["kt1"] - dev["items"]["kt0"]) * dev["items"]["nrb"] + 4).astype(np.int64)
    loads = np.array([cost[off[c]:off[c + 1]].sum() for c in range(len(off) - 1)])
    assert loads.max() - loads.mean() <= cost.max() + 1e-9


def _plans(fk, w, md):
    ha = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(4), w.bf16,
                          w.num_blocks)
    da = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(4), w.bf16,
                          w.num_blocks)
    ha.prepare(md.qo, md.kv, md.pages, md.last, graph=True)
    da.prepare_device(_dev_i32(md.qo), _dev_i32(md.kv), _dev_i32(md.pages), _dev_i32(md.last),
                      md.batch, md.rows)
    return ha, da


def _attend_both(fk, w, md, ha, da, causal):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    dt = torch.bfloat16 if w.bf16 else torch.float16
    kc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    vc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    q = torch.randn(md.rows, w.hq, w.dim, generator=g, device="cuda").to(dt)
    oh = torch.full_like(q, float("nan"))
    od = torch.full_like(q, float("nan"))
    ha.attention(q, kc, vc, oh, causal)
    da.attention(q, kc, vc, od, causal)
    torch.cuda.synchronize()
    assert fk.device_errors() == 0
    np.testing.assert_array_equal(to_host_bits(od), to_host_bits(oh))
    assert np.isfinite(od.float().cpu().numpy()).all()


@pytest.mark.parametrize("which", ["c2", "long_mixed", "hkv4"])
def test_device_decode_list_equals_host(fk, which):
    import fekv.workloads as wl
    if which == "c2":
        w = wl.c2(seed=3)
    elif which == "long_mixed":
        w = wl.decode_workload("m", 32, 8, [20000, 17, 3000, 1, 900, 16, 33], True, 5)
    else:
        w = wl.decode_workload("h4", 32, 4, list(np.random.default_rng(2).integers(1, 5000, 40)),
                               False, 9)
    md = w.metadata()
    ha, da = _plans(fk, w, md)
    host = ha.host_meta()
    dev = da.device_meta(total_pages=int(md.kv[-1]))
    assert dev["batch"] == host["batch"] and dev["rows"] == host["rows"]
    np.testing.assert_array_equal(dev["seqs"], host["seqs"])
    np.testing.assert_array_equal(dev["pages"], host["pages"][: int(md.kv[-1])])
    _same_list(dev["views"][2], host["views"][2])
    assert dev["views"][0]["n_items"] == 0 and dev["views"][1]["n_items"] == 0
    _attend_both(fk, w, md, ha, da, True)
    ha.close()
    da.close()


@pytest.mark.parametrize("which", ["c3", "c4"])
def test_device_row_lists_hold_host_items(fk, which):
    import fekv.workloads as wl
    w = wl.c3(seed=2) if which == "c3" else wl.c4(seed=2, batch=32)
    md = w.metadata()
    ha, da = _plans(fk, w, md)
    host = ha.host_meta()
    dev = da.device_meta(total_pages=int(md.kv[-1]))
    np.testing.assert_array_equal(dev["seqs"], host["seqs"])
    np.testing.assert_array_equal(dev["pages"], host["pages"][: int(md.kv[-1])])
    _same_list(dev["views"][2], host["views"][2])
    grid_cap = host["views"][1]["grid"]
    for v in (0, 1):
        _same_row_list(dev["views"][v], host["views"][v], grid_cap)
    for causal in (True, False):
        _attend_both(fk, w, md, ha, da, causal)
    ha.close()
    da.close()


@pytest.mark.parametrize("rps", [1, 3, 16])
def test_step_prepare_device_slot_mapping(fk, rps):
    import torch
    rng = np.random.default_rng(rps)
    batch, stride, nblocks, hq, hkv = 24, 80, 2000, 32, 8
    tables = np.stack([rng.permutation(nblocks)[:stride] for _ in range(batch)]).astype(np.int32)
    starts = rng.integers(0, stride * PAGE - rps - 1, batch).astype(np.int32)
    starts[[3, 7, 23]] = -1  # graph padding entries
    starts[5] = 0
    slots = torch.full((batch * rps,), 12345, dtype=torch.int64, device="cuda")
    pos = torch.full((batch * rps,), 12345, dtype=torch.int64, device="cuda")
    plan = fk.AttentionPlan(hq, hkv, 128, PAGE, batch, stride + 1, True, nblocks)
    plan.step_prepare_device(_dev_i32(tables), _dev_i32(starts), rps, slots, pos)
    torch.cuda.synchronize()
    assert fk.device_errors() == 0
    w_slots, w_pos, qo, kv, pages, last = _host_step(tables, starts, rps, PAGE, nblocks)
    np.testing.assert_array_equal(slots.cpu().numpy(), w_slots)
    np.testing.assert_array_equal(pos.cpu().numpy(), w_pos)
    dev = plan.device_meta(total_pages=int(kv[-1]))
    np.testing.assert_array_equal(dev["pages"], pages)
    seqs = dev["seqs"]
    np.testing.assert_array_equal(seqs["q_row0"], qo[:-1])
    np.testing.assert_array_equal(seqs["qrows"], np.diff(qo))
    np.testing.assert_array_equal(seqs["page_off"], kv[:-1])
    np.testing.assert_array_equal(seqs["length"], (np.diff(kv) - 1) * PAGE + last)
    # and the work lists are those of the restated metadata
    ref = fk.AttentionPlan(hq, hkv, 128, PAGE, batch, stride + 1, True, nblocks)
    ref.prepare(qo, kv, pages, last, graph=True)
    host = ref.host_meta()
    _same_list(dev["views"][2], host["views"][2])
    for v in (0, 1):
        _same_row_list(dev["views"][v], host["views"][v], host["views"][1]["grid"] or 1)
    plan.close()
    ref.close()


def test_step_prepare_device_graph_replay(fk):
    """One captured graph (device prepare, append, attention) replayed over
    several decode steps equals the eager, host-planned step bit for bit."""
    import torch
    rng = np.random.default_rng(21)
    batch, stride, nblocks, hq, hkv = 16, 64, 1100, 32, 8
    width = hkv * 128
    cache_slots = (nblocks + 1) * PAGE
    perm = rng.permutation(nblocks)
    tables = perm[: batch * stride].reshape(batch, stride).astype(np.int32)
    starts0 = rng.integers(0, 900, batch).astype(np.int32)
    starts0[[2, 9]] = -1  # padding entries of the bucket
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    kc = torch.randn(cache_slots, width, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(cache_slots, width, generator=g, device="cuda").to(torch.bfloat16)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    q = torch.zeros(batch, hq, 128, dtype=torch.bfloat16, device="cuda")
    knew = torch.zeros(batch, width, dtype=torch.bfloat16, device="cuda")
    vnew = torch.zeros_like(knew)
    out = torch.empty_like(q)
    tables_d = _dev_i32(tables)
    starts_d = _dev_i32(starts0)
    slots = torch.empty(batch, dtype=torch.int64, device="cuda")
    pos = torch.empty(batch, dtype=torch.int64, device="cuda")
    plan = fk.AttentionPlan(hq, hkv, 128, PAGE, batch, stride + 1, True, nblocks)
    ref = fk.AttentionPlan(hq, hkv, 128, PAGE, batch, stride + 1, True, nblocks)

    def step(stream):
        plan.step_prepare_device(tables_d, starts_d, 1, slots, pos, stream)
        fk.store(knew, vnew, kc, vc, slots, batch, width, True, stream, cache_slots)
        plan.attention(q, kc, vc, out, True, stream)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(s)  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    kc.copy_(kc_ref)
    vc.copy_(vc_ref)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(torch.cuda.current_stream())
    starts = starts0.copy()
    for it in range(4):
        q.copy_(torch.randn(batch, hq, 128, generator=g, device="cuda").to(torch.bfloat16))
        knew.copy_(torch.randn(batch, width, generator=g, device="cuda").to(torch.bfloat16))
        vnew.copy_(torch.randn(batch, width, generator=g, device="cuda").to(torch.bfloat16))
        starts_d.copy_(_dev_i32(starts))
        graph.replay()
        # eager reference step: host slot mapping, host plan
        w_slots, _, qo, kv, pages, last = _host_step(tables, starts, 1, PAGE, nblocks)
        fk.store(knew, vnew, kc_ref, vc_ref, torch.from_numpy(w_slots).cuda(), batch, width, True,
                 None, cache_slots)
        ref.prepare(qo, kv, pages, last)
        want = torch.empty_like(out)
        ref.attention(q, kc_ref, vc_ref, want, True)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(to_host_bits(kc), to_host_bits(kc_ref))
        np.testing.assert_array_equal(to_host_bits(vc), to_host_bits(vc_ref))
        np.testing.assert_array_equal(to_host_bits(out), to_host_bits(want))
        starts = np.where(starts >= 0, starts + 1 + it * 7, -1).astype(np.int32)
    del graph
    plan.close()
    ref.close()
    assert fk.device_errors() == 0


def test_device_prepare_invalid_metadata_empties_plan(fk):
    """A page id past the padding page: the device planner cannot fail the
    call, so it empties the plan and raises FE_DEVERR_PLAN; attention then
    writes nothing. A later valid prepare recovers."""
    import torch
    from fekv._lib import FE_DEVERR_PLAN
    import fekv.workloads as wl
    w = wl.decode_workload("bad", 16, 8, [100, 300, 40], True, 1)
    md = w.metadata()
    pages = md.pages.copy()
    pages[4] = w.num_blocks + 1
    plan = fk.AttentionPlan(w.hq, w.hkv, w.dim, w.page, md.batch, w.max_pages(), True,
                            w.num_blocks)
    plan.prepare_device(_dev_i32(md.qo), _dev_i32(md.kv), _dev_i32(pages), _dev_i32(md.last),
                        md.batch, md.rows)
    kc = torch.zeros(w.cache_slots, w.width, dtype=torch.bfloat16, device="cuda")
    q = torch.ones(md.rows, w.hq, w.dim, dtype=torch.bfloat16, device="cuda")
    out = torch.full_like(q, 7.0)
    plan.attention(q, kc, kc, out, True)
    torch.cuda.synchronize()
    assert fk.device_errors() == FE_DEVERR_PLAN
    assert (out == 7.0).all()
    plan.prepare_device(_dev_i32(md.qo), _dev_i32(md.kv), _dev_i32(md.pages), _dev_i32(md.last),
                        md.batch, md.rows)
    plan.attention(q, kc, kc, out, True)
    torch.cuda.synchronize()
    assert fk.device_errors() == 0
    assert not (out == 7.0).any()
    plan.close()


@pytest.mark.parametrize("which", ["q35", "mixed"])
def test_device_decode_list_equals_host_head_dim_256(fk, which):
    """head_dim 256 plans: the device-built decode list is the host's item for
    item (two KV heads per item, split records of rows x 258 floats), so the
    outputs are the same bits."""
    import fekv.workloads as wl
    if which == "q35":
        w = wl.q35(seed=4)
    else:
        w = wl.decode_workload("m256", 16, 2, [9000, 17, 3000, 1, 900, 16, 33], True, 6, dim=256)
    md = w.metadata()
    ha, da = _plans(fk, w, md)
    host = ha.host_meta()
    dev = da.device_meta(total_pages=int(md.kv[-1]))
    np.testing.assert_array_equal(dev["seqs"], host["seqs"])
    _same_list(dev["views"][2], host["views"][2])
    assert (host["views"][2]["groups"]["nsplit"] > 1).any()
    _attend_both(fk, w, md, ha, da, True)
    ha.close()
    da.close()


@pytest.mark.parametrize("causal", [True, False])
def test_device_row_lists_head_dim_256(fk, causal):
    """head_dim 256 draft blocks: the device planner deals whole 128-row items
    (the host cuts them into pieces across CTAs); both outputs match the fp32
    restatement of the reference's attention."""
    import torch
    import fekv.workloads as wl
    w = wl.draft(seed=3, batch=6)
    md = w.metadata()
    ha, da = _plans(fk, w, md)
    host = ha.host_meta()
    dev = da.device_meta(total_pages=int(md.kv[-1]))
    view = 1 if causal else 0
    _same_row_list(dev["views"][view], host["views"][view], dev["views"][view]["grid"])
    assert len(host["views"][view]["groups"]) > 0  # the host split some items
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    dt = torch.bfloat16
    kc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    vc = torch.randn(w.cache_slots, w.width, generator=g, device="cuda").to(dt)
    q = torch.randn(md.rows, w.hq, w.dim, generator=g, device="cuda").to(dt)
    ref = torch_reference_attention(q, kc, vc, md.qo, md.kv, md.pages, md.last, w.hq, w.hkv,
                                    w.page, causal)
    for plan in (ha, da):
        out = torch.full_like(q, float("nan"))
        plan.attention(q, kc, vc, out, causal)
        torch.cuda.synchronize()
        assert fk.device_errors() == 0
        res = compare_attention(to_host_bits(out), to_host_bits(ref.to(dt)), True,
                                ref_f32=ref.cpu().numpy())
        assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    ha.close()
    da.close()
