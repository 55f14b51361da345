"""Host work planner (fe_attn_plan.cpp) without a GPU: every (sequence, KV
head, packed query row, key tile) the attention needs is covered exactly
once by the work lists, split units are consistent, CTAs are balanced, and
bad metadata is rejected with the reference's error classes."""
import numpy as np
import pytest

import cases
import fekv
from fekv import HostPlan, workloads
from fekv import _lib


def _plan(w_or_case, grid_cap=296, graph=False):
    md = w_or_case.metadata()
    hp = HostPlan(w_or_case.hq, w_or_case.hkv, 128, w_or_case.page, md.batch,
                  int((md.kv[1:] - md.kv[:-1]).max()) + 1, w_or_case.bf16, w_or_case.num_blocks,
                  grid_cap=grid_cap)
    return md, hp.prepare(md.qo, md.kv, md.pages, md.last, graph=graph), hp


def _coverage(md, meta, hq, hkv, page, causal):
    """Count how many times each (seq, kv head, packed row, tile) is visited."""
    G = hq // hkv
    H = meta["dec_heads"]
    lengths = md.lengths(page)
    qrows = md.qo[1:] - md.qo[:-1]
    seen = {}
    lists = [meta["views"][1 if causal else 0], meta["views"][2]]
    for li, v in enumerate(lists):
        for it in v["items"]:
            b = int(it["seq"])
            heads = range(int(it["kvh"]), int(it["kvh"]) + (H if li == 1 else 1))
            P = int(qrows[b]) * G
            rows = range(int(it["rb0"]) * 16, min(P, (int(it["rb0"]) + int(it["nrb"])) * 16))
            for h in heads:
                for p in rows:
                    for t in range(int(it["kt0"]), int(it["kt1"])):
                        key = (b, h, p, t)
                        seen[key] = seen.get(key, 0) + 1
    # every needed tile exactly once
    for b in range(md.batch):
        P = int(qrows[b]) * G
        for h in range(hkv):
            for p in range(P):
                i = p // G
                limit = int(lengths[b]) - int(qrows[b]) + i + 1 if causal else int(lengths[b])
                need = -(-limit // 16)
                for t in range(need):
                    assert seen.pop((b, h, p, t), 0) == 1, (b, h, p, t)
    # anything left over must lie beyond the causal limit of its row (row
    # blocks share a key range) -- never beyond the sequence itself
    for (b, h, p, t), n in seen.items():
        assert n == 1
        assert t * 16 < lengths[b], (b, h, p, t)


@pytest.mark.parametrize("name", [c.name for c in cases.all_cases()])
@pytest.mark.parametrize("causal", [True, False])
def test_work_lists_cover_each_tile_once(name, causal):
    case = cases.case_by_name(name)
    md, meta, _ = _plan(case, grid_cap=8)
    _coverage(md, meta, case.hq, case.hkv, case.page, causal)


@pytest.mark.parametrize("maker", [workloads.c1, workloads.c2, workloads.c3, workloads.c4])
def test_configs_plan_and_balance(maker):
    w = maker()
    md, meta, _ = _plan(w)
    dec = meta["views"][2]
    if len(dec["items"]):
        co = dec["cta_off"]
        loads = [int((dec["items"][co[g]:co[g + 1]]["kt1"] - dec["items"][co[g]:co[g + 1]]["kt0"]).sum())
                 for g in range(dec["grid"])]
        # exact cut: all CTAs but the last stream the same number of tiles
        assert max(loads[:-1]) - min(loads[:-1]) <= 0 if len(loads) > 1 else True
        assert dec["grid"] <= 148
    for v in meta["views"]:
        for it in v["items"]:
            assert it["kt1"] > it["kt0"]


def test_split_groups_are_consistent():
    w = workloads.c5(steps=1)
    md, meta, _ = _plan(w)
    for v in meta["views"]:
        groups = v["groups"]
        by_group = {}
        for it in v["items"]:
            if it["group"] >= 0:
                by_group.setdefault(int(it["group"]), []).append(it)
            else:
                assert it["part"] == -1
        for gid, its in by_group.items():
            gi = groups[gid]
            assert gi["nsplit"] == len(its)
            parts = sorted(int(i["part"]) for i in its)
            assert parts == [int(gi["part0"]) + s * int(gi["rec_floats"]) for s in range(len(its))]
            ranges = sorted((int(i["kt0"]), int(i["kt1"])) for i in its)
            for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                assert a1 == b0
    # partial records of different groups never overlap
    recs = []
    for v in meta["views"]:
        for gi in v["groups"]:
            if gi["nsplit"]:
                recs.append((int(gi["part0"]), int(gi["part0"]) + int(gi["nsplit"]) * int(gi["rec_floats"])))
    recs = sorted(set(recs))
    for (a0, a1), (b0, b1) in zip(recs, recs[1:]):
        assert a1 <= b0


def test_graph_mode_uses_full_grid():
    w = workloads.c2()
    _, meta, _ = _plan(w, graph=True)
    assert meta["views"][2]["grid"] == 148


def _err(fn):
    with pytest.raises(fekv.FeError) as e:
        fn()
    return e.value.status


def test_validation_matches_reference_error_classes():
    hp = HostPlan(8, 2, 128, 16, 2, 4, True, 10, grid_cap=8)
    # src/portable_gpu_ops.cpp:30 -- fewer keys than query rows
    assert _err(lambda: hp.prepare([0, 5], [0, 1], [0], [3])) == _lib.FE_ERR_CONTEXT
    # src/flashinfer_attention.cu:30 -- batch beyond the plan
    assert _err(lambda: hp.prepare([0, 1, 2, 3], [0, 1, 2, 3], [0, 1, 2], [1, 1, 1])) == \
        _lib.FE_ERR_CAPACITY
    # page id out of [0, num_blocks]
    assert _err(lambda: hp.prepare([0, 1], [0, 1], [11], [1])) == _lib.FE_ERR_INVALID_ARGUMENT
    assert _err(lambda: hp.prepare([0, 1], [0, 1], [-1], [1])) == _lib.FE_ERR_INVALID_ARGUMENT
    # last outside [1, page]
    assert _err(lambda: hp.prepare([0, 1], [0, 1], [0], [17])) == _lib.FE_ERR_INVALID_ARGUMENT
    assert _err(lambda: hp.prepare([0, 1], [0, 1], [0], [0])) == _lib.FE_ERR_INVALID_ARGUMENT
    # more pages than max_pages
    assert _err(lambda: hp.prepare([0, 1], [0, 5], [0, 1, 2, 3, 4], [1])) == _lib.FE_ERR_CAPACITY
    # qo[batch] must equal rows
    assert _err(lambda: hp.prepare([0, 1], [0, 1], [0], [1], rows=2)) == _lib.FE_ERR_INVALID_ARGUMENT
    # the dummy page (num_blocks) is a valid page id (graph padding)
    hp.prepare([0, 1], [0, 1], [10], [1])
    # empty batch is a no-op
    meta = hp.prepare([0], [0], [], [])
    assert all(len(v["items"]) == 0 for v in meta["views"])


def test_zero_row_sequences_are_skipped():
    hp = HostPlan(8, 2, 128, 16, 3, 4, True, 10, grid_cap=8)
    meta = hp.prepare([0, 0, 1, 1], [0, 1, 2, 3], [0, 1, 2], [5, 5, 5])
    seqs = [int(it["seq"]) for v in meta["views"] for it in v["items"]]
    assert set(seqs) == {1}


def _wide_units_covered(view, md, G, causal):
    """Every (sequence, KV head, 128-row block) of the multi-block sequences
    is on the list once per key tile of its mask's range, pieces contiguous."""
    items = view["items"]
    q = np.diff(md.qo)
    L = md.lengths(16)
    for b in range(len(q)):
        P = int(q[b]) * G
        if P <= 16:
            assert not (items["seq"] == b).any()
            continue
        for h in range(2):
            for rb0 in range(0, -(-P // 16), 8):
                its = items[(items["seq"] == b) & (items["kvh"] == h) & (items["rb0"] == rb0)]
                its = np.sort(its, order="kt0")
                last_row = min(P, (rb0 + 8) * 16) - 1
                keys = int(L[b]) - int(q[b]) + last_row // G + 1 if causal else int(L[b])
                assert len(its) >= 1 and (its["key_mode"] == 0).all()
                assert its["kt0"][0] == 0 and its["kt1"][-1] == -(-keys // 16)
                assert (its["kt0"][1:] == its["kt1"][:-1]).all()
                assert (its["nrb"] == min(8, -(-P // 16) - rb0)).all()


def test_head_dim_256_plan_lists():
    """head_dim 256 plans put every (sequence, KV head, 128-row block) of the
    multi-block sequences on the row lists for the tcgen05 kernel, with each
    mask's key range; sequences whose packed rows fit one 16-row block go to
    the decode list (two KV heads per item), cut exactly like head_dim 128,
    with split records of rows x (256 + 2) floats."""
    # a decode row, a 100-row chunk, a 3-row block and a long decode row
    from fekv.metadata import build_step_metadata
    tables = [np.arange(i * 400, i * 400 + 400) for i in range(4)]
    md = build_step_metadata(tables, [40, 2900, 700, 6000], [1, 100, 3, 1], 16)
    hp = HostPlan(16, 2, 256, 16, 4, 400, True, 1600, grid_cap=8)
    meta = hp.prepare(md.qo, md.kv, md.pages, md.last)
    G = 8
    v0, v1, v2 = meta["views"]
    _wide_units_covered(v0, md, G, causal=False)
    _wide_units_covered(v1, md, G, causal=True)
    for v in (v0, v1):
        assert v["grid"] <= 8 and len(v["cta_off"]) == v["grid"] + 1
        assert v["cta_off"][-1] == len(v["items"]) and (np.diff(v["cta_off"]) >= 0).all()
    # decode list: both KV heads in one unit, key tiles covered exactly once
    it2 = v2["items"]
    assert set(it2["seq"]) == {0, 3} and (it2["kvh"] == 0).all() and (it2["key_mode"] == 1).all()
    for b in (0, 3):
        its = np.sort(it2[it2["seq"] == b], order="kt0")
        tiles = -(-((int(md.kv[b + 1] - md.kv[b]) - 1) * 16 + int(md.last[b])) // 16)
        assert its["kt0"][0] == 0 and its["kt1"][-1] == tiles
        assert (its["kt0"][1:] == its["kt1"][:-1]).all()
    split = v2["groups"][v2["groups"]["nsplit"] > 1]
    assert len(split) >= 1
    for gi in split:
        assert gi["rows"] == 2 * G and gi["rec_floats"] == (2 * G * 258 + 3) // 4 * 4
        assert gi["row0"] == 0 and gi["rows_per_head"] == 0
    hp.close()


def test_head_dim_256_draft_blocks_are_split():
    """DFlash-style draft blocks (16 rows over long contexts) give too few
    128-row items to fill the GPU: the row lists are cut into equal tile
    ranges per CTA, and units cut in pieces write records (one KV head, the
    unit's rows) that the merge kernel maps back with row0 / rows_per_head."""
    from fekv.metadata import build_step_metadata
    tables = [np.arange(i * 200, i * 200 + 200) for i in range(2)]
    md = build_step_metadata(tables, [3000, 2500], [16, 16], 16)
    hp = HostPlan(16, 2, 256, 16, 2, 200, True, 400, grid_cap=148)
    meta = hp.prepare(md.qo, md.kv, md.pages, md.last)
    G = 8
    for causal, v in ((False, meta["views"][0]), (True, meta["views"][1])):
        _wide_units_covered(v, md, G, causal)
        it = v["items"]
        assert len(it) > 4  # 2 seqs x 2 KV heads x 1 row item, split
        split = it[it["part"] >= 0]
        assert len(split) >= 1
        # exact cut: every CTA but the last streams the same number of tiles
        co = v["cta_off"]
        loads = [int((it[co[c]:co[c + 1]]["kt1"] - it[co[c]:co[c + 1]]["kt0"]).sum())
                 for c in range(v["grid"])]
        assert v["grid"] <= 148 and max(loads[:-1]) == min(loads[:-1]) >= 16
        for gi in v["groups"]:
            assert gi["nsplit"] >= 2 and gi["rows"] == 128
            assert gi["row0"] == 0 and gi["rows_per_head"] == 128
            assert gi["rec_floats"] == 128 * 258
        # every piece's record lies inside its group's records
        for x in split:
            gi = v["groups"][x["group"]]
            assert gi["part0"] <= x["part"] < gi["part0"] + gi["nsplit"] * gi["rec_floats"]
            assert (x["part"] - gi["part0"]) % gi["rec_floats"] == 0
    assert len(meta["views"][2]["items"]) == 0
    hp.close()


def test_mixed_step_splits_the_sms_between_the_kernels():
    """C3 (chunked prefill + decode rows): outside graph mode the decode
    list gets part of the SMs and the row list the rest, so the two kernels
    run side by side; every tile is still covered once. Graph mode and
    single-list steps keep the full width."""
    w = workloads.c3(seed=1000)
    # a host plan with grid_cap 296 models 148 SMs (two row CTAs per SM)
    md, meta, hp = _plan(w, grid_cap=296)
    sms = 148
    dec, rows = meta["views"][2]["grid"], meta["views"][1]["grid"]
    assert 8 <= dec <= 80, dec
    assert rows == (sms - dec) * 2, (dec, rows)
    hp.close()
    _coverage(md, meta, w.hq, w.hkv, w.page, True)
    _coverage(md, meta, w.hq, w.hkv, w.page, False)
    md, meta, hp = _plan(w, grid_cap=296, graph=True)
    assert meta["views"][2]["grid"] == sms and meta["views"][1]["grid"] == 296
    hp.close()
    for single in (workloads.c2_shard(0), workloads.c4(seed=0)):
        md, meta, hp = _plan(single, grid_cap=296)
        assert meta["views"][2]["grid"] in (0, min(sms, meta["views"][2]["grid"]))
        assert meta["views"][2]["grid"] in (0, 148) or meta["views"][1]["grid"] == 0
        assert meta["views"][1]["grid"] in (0, 296)
        hp.close()


def test_mixed_step_with_a_tiny_decode_part_stays_serial_or_balances():
    """One short decode row beside a large prefill: whatever the split, the
    decode list gets at least one CTA and the row list keeps most SMs."""
    from fekv.metadata import build_step_metadata
    tables = [np.arange(0, 200), np.arange(200, 203)]
    md = build_step_metadata(tables, [1000, 40], [1024, 1], 16)
    hp = HostPlan(32, 8, 128, 16, 2, 200, True, 300, grid_cap=296)
    meta = hp.prepare(md.qo, md.kv, md.pages, md.last)
    dec, rows = meta["views"][2]["grid"], meta["views"][1]["grid"]
    items = len(meta["views"][1]["items"])  # 256 row items: one CTA each
    assert dec >= 1 and rows >= min(items, 2 * 140), (dec, rows)
    hp.close()
