"""The CPU oracle (oracle/fe_oracle.c) pinned against the reference's own
outputs: the golden fixtures made by running FlashEngine.cpp's ATen path
(src/portable_gpu_ops.cpp) and, where oracle/_ref is built, the reference
library live on fresh random cases."""
import hashlib

import numpy as np
import pytest

import cases
import oracle
from fe_testutil import compare_attention

ALL = [c.name for c in cases.all_cases()]


def _fixture(name):
    return dict(np.load(cases.fixture_path(name)))


def test_half_conversion_matches_numpy():
    lib = oracle.c_oracle()
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * 10 ** rng.uniform(-8, 5, 2000).astype(np.float32),
        np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e9, -1e9, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8,
                  1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, np.inf, -np.inf], dtype=np.float32),
    ])
    for x in vals:
        want = np.float32(x).astype(np.float16).view(np.uint16)
        got = lib.fe_oracle_float_to_half(float(x))
        assert got == want, (x, got, want)
        back = lib.fe_oracle_half_to_float(int(want))
        assert np.float32(back) == np.float16(np.float32(x)).astype(np.float32) or np.isnan(back)
    # every half pattern round-trips
    for h in range(0, 1 << 16, 7):
        f = lib.fe_oracle_half_to_float(h)
        if not np.isnan(f):
            assert lib.fe_oracle_float_to_half(f) == h


def test_bf16_conversion_matches_torch():
    torch = pytest.importorskip("torch")
    lib = oracle.c_oracle()
    rng = np.random.default_rng(1)
    vals = (rng.standard_normal(4000) * 10 ** rng.uniform(-30, 30, 4000)).astype(np.float32)
    vals = np.concatenate([vals, np.array([0, -0.0, 1 + 2 ** -8, 1 + 3 * 2 ** -8, 3.4e38,
                                           np.inf, -np.inf], dtype=np.float32)])
    want = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([lib.fe_oracle_float_to_bf16(float(x)) for x in vals], dtype=np.uint16)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(oracle.from_float(vals, 1), want)


@pytest.mark.parametrize("name", ALL)
def test_inputs_reproduce_fixture(name):
    case = cases.case_by_name(name)
    fx = _fixture(name)
    inp = case.inputs()
    assert cases.input_digest(inp) == str(fx["input_sha256"]), "seeded input generator drifted"
    md = case.metadata()
    for key, arr in (("meta_qo", md.qo), ("meta_kv", md.kv), ("meta_pages", md.pages),
                     ("meta_last", md.last), ("meta_slots", md.slots)):
        np.testing.assert_array_equal(fx[key], arr)


@pytest.mark.parametrize("name", ALL)
def test_oracle_append_bit_exact_vs_reference(name):
    """Append with the ATen variant's redirect of slot<0 rows reproduces the
    reference pools bit for bit; with the CUDA kernel's skip semantics every
    page but the padding page is identical."""
    case = cases.case_by_name(name)
    fx = _fixture(name)
    inp = case.inputs()
    md = case.metadata()
    k, v = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], k, v, md.slots, case.cache_slots, redirect_negative=True)
    assert hashlib.sha256(k.tobytes()).hexdigest() == str(fx["ref_k_sha256"])
    assert hashlib.sha256(v.tobytes()).hexdigest() == str(fx["ref_v_sha256"])
    ks, vs = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ks, vs, md.slots, case.cache_slots)
    pad0 = case.num_blocks * case.page
    np.testing.assert_array_equal(ks[:pad0], k[:pad0])
    np.testing.assert_array_equal(vs[:pad0], v[:pad0])
    if (md.slots < 0).any():
        assert (ks[pad0:] == 0).all(), "skip semantics must leave the padding page untouched"


@pytest.mark.parametrize("name", ALL)
def test_oracle_attention_vs_reference(name):
    case = cases.case_by_name(name)
    fx = _fixture(name)
    inp = case.inputs()
    md = case.metadata()
    k, v = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], k, v, md.slots, case.cache_slots, redirect_negative=True)
    out, out32 = oracle.attention(inp["q"], k, v, md.qo, md.kv, md.pages, md.last, case.hq,
                                  case.hkv, case.dim, case.page, case.causal, case.dtype_code)
    res = compare_attention(out, fx["ref_out"], case.bf16)
    assert res["excess"] <= 0, res
    # the restatement is float64 throughout: it rounds to the same 16-bit value
    # as the float32 reference almost everywhere
    assert res["exact_frac"] > 0.99, res


def test_oracle_gather_matches_slot_formula():
    case = cases.case_by_name("prefill_causal_bf16")
    inp = case.inputs()
    md = case.metadata()
    dense = oracle.gather(inp["kpool"], md.kv, md.pages, md.last, case.page, case.width)
    lengths = md.lengths(case.page)
    row = 0
    for b, n in enumerate(lengths):
        t = np.arange(n)
        slots = md.pages[md.kv[b] + t // case.page].astype(np.int64) * case.page + t % case.page
        np.testing.assert_array_equal(dense[row:row + n], inp["kpool"][slots])
        row += n
    assert row == dense.shape[0]


def test_oracle_copy_blocks_is_memcpy():
    rng = np.random.default_rng(3)
    page, width, pages = 16, 256, 12
    pools = [rng.integers(0, 65535, size=(pages * page, width), dtype=np.uint16) for _ in range(4)]
    before = [p.copy() for p in pools]
    src, dst, ntok = [1, 5, 7], [2, 9, 0], [16, 3, 0]
    oracle.copy_blocks(pools[:2], pools[2:], src, dst, ntok, page, width)
    for i, p in enumerate(pools):
        want = before[i].copy()
        for s, d, n in zip(src, dst, ntok):
            want[d * page:d * page + n] = before[i][s * page:s * page + n]
        np.testing.assert_array_equal(p, want)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("seed", range(4))
def test_oracle_vs_reference_live(seed):
    """Fresh random shapes through both checkers: the C restatement and the
    reference library itself."""
    rng = np.random.default_rng(100 + seed)
    hkv = int(rng.choice([1, 2, 4]))
    G = int(rng.choice([1, 2, 4, 8]))
    batch = int(rng.integers(1, 5))
    cached = rng.integers(0, 300, size=batch)
    rows = rng.integers(1, 24, size=batch)
    case = cases._case("live", hkv * G, hkv, cached, rows, bool(seed % 2), bool(seed < 3), seed)
    inp = case.inputs()
    md = case.metadata()
    ref = oracle.RefAten(case.hq, case.hkv, case.dim, case.page, md.batch, case.max_pages(),
                         case.bf16, case.num_blocks)
    kr, vr = inp["kpool"].copy(), inp["vpool"].copy()
    ref.store(inp["knew"], inp["vnew"], kr, vr, md.slots)
    ref.prepare(md.qo, md.kv, md.pages, md.last)
    want = ref.attention(inp["q"], kr, vr, case.causal)
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    np.testing.assert_array_equal(ko, kr)
    np.testing.assert_array_equal(vo, vr)
    got, _ = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq, case.hkv,
                              case.dim, case.page, case.causal, case.dtype_code)
    res = compare_attention(got, want, case.bf16)
    assert res["excess"] <= 0, res


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
def test_reference_error_behaviour():
    """The reference throws when a sequence has fewer keys than query rows
    and when the batch exceeds the plan; the C-ABI maps these to
    FE_ERR_CONTEXT / FE_ERR_CAPACITY (tested in test_cpu_planner)."""
    ref = oracle.RefAten(4, 2, 128, 16, 2, 4, True, 8)
    with pytest.raises(oracle.RefError):
        ref.prepare([0, 5], [0, 1], [0], [3])  # length 3 < 5 rows
    with pytest.raises(oracle.RefError):
        ref.prepare([0, 1, 2, 3], [0, 1, 2, 3], [0, 1, 2], [1, 1, 1])  # batch 3 > max 2
