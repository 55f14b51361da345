"""Paged attention at extreme score ranges, through the C ABI, against the CPU
oracle (the restatement of src/portable_gpu_ops.cpp:39-44, pinned by the
reference's golden fixtures), with the tolerance of fe_testutil (2e-3 plus
one output ulp against the 16-bit reference, 2e-3 plus half an ulp against
fp32).

- Large logits: q, K and V drawn N(0, s^2) with s = 2 or 4, so the scaled
  scores have a standard deviation of s^2 and each row's weights are peaked
  on a few keys; the online softmax rescales whenever a later tile holds a
  larger score.
- Late needles: for each sequence, one key late in its context is set to a
  multiple of one query head's vector, so that head's maximum first appears
  tens of tiles after the running maximum was fixed, and nearly all of the
  row's weight moves to it; another head sees a needle at the first key.
- NaN outside the sequences: every pool slot that holds none of the step's
  keys (the rest of each last page, unused pages) is NaN in K and V.
Shapes cover the decode kernel (one query row per sequence, GQA 4 and 8),
the tcgen05 kernel (verify blocks with the full mask, causal prefill
chunks) and both 16-bit types.
"""
import numpy as np
import pytest

import cases
import oracle
from fe_testutil import compare_attention, to_device, to_host_bits

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


def _run(fk, case, inp, md):
    import torch
    kc, vc = to_device(inp["kpool"], case.bf16), to_device(inp["vpool"], case.bf16)
    fk.store(to_device(inp["knew"], case.bf16), to_device(inp["vnew"], case.bf16), kc, vc,
             _i64(md.slots), md.rows, case.width, case.bf16, None, case.cache_slots)
    plan = fk.AttentionPlan(case.hq, case.hkv, case.dim, case.page, md.batch, case.max_pages(),
                            case.bf16, case.num_blocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last)
    q = to_device(inp["q"], case.bf16)
    out = torch.full_like(q, float("nan"))
    plan.attention(q, kc, vc, out, case.causal)
    torch.cuda.synchronize()
    assert fk.device_errors() == 0
    plan.close()
    return to_host_bits(out).reshape(inp["q"].shape)


def _check(fk, case, inp, md):
    out = _run(fk, case, inp, md)
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    want, want32 = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq,
                                    case.hkv, case.dim, case.page, case.causal, case.dtype_code)
    res = compare_attention(out, want, case.bf16, ref_f32=want32)
    assert np.isfinite(oracle.to_float(out, case.dtype_code)).all()
    assert res["excess"] <= 0 and res["excess_vs_f32"] <= 0, res
    return res


# (name, hq, hkv, cached, rows, causal): decode rows, verify blocks, prefill chunks
SHAPES = [
    ("decode_g4", 32, 8, [700, 2100, 95, 1500], [1, 1, 1, 1], True),
    ("decode_g8", 16, 2, [3000, 41, 1200], [1, 1, 1], True),
    ("verify_full_g8", 32, 4, [900, 2000, 300], [16, 16, 16], False),
    ("prefill_causal_g4", 16, 4, [0, 600, 1500], [300, 200, 129], True),
]


@pytest.mark.parametrize("scale", [2.0, 4.0])
@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("shape", SHAPES, ids=[s[0] for s in SHAPES])
def test_large_logits_vs_oracle(fk, parity_record, shape, bf16, scale):
    name, hq, hkv, cached, rows, causal = shape
    seed = 7000 + SHAPES.index(shape) * 10 + int(scale) + (0 if bf16 else 5)
    case = cases._case(f"{name}_s{scale}", hq, hkv, cached, rows, bf16, causal, seed,
                       scale=scale)
    res = _check(fk, case, case.inputs(), case.metadata())
    parity_record(f"large logits {name} scale {scale} {'bf16' if bf16 else 'f16'}", res)


def _plant_needles(case, inp, md, factor):
    """Per sequence: key position ~90% into the cached context of KV head 0
    becomes `factor` x the query vector of head 0 of the sequence's last query
    row, and key 0 of the last KV head becomes `factor` x that row's query of
    the last head (in the 16-bit type; values stay well inside its range)."""
    dt = case.dtype_code
    q = oracle.to_float(inp["q"], dt)
    kpool = oracle.to_float(inp["kpool"], dt)
    G = case.hq // case.hkv
    for b, table in enumerate(case.block_tables):
        row = int(md.qo[b + 1]) - 1
        n = int(case.cached[b])
        if n < 2:
            continue
        for pos, kvh in ((int(0.9 * (n - 1)), 0), (0, case.hkv - 1)):
            slot = int(table[pos // case.page]) * case.page + pos % case.page
            head = kvh * G
            kpool[slot, kvh * case.dim:(kvh + 1) * case.dim] = factor * q[row, head]
    inp["kpool"] = oracle.from_float(kpool, dt)
    return inp


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("shape", SHAPES, ids=[s[0] for s in SHAPES])
def test_late_needles_vs_oracle(fk, parity_record, shape, bf16):
    name, hq, hkv, cached, rows, causal = shape
    seed = 7500 + SHAPES.index(shape) + (0 if bf16 else 50)
    case = cases._case(f"{name}_needle", hq, hkv, cached, rows, bf16, causal, seed)
    md = case.metadata()
    # scores of the needle: |q|^2 x 3 / sqrt(128) ~ 34 in natural-log units
    # above the others' spread (N(0,1) inputs), i.e. ~49 in the kernels' base 2
    inp = _plant_needles(case, case.inputs(), md, 3.0)
    res = _check(fk, case, inp, md)
    parity_record(f"late needles {name} {'bf16' if bf16 else 'f16'}", res)


def _poison_unused_slots(case, inp):
    """Every pool slot outside the sequences' cached keys becomes NaN in K
    and V (the rest of each last page, unused pages); the step's appends
    then overwrite their own slots. The kernels read whole 16-token tiles
    and must give those keys no weight and let none of their V in."""
    nan = np.uint16(0x7FC0 if case.bf16 else 0x7E00)
    used = np.zeros(case.cache_slots, bool)
    for b, table in enumerate(case.block_tables):
        pos = np.arange(int(case.cached[b]))
        used[np.asarray(table, np.int64)[pos // case.page] * case.page + pos % case.page] = True
    used[case.num_blocks * case.page:] = True  # the padding page stays zero
    for key in ("kpool", "vpool"):
        inp[key] = inp[key].copy()
        inp[key][~used] = nan
    return inp


@pytest.mark.parametrize("page", [16, 32])
@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("shape", SHAPES, ids=[s[0] for s in SHAPES])
def test_nan_outside_sequences_vs_oracle(fk, shape, bf16, page):
    name, hq, hkv, cached, rows, causal = shape
    seed = 7800 + SHAPES.index(shape) + (0 if bf16 else 20) + page
    case = cases._case(f"{name}_nan", hq, hkv, cached, rows, bf16, causal, seed, page=page,
                       spare=3)
    md = case.metadata()
    _check(fk, case, _poison_unused_slots(case, case.inputs()), md)


WIDE_SHAPES = [
    ("decode_d256", 16, 2, [1500, 90, 3100], [1, 1, 1], True),
    ("draft_d256", 16, 2, [800, 2400], [16, 16], False),
]


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("shape", WIDE_SHAPES, ids=[s[0] for s in WIDE_SHAPES])
def test_nan_outside_sequences_head_dim_256(fk, shape, bf16):
    name, hq, hkv, cached, rows, causal = shape
    seed = 7900 + WIDE_SHAPES.index(shape) + (0 if bf16 else 20)
    case = cases._case(f"{name}_nan", hq, hkv, cached, rows, bf16, causal, seed, spare=3,
                       dim=256)
    md = case.metadata()
    _check(fk, case, _poison_unused_slots(case, case.inputs()), md)
