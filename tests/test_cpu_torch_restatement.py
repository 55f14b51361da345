"""The fp32 torch restatement of the reference attention
(fe_testutil.torch_reference_attention), pinned on the CPU.

The GPU parity tests use that restatement as the checker wherever the CPU
oracle is too slow (full C2-C5 layers, graph replay, head_dim 256, the greedy
model). Here it runs with CPU tensors and is compared with

* the golden fixtures, i.e. outputs of the reference's own ATen path
  (src/portable_gpu_ops.cpp:27-44) run by tests/golden/make_golden.py;
* the reference library itself (oracle/_ref/libfe_ref_aten.so) on random
  shapes: GQA groups 1-16, pages of 16/32/64 tokens, both masks, fp16 and
  bf16, head_dim 128 and 256 (the reference ATen path takes any head_dim);
* the float64 C oracle, before rounding.

Both sides compute the same fp32 gather / bmm / softmax / bmm, so after
rounding to the 16-bit output type nearly every element must be identical,
and all must meet the attention tolerance.
"""
import numpy as np
import pytest

import cases
import oracle
from fe_testutil import compare_attention, torch_reference_attention

torch = pytest.importorskip("torch")


def _after_append(case, inp, md):
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    return ko, vo


def _torch_ref(q_bits, ko, vo, md, hq, hkv, dim, page, causal, bf16):
    dt = torch.bfloat16 if bf16 else torch.float16

    def t(a, shape):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dt).reshape(shape)

    rows = q_bits.shape[0]
    q = t(q_bits, (rows, hq, dim))
    kc = t(ko, (-1, hkv * dim))
    vc = t(vo, (-1, hkv * dim))
    out32 = torch_reference_attention(q, kc, vc, md.qo, md.kv, md.pages, md.last, hq, hkv, page,
                                      causal)
    bits = out32.to(dt).view(torch.int16).numpy().view(np.uint16)
    return bits, out32.numpy()


@pytest.mark.parametrize("name", [c.name for c in cases.all_cases()])
def test_restatement_matches_reference_fixture(name):
    case = cases.case_by_name(name)
    fx = dict(np.load(cases.fixture_path(name)))
    inp = case.inputs()
    md = case.metadata()
    ko, vo = _after_append(case, inp, md)
    got, got32 = _torch_ref(inp["q"], ko, vo, md, case.hq, case.hkv, case.dim, case.page,
                            case.causal, case.bf16)
    real = np.arange(md.rows) < int(md.qo[len(case.block_tables)])  # graph padding excluded
    res = compare_attention(got, fx["ref_out"], case.bf16, rows=real)
    assert res["excess"] <= 0, res
    assert res["exact_frac"] >= 0.99, res
    _, want32 = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq,
                                 case.hkv, case.dim, case.page, case.causal, case.dtype_code)
    assert float(np.abs(got32[real] - want32[real]).max()) < 2e-5


def _random_case(seed):
    rng = np.random.default_rng(7000 + seed)
    hkv = int(rng.choice([1, 2, 4, 8]))
    G = int(rng.choice([1, 2, 4, 8, 16]))
    batch = int(rng.integers(1, 5))
    cached = rng.integers(0, 900, size=batch)
    rows = np.where(rng.random(batch) < 0.5, 1, rng.integers(1, 24, size=batch))
    dim = 256 if seed % 3 == 2 else 128
    case = cases._case(f"pin{seed}", hkv * G, hkv, cached, rows, bool(seed % 2), bool(seed % 4 < 2),
                       9000 + seed, page=int(rng.choice([16, 32, 64])), dim=dim)
    return case


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("seed", range(12))
def test_restatement_matches_live_reference(seed):
    case = _random_case(seed)
    inp = case.inputs()
    md = case.metadata()
    ko, vo = _after_append(case, inp, md)
    ref = oracle.RefAten(case.hq, case.hkv, case.dim, case.page, md.batch, case.max_pages(),
                         case.bf16, case.num_blocks)
    ref.prepare(md.qo, md.kv, md.pages, md.last)
    want = ref.attention(inp["q"], ko, vo, case.causal)
    ref.close()
    got, got32 = _torch_ref(inp["q"], ko, vo, md, case.hq, case.hkv, case.dim, case.page,
                            case.causal, case.bf16)
    res = compare_attention(got, want, case.bf16)
    assert res["excess"] <= 0, (case.hq, case.hkv, case.dim, res)
    assert res["exact_frac"] >= 0.99, res
    _, want32 = oracle.attention(inp["q"], ko, vo, md.qo, md.kv, md.pages, md.last, case.hq,
                                 case.hkv, case.dim, case.page, case.causal, case.dtype_code)
    assert float(np.abs(got32 - want32).max()) < 2e-5
