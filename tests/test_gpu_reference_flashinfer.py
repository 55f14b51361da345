"""The reference's own CUDA attention (src/flashinfer_attention.cu: FlashInfer's
FA2 paged prefill kernel with split-KV disabled, built for sm_100a from the
reference source by oracle/build_oracle.py) on the GPU, beside this
repository's kernels on the same inputs:

* on the golden cases, both are compared with the reference's ATen outputs
  (the fixtures): this repository's kernels within the attention tolerance,
  the reference GPU path within a loose sanity bound (FlashInfer rounds the
  softmax weights to 16 bits before P.V, so its error against the fp32 ATen
  path is larger; the figures are recorded);
* on a full C2 decode layer and a full C4 verify layer, both against the fp32
  restatement of the ATen path (pinned by test_cpu_torch_restatement.py).
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
    if not oracle.ref_flashinfer_available():
        pytest.skip("oracle/_ref/libfe_ref_flashinfer.so not built")
    import fekv
    fekv.load()
    return fekv


def _both(fk, hq, hkv, page, num_blocks, md, q, kc, vc, causal, bf16, max_pages):
    import torch
    ours = torch.full_like(q, float("nan"))
    plan = fk.AttentionPlan(hq, hkv, 128, page, md.batch, max_pages, bf16, num_blocks)
    plan.prepare(md.qo, md.kv, md.pages, md.last)
    plan.attention(q, kc, vc, ours, causal)
    ref = torch.full_like(q, float("nan"))
    fi = oracle.RefFlashInfer(hq, hkv, 128, page, md.batch, max_pages, bf16, num_blocks)
    stream = torch.cuda.current_stream().cuda_stream
    fi.prepare(md.qo, md.kv, md.pages, md.last, stream)
    fi.attention(q, kc, vc, ref, causal, stream)
    torch.cuda.synchronize()
    fi.close()
    plan.close()
    assert fk.device_errors() == 0
    return to_host_bits(ours), to_host_bits(ref)


# the reference's CUDA build serves page 16 and any GQA group (graph padding
# rows excluded from the comparison)
NAMES = [c.name for c in cases.all_cases() if c.page == 16]


@pytest.mark.parametrize("name", NAMES)
def test_flashinfer_and_ours_match_reference_fixtures(fk, parity_record, name):
    case = cases.case_by_name(name)
    fx = dict(np.load(cases.fixture_path(name)))
    inp = case.inputs()
    md = case.metadata()
    ko, vo = inp["kpool"].copy(), inp["vpool"].copy()
    oracle.append(inp["knew"], inp["vnew"], ko, vo, md.slots, case.cache_slots)
    q = to_device(inp["q"], case.bf16)
    ours, fi = _both(fk, case.hq, case.hkv, case.page, case.num_blocks, md, q,
                     to_device(ko, case.bf16), to_device(vo, case.bf16), case.causal, case.bf16,
                     case.max_pages())
    real = np.arange(md.rows) < int(md.qo[len(case.block_tables)])
    shape = inp["q"].shape
    res_fi = compare_attention(fi.reshape(shape), fx["ref_out"], case.bf16, rows=real)
    res_ours = compare_attention(ours.reshape(shape), fx["ref_out"], case.bf16, rows=real)
    parity_record(f"reference FlashInfer GPU path on fixture {name}", res_fi)
    assert res_ours["excess"] <= 0, res_ours
    assert res_fi["max_abs"] < 0.05, res_fi  # a working comparator, not a parity bar


@pytest.mark.parametrize("config", ["c2", "c4"])
def test_full_layer_against_fp32_both_paths(fk, parity_record, config):
    import torch
    import fekv.workloads as wl
    from fe_testutil import torch_reference_attention
    w = wl.c2_shard(0) if config == "c2" else wl.c4(seed=0)
    md = w.metadata()
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    dt = torch.bfloat16
    kc = (torch.randn(w.cache_slots, w.width, generator=g, device="cuda") * w.scale).to(dt)
    vc = (torch.randn(w.cache_slots, w.width, generator=g, device="cuda") * w.scale).to(dt)
    q = (torch.randn(md.rows, w.hq, w.dim, generator=g, device="cuda") * w.scale).to(dt)
    ours, fi = _both(fk, w.hq, w.hkv, w.page, w.num_blocks, md, q, kc, vc, w.causal, True,
                     w.max_pages())
    ref = torch_reference_attention(q, kc, vc, md.qo, md.kv, md.pages, md.last, w.hq, w.hkv,
                                    w.page, w.causal)
    ref_bits = to_host_bits(ref.to(dt))
    ref32 = ref.cpu().numpy()
    res_ours = compare_attention(ours, ref_bits, True, ref_f32=ref32)
    res_fi = compare_attention(fi, ref_bits, True, ref_f32=ref32)
    parity_record(f"{config} layer: this repository vs fp32 ATen restatement", res_ours)
    parity_record(f"{config} layer: reference FlashInfer GPU path vs fp32 ATen restatement",
                  res_fi)
    assert res_ours["excess"] <= 0 and res_ours["excess_vs_f32"] <= 0, res_ours
    assert res_fi["max_abs"] < 0.05, res_fi
