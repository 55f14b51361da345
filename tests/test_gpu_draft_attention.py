"""Draft / hybrid attention through the paged kernels (the hot path's
neighbours in the hybrid and draft models), against torch restatements of the reference's dense
formulations on the GPU:

* DFlash draft block (src/block_draft.cpp:24-30, read_/valid_ built at
  :50-53): RoPE over the whole head, store through the block's slots, then
  attention of the block rows over max_model_len gathered slots with every
  position >= valid masked. Here: fe_rope_append + the attention plan with the
  full mask over the sequence's block table (no max_model_len gather).
* Qwen3.5-style full attention (src/hybrid_model.cpp:41-50): partial rotary
  (leading rotary dims only), store, attention of one row over its context.

head_dim 128 runs on the decode / tcgen05 kernels; head_dim 256 (Qwen3.5's
full-attention layers) on the same kernels instantiated for 256 dims."""
import math

import numpy as np
import pytest

import oracle
from fe_testutil import compare_attention, to_host_bits

pytestmark = pytest.mark.gpu

DIM = 128
PAGE = 16


def _cos_sin(max_pos, rot, theta=1.0e6):
    import torch
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float().cuda(), torch.sin(ang).float().cuda()


def _rotate(x, cos, sin, pos, rot):
    """The reference's rotate (src/block_draft.cpp:22 for rot = dim,
    src/hybrid_model.cpp:44 for a partial rotary): fp32 products and sums on
    the leading `rot` dims, the rest passed through."""
    import torch
    cs = cos.index_select(0, pos).unsqueeze(1)
    sn = sin.index_select(0, pos).unsqueeze(1)
    a = x[..., : rot // 2].float()
    b = x[..., rot // 2: rot].float()
    return torch.cat([(a * cs - b * sn).to(x.dtype), (b * cs + a * sn).to(x.dtype), x[..., rot:]],
                     dim=-1)


def _dense_attention(q, kc, vc, read, valid, hq, hkv, dim=DIM):
    """src/block_draft.cpp:28-29 / src/hybrid_model.cpp:48-49: gather the read
    slots, mask timeline >= valid, fp32 softmax attention."""
    import torch
    G = hq // hkv
    keys = kc.view(-1, hkv, dim).index_select(0, read).repeat_interleave(G, 1).permute(1, 2, 0)
    values = vc.view(-1, hkv, dim).index_select(0, read).repeat_interleave(G, 1).permute(1, 0, 2)
    scores = torch.bmm(q.permute(1, 0, 2).float(), keys.float()) / math.sqrt(dim)
    timeline = torch.arange(read.shape[0], device=q.device)
    scores = scores.masked_fill((timeline >= valid)[None, None, :], float("-inf"))
    return torch.bmm(torch.softmax(scores, -1), values.float()).permute(1, 0, 2).to(q.dtype)


def _run_case(hq, hkv, start, rows, rot, max_model_len, seed, dim=DIM):
    import torch

    import fekv
    from fekv.metadata import draft_block_metadata
    rng = np.random.default_rng(seed)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    num_blocks = 400
    cache_slots = (num_blocks + 1) * PAGE
    width = hkv * dim
    end = start + rows
    blocks = rng.permutation(num_blocks)[: -(-max_model_len // PAGE)].astype(np.int64)
    kc0 = torch.randn(cache_slots, width, generator=g, device="cuda").to(torch.bfloat16)
    vc0 = torch.randn(cache_slots, width, generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn(rows, hq, dim, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(rows, hkv, dim, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(rows, hkv, dim, generator=g, device="cuda").to(torch.bfloat16)
    cos, sin = _cos_sin(max_model_len, rot)
    pos = torch.arange(start, end, device="cuda")
    slots = torch.from_numpy(blocks[np.arange(start, end) // PAGE] * PAGE +
                             np.arange(start, end) % PAGE).cuda()
    # reference: rotate, index_copy_, dense attention over max_model_len slots
    q_ref, k_ref = _rotate(q, cos, sin, pos, rot), _rotate(k, cos, sin, pos, rot)
    kc_ref, vc_ref = kc0.clone(), vc0.clone()
    kc_ref.index_copy_(0, slots, k_ref.view(rows, width))
    vc_ref.index_copy_(0, slots, v.view(rows, width))
    read = np.full(max_model_len, num_blocks * PAGE, np.int64)  # the padding page's first slot
    t = np.arange(end)
    read[:end] = blocks[t // PAGE] * PAGE + t % PAGE
    out_ref = _dense_attention(q_ref, kc_ref, vc_ref, torch.from_numpy(read).cuda(), end, hq, hkv,
                               dim)
    # ours: fused RoPE + append, then the plan with the full mask
    qd, kc, vc = q.clone(), kc0.clone(), vc0.clone()
    cache = torch.cat([cos, sin], dim=1).contiguous()
    fekv.rope_append(qd, k, v, kc, vc, slots, pos, cache)
    plan = fekv.AttentionPlan(hq, hkv, dim, PAGE, 1, -(-max_model_len // PAGE) + 1, True,
                              num_blocks)
    md = draft_block_metadata(blocks, start, rows, PAGE)
    plan.prepare(md.qo, md.kv, md.pages, md.last)
    out = torch.empty_like(qd)
    plan.attention(qd, kc, vc, out, causal=False)
    torch.cuda.synchronize()
    plan.close()
    np.testing.assert_array_equal(to_host_bits(qd), to_host_bits(q_ref))
    np.testing.assert_array_equal(to_host_bits(kc), to_host_bits(kc_ref))
    np.testing.assert_array_equal(to_host_bits(vc), to_host_bits(vc_ref))
    res = compare_attention(to_host_bits(out), to_host_bits(out_ref), True)
    assert res["excess"] <= 0.0, res
    assert fekv.device_errors() == 0
    return res


@pytest.mark.parametrize("hq,hkv,start,rows", [(32, 8, 300, 17), (32, 4, 1021, 17),
                                               (16, 8, 0, 16), (32, 8, 2047, 9)])
def test_dflash_draft_block_matches_dense_reference(hq, hkv, start, rows):
    _run_case(hq, hkv, start, rows, DIM, max_model_len=4096, seed=start + rows)


@pytest.mark.parametrize("rot,start", [(64, 777), (32, 5), (128, 1500)])
def test_partial_rotary_full_attention_row_matches_dense_reference(rot, start):
    _run_case(16, 2, start, 1, rot, max_model_len=2048, seed=rot + start)


@pytest.mark.parametrize("hq,hkv,start,rows", [(16, 2, 700, 17), (8, 1, 0, 16), (24, 4, 2000, 9)])
def test_dflash_draft_block_head_dim_256(hq, hkv, start, rows):
    _run_case(hq, hkv, start, rows, 256, max_model_len=3072, seed=start + rows, dim=256)


@pytest.mark.parametrize("rot,start", [(64, 1234), (256, 77)])
def test_qwen35_full_attention_row_head_dim_256(rot, start):
    """Qwen3.5's full-attention layers: head_dim 256 with a partial rotary."""
    _run_case(16, 2, start, 1, rot, max_model_len=2048, seed=rot + start, dim=256)
