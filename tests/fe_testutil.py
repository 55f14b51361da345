"""Shared helpers for the parity tests (test infrastructure)."""
from __future__ import annotations

import numpy as np

import oracle

# Attention tolerance. The north-star bar is max-abs 2e-3 against the
# reference's ATen path. The reference rounds an fp32 result to fp16/bf16;
# two correct fp32 results a few 1e-7 apart can round to adjacent 16-bit
# values, and one bf16 unit in the last place exceeds 2e-3 once |o| >= 0.5
# (one fp16 ulp once |o| >= 4). The bound therefore is
#   |out - ref| <= 2e-3 + ulp(ref)
# i.e. 2e-3, widened by exactly one output ulp where that ulp is itself
# larger than the bar. Against the unrounded float32 oracle the kernel must
# meet 2e-3 + ulp/2 (its own rounding).
ATOL = 2e-3


def ulp16(ref_f32: np.ndarray, bf16: bool) -> np.ndarray:
    a = np.abs(ref_f32.astype(np.float64))
    mant = 7 if bf16 else 10
    min_exp = -126 if bf16 else -14
    e = np.floor(np.log2(np.maximum(a, 2.0 ** min_exp)))
    return 2.0 ** (e - mant)


def attn_tolerance(ref_f32: np.ndarray, bf16: bool, ulps: float = 1.0) -> np.ndarray:
    return ATOL + ulps * ulp16(ref_f32, bf16)


def compare_attention(out_bits, ref_bits, bf16, rows=None, ref_f32=None):
    """Returns (max_abs_err, worst_excess) where worst_excess > 0 means a
    violation of the tolerance."""
    dt = 1 if bf16 else 0
    out = oracle.to_float(out_bits, dt).astype(np.float64)
    ref = oracle.to_float(ref_bits, dt).astype(np.float64)
    if rows is not None:
        out, ref = out[rows], ref[rows]
    err = np.abs(out - ref)
    tol = attn_tolerance(ref, bf16)
    excess = float((err - tol).max()) if err.size else -1.0
    res = {"max_abs": float(err.max()) if err.size else 0.0, "excess": excess,
           "exact_frac": float(np.mean(out == ref)) if err.size else 1.0,
           "n_over_2e-3": int((err > ATOL).sum())}
    if ref_f32 is not None:
        r32 = ref_f32.astype(np.float64)
        if rows is not None:
            r32 = r32[rows]
        e32 = np.abs(out - r32)
        res["excess_vs_f32"] = float((e32 - attn_tolerance(r32, bf16, 0.5)).max()) if e32.size else -1.0
        res["max_abs_vs_f32"] = float(e32.max()) if e32.size else 0.0
    return res


def ref_aten_attention(q_bits, kpool_bits, vpool_bits, md, hq, hkv, dim, page, causal, bf16,
                       num_blocks):
    """The reference's own ATen attention (oracle/_ref, src/portable_gpu_ops.cpp:27-44)
    on host uint16 arrays; returns its 16-bit output bits [rows, hq, dim]."""
    max_pages = int((np.asarray(md.kv)[1:] - np.asarray(md.kv)[:-1]).max()) + 1
    ref = oracle.RefAten(hq, hkv, dim, page, md.batch, max_pages, bf16, num_blocks)
    try:
        ref.prepare(md.qo, md.kv, md.pages, md.last)
        return ref.attention(np.ascontiguousarray(q_bits), np.ascontiguousarray(kpool_bits),
                             np.ascontiguousarray(vpool_bits), causal)
    finally:
        ref.close()


def torch_dtype(bf16):
    import torch
    return torch.bfloat16 if bf16 else torch.float16


def to_device(bits: np.ndarray, bf16: bool):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.to("cuda").view(torch_dtype(bf16))


def to_host_bits(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def torch_reference_attention(q, kpool, vpool, qo, kv, pages, last, hq, hkv, page, causal):
    """fp32 restatement of src/portable_gpu_ops.cpp:39-44, for sizes the CPU
    oracle cannot finish quickly. q: [rows, hq, d]; pools [cache_slots, hkv, d]
    (all on one device, cuda or cpu); metadata numpy. Returns fp32 [rows, hq, d].
    Pinned against the reference's fixtures and live library by
    tests/test_cpu_torch_restatement.py."""
    import torch
    dim = q.shape[-1]
    G = hq // hkv
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    pages_t = torch.from_numpy(np.asarray(pages, np.int64)).to(q.device)
    for b in range(len(kv) - 1):
        length = int((kv[b + 1] - kv[b] - 1) * page + last[b])
        q0, q1 = int(qo[b]), int(qo[b + 1])
        qrows = q1 - q0
        if qrows == 0:
            continue
        t = torch.arange(length, device=q.device)
        slots = pages_t[kv[b] + t // page] * page + t % page
        k = kpool.view(-1, hkv, dim).index_select(0, slots).float()  # [L, hkv, d]
        v = vpool.view(-1, hkv, dim).index_select(0, slots).float()
        k = k.repeat_interleave(G, dim=1).permute(1, 2, 0)  # [hq, d, L]
        v = v.repeat_interleave(G, dim=1).permute(1, 0, 2)  # [hq, L, d]
        x = q[q0:q1].float().permute(1, 0, 2)  # [hq, rows, d]
        logits = torch.bmm(x, k) / float(np.sqrt(dim))
        if causal:
            r = torch.arange(qrows, device=q.device).unsqueeze(1)
            mask = t.unsqueeze(0) <= (length - qrows + r)
            logits = logits.masked_fill(~mask.unsqueeze(0), float("-inf"))
        p = torch.softmax(logits, dim=-1)
        out[q0:q1] = torch.bmm(p, v).permute(1, 0, 2)
    return out
