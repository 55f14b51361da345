"""Seeded synthetic Qwen3-style decoder for the greedy-token parity check
(test infrastructure).

The layer math follows the reference's ``Net::forward``
(Cambridgebit/FlashEngine.cpp src/cuda_model.cpp:86-101): embed -> RMSNorm ->
Q/K/V projections -> per-head q/k RMSNorm -> RoPE -> **store** -> **attention**
-> o_proj + residual -> RMSNorm -> SwiGLU MLP + residual, x L -> final RMSNorm
-> lm_head -> argmax. Weights are random (seeded) bf16 values, the dense math
runs in fp32 in torch on the GPU (so that a last-bit difference at the
attention boundary is not re-rounded into every later activation), q/k/v cross
into the paged-KV operators as bf16 and the attention output comes back as
bf16. A ``backend`` object supplies only the three paged-KV
operators the reference delegates to its CUDA kernels: ``store`` (append
through the slot mapping), ``copy_blocks`` (copy-on-write of a shared partial
tail page) and ``attention`` (paged GQA attention with the bottom-right causal
mask). Running the same generation twice with two backends and comparing the
tokens checks that swapping the operators leaves greedy decoding unchanged.

The generation loop exercises every row shape of the hot path: one chunked
prefill of all prompts (multi-row causal rows), single-row decode steps, a fork
of a sequence that shares its full pages and copies its partial tail page, and
speculative verify steps (several rows per sequence) with greedy acceptance
(the rule of the reference's ``accept_kernel``, src/cuda_kernels.cu:25:
accept draft tokens while they equal the target's argmax, then take the
target's token), after which rejected rows are rolled back by shortening the
sequence (their slots are rewritten later).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from fekv.metadata import build_step_metadata


class SynthQwen3:
    def __init__(self, seed=0, vocab=512, hidden=512, hq=8, hkv=2, dim=128, inter=1024,
                 layers=2, rope_theta=1.0e6, max_pos=1024, device="cuda"):
        self.vocab, self.hidden, self.hq, self.hkv, self.dim = vocab, hidden, hq, hkv, dim
        self.layers_n = layers
        self.device = device
        g = torch.Generator(device=device)
        g.manual_seed(seed)

        def w(*shape, scale=1.0):  # bf16-representable fp32 weights
            return (torch.randn(*shape, generator=g, device=device) * scale).to(torch.bfloat16).float()

        def ln(n):
            return (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16).float()

        self.embed = w(vocab, hidden)
        self.layers = []
        for _ in range(layers):
            self.layers.append(dict(
                ln1=ln(hidden), wq=w(hidden, hq * dim, scale=hidden ** -0.5),
                wk=w(hidden, hkv * dim, scale=hidden ** -0.5),
                wv=w(hidden, hkv * dim, scale=hidden ** -0.5),
                qn=ln(dim), kn=ln(dim), wo=w(hq * dim, hidden, scale=(hq * dim) ** -0.5),
                ln2=ln(hidden), wg=w(hidden, inter, scale=hidden ** -0.5),
                wu=w(hidden, inter, scale=hidden ** -0.5), wd=w(inter, hidden, scale=inter ** -0.5)))
        self.norm = ln(hidden)
        self.lm_head = w(hidden, vocab, scale=hidden ** -0.5)
        inv = 1.0 / (rope_theta ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
        ang = torch.arange(max_pos, device=device, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos, self.sin = torch.cos(ang), torch.sin(ang)  # fp32 cache, [max_pos, dim/2]

    @staticmethod
    def rmsnorm(x, weight, eps=1e-6):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight

    def rope(self, x, pos):
        # rotate-half RoPE on [rows, heads, dim] with the fp32 cos/sin cache
        c = self.cos[pos][:, None, :]
        s = self.sin[pos][:, None, :]
        x1, x2 = x[..., : self.dim // 2], x[..., self.dim // 2:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)

    def forward(self, tokens, positions, md, kv, backend):
        """tokens/positions: int64 [rows] (cuda); md: StepMetadata of this
        step. Returns fp32 logits [rows, vocab]."""
        x = self.embed[tokens]
        rows = x.shape[0]
        backend.prepare(md)
        for li, L in enumerate(self.layers):
            h = self.rmsnorm(x, L["ln1"])
            q = (h @ L["wq"]).view(rows, self.hq, self.dim)
            k = (h @ L["wk"]).view(rows, self.hkv, self.dim)
            v = (h @ L["wv"]).view(rows, self.hkv, self.dim)
            q = self.rope(self.rmsnorm(q, L["qn"]), positions).to(torch.bfloat16)
            k = self.rope(self.rmsnorm(k, L["kn"]), positions).to(torch.bfloat16)
            v = v.to(torch.bfloat16)
            backend.store(k.contiguous(), v.contiguous(), kv.kpools[li], kv.vpools[li], md)
            o = backend.attention(q.contiguous(), kv.kpools[li], kv.vpools[li], md)
            x = x + o.float().view(rows, self.hq * self.dim) @ L["wo"]
            h = self.rmsnorm(x, L["ln2"])
            x = x + (torch.nn.functional.silu(h @ L["wg"]) * (h @ L["wu"])) @ L["wd"]
        x = self.rmsnorm(x, self.norm)
        return x @ self.lm_head


class PagedKV:
    """Per-layer K/V pools [(num_blocks+1)*page, hkv*dim] (page num_blocks is
    the zeroed padding page) and a FIFO free list of page ids, as the
    reference's BlockManager hands them out (src/scheduler.cpp:6-36)."""

    def __init__(self, model, num_blocks, page=16, seed=0):
        self.page, self.num_blocks = page, num_blocks
        self.width = model.hkv * model.dim
        self.cache_slots = (num_blocks + 1) * page
        self.kpools = [torch.zeros(self.cache_slots, self.width, dtype=torch.bfloat16,
                                   device=model.device) for _ in range(model.layers_n)]
        self.vpools = [torch.zeros_like(p) for p in self.kpools]
        rng = np.random.default_rng(seed)
        self.free = [int(x) for x in rng.permutation(num_blocks)]

    def alloc(self):
        return self.free.pop(0)

    def ensure(self, blocks, length):
        while len(blocks) * self.page < length:
            blocks.append(self.alloc())


class TorchBackend:
    """The reference's paged-KV operators restated in torch on the GPU: store
    = the CUDA store_kernel (src/cuda_kernels.cu:24,34; rows with slot < 0 are
    skipped), attention = the fp32 ATen path (src/portable_gpu_ops.cpp:27-44)."""

    def __init__(self, model, kv, drop_last_key=False):
        self.m, self.kv = model, kv
        # planted mistake for the test of this check: every row misses its
        # last visible key
        self.drop_last_key = drop_last_key

    def prepare(self, md):
        self.md = md
        self.slots = torch.from_numpy(md.slots).to(self.m.device)

    def store(self, k, v, kpool, vpool, md):
        keep = self.slots >= 0
        kpool[self.slots[keep]] = k.view(-1, self.kv.width)[keep]
        vpool[self.slots[keep]] = v.view(-1, self.kv.width)[keep]

    def copy_blocks(self, src, dst, ntok):
        for pools in (self.kv.kpools, self.kv.vpools):
            for p in pools:
                pv = p.view(-1, self.kv.page, self.kv.width)
                for s, d, n in zip(src, dst, ntok):
                    pv[d, :n] = pv[s, :n]

    def attention(self, q, kpool, vpool, md):
        from fe_testutil import torch_reference_attention
        last = md.last
        if self.drop_last_key:
            # one key fewer per sequence; the causal diagonal moves with it
            lengths = md.lengths(self.kv.page) - 1
            if (lengths < 1).any():
                return torch.zeros_like(q)
            last = ((lengths - 1) % self.kv.page + 1).astype(np.int32)
            # sequences whose last page held one token now end a page earlier
            kvp = md.kv.copy()
            pages = []
            for b in range(md.batch):
                n = -(-int(lengths[b]) // self.kv.page)
                pages.append(md.pages[md.kv[b]:md.kv[b] + n])
                kvp[b + 1] = kvp[b] + n
            o = torch_reference_attention(q, kpool, vpool, md.qo, kvp, np.concatenate(pages),
                                          last, self.m.hq, self.m.hkv, self.kv.page, True)
            return o.to(torch.bfloat16)
        o = torch_reference_attention(q, kpool, vpool, md.qo, md.kv, md.pages, last,
                                      self.m.hq, self.m.hkv, self.kv.page, True)
        return o.to(torch.bfloat16)


class FekvBackend:
    """This repository's operators through the C ABI (libfe_kv_b200.so)."""

    def __init__(self, model, kv, max_batch=16):
        import fekv
        self.fekv, self.m, self.kv = fekv, model, kv
        max_pages = kv.num_blocks + 1
        self.plan = fekv.AttentionPlan(model.hq, model.hkv, model.dim, kv.page, max_batch,
                                       max_pages, True, kv.num_blocks)

    def prepare(self, md):
        self.md = md
        self.slots = torch.from_numpy(md.slots).cuda()
        self.plan.prepare(md.qo, md.kv, md.pages, md.last)

    def store(self, k, v, kpool, vpool, md):
        self.fekv.store(k, v, kpool, vpool, self.slots)

    def copy_blocks(self, src, dst, ntok):
        t = lambda a: torch.tensor(a, dtype=torch.int32, device="cuda")  # noqa: E731
        self.fekv.copy_blocks(self.kv.kpools, self.kv.vpools, t(src), t(dst), t(ntok),
                              self.kv.page, self.kv.width, self.kv.num_blocks + 1)

    def attention(self, q, kpool, vpool, md):
        out = torch.empty_like(q)
        self.plan.attention(q, kpool, vpool, out, causal=True)
        return out

    def close(self):
        self.plan.close()


def generate(model, kv, backend, prompts, steps=24, verify_at=(8, 16), draft_len=4,
             fork_from=0, seed=0):
    """Greedy generation; returns (tokens per sequence, smallest top-2 logit
    gap seen, number of accepted draft tokens)."""
    rng = np.random.default_rng(seed + 17)
    seqs = [dict(tokens=list(map(int, p)), blocks=[], length=0) for p in prompts]
    min_gap = math.inf
    accepted = 0

    def run(batch, new_tokens):
        """batch: sequence indices; new_tokens[i]: tokens appended to seq."""
        nonlocal min_gap
        starts, rows, tables = [], [], []
        for b, toks in zip(batch, new_tokens):
            s = seqs[b]
            kv.ensure(s["blocks"], s["length"] + len(toks))
            starts.append(s["length"])
            rows.append(len(toks))
            tables.append(np.asarray(s["blocks"], np.int64))
        md = build_step_metadata(tables, starts, rows, kv.page)
        tok = torch.tensor(np.concatenate(new_tokens), dtype=torch.int64, device=model.device)
        pos = torch.from_numpy(md.positions).to(model.device)
        logits = model.forward(tok, pos, md, kv, backend)
        top2 = torch.topk(logits, 2, dim=-1).values
        min_gap = min(min_gap, float((top2[:, 0] - top2[:, 1]).min()))
        for b, toks in zip(batch, new_tokens):
            seqs[b]["length"] += len(toks)
        return logits.argmax(-1).cpu().numpy(), md

    # prefill: all prompts in one chunked step
    out, md = run(list(range(len(seqs))), [np.asarray(s["tokens"]) for s in seqs])
    ends = md.qo[1:] - 1
    nxt = [int(out[e]) for e in ends]
    # fork: a child shares the parent's full pages and copy-on-writes its tail
    par = seqs[fork_from]
    full = par["length"] // kv.page
    child = dict(tokens=list(par["tokens"]), blocks=list(par["blocks"][:full]),
                 length=par["length"])
    tail = par["length"] % kv.page
    if tail:
        newp = kv.alloc()
        backend.copy_blocks([par["blocks"][full]], [newp], [tail])
        child["blocks"].append(newp)
    seqs.append(child)
    nxt.append((nxt[fork_from] + 1) % model.vocab)  # diverge from the parent
    for i, s in enumerate(seqs):
        s["tokens"].append(nxt[i])
    batch = list(range(len(seqs)))
    step = 0
    while step < steps:
        if step in verify_at:
            # speculative verify: the last token plus draft_len - 1 proposals
            drafts = []
            for b in batch:
                d = [seqs[b]["tokens"][-1]] + [int(x) for x in rng.integers(0, model.vocab,
                                                                              draft_len - 1)]
                drafts.append(np.asarray(d))
            out, md = run(batch, drafts)
            for i, b in enumerate(batch):
                r0 = int(md.qo[i])
                target = [int(out[r0 + j]) for j in range(draft_len)]
                d = drafts[i]
                n_ok = 0
                while n_ok + 1 < draft_len and int(d[n_ok + 1]) == target[n_ok]:
                    n_ok += 1
                accepted += n_ok
                s = seqs[b]
                # keep the accepted drafts, drop the rest, append the target token
                s["length"] -= draft_len - 1 - n_ok
                s["tokens"].extend(int(x) for x in d[1:1 + n_ok])
                s["tokens"].append(target[n_ok])
        else:
            out, md = run(batch, [np.asarray([seqs[b]["tokens"][-1]]) for b in batch])
            for i, b in enumerate(batch):
                seqs[b]["tokens"].append(int(out[i]))
        step += 1
    return [s["tokens"] for s in seqs], min_gap, accepted
