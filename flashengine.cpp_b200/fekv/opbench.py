"""Timings of the path's smaller operators on one GPU: K/V append, block copy,
RoPE, fused RoPE + append, greedy accept, and step preparation on the host
and on the device. One JSON line per case.

    python -m fekv.opbench            (from flashengine.cpp_b200/, or with it on sys.path)

Each case runs `--warmup` untimed calls, then times `--iters` calls captured
in one CUDA graph (host-side argument handling stays out of the timing; the
host planner, which cannot be captured, is timed eagerly) between CUDA events
on the launching stream; `us` is the mean per call.
`bytes` is the algorithmic traffic of one call (every byte the operation must
read or write once) and `gbs` / `frac_hbm` relate it to the measured HBM copy
peak (MEASURED_PEAKS.json at the repository root, else 6650 GB/s). The
decode-size cases (one row per sequence) move a few hundred KiB and are bound
by launch latency, not bandwidth; the large cases show each kernel's
bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _peak_gbs() -> float:
    try:
        with open(os.path.join(_ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:
        return 6650.0


def _time(fn, iters: int, warmup: int, graph: bool = True) -> float:
    """Mean device time per call. With `graph`, `iters` calls are captured in
    one CUDA graph and replayed, so the launches reach the GPU back to back
    (host-side argument handling stays out of the timing); without, the
    calls are issued eagerly (host work that cannot be captured)."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
    else:
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / iters


def _emit(op, case, us, nbytes, peak, **extra):
    line = {"op": op, "case": case, "us": round(us, 2)}
    if nbytes:
        gbs = nbytes / (us * 1e-6) / 1e9
        line.update({"bytes": int(nbytes), "gbs": round(gbs, 1), "frac_hbm": round(gbs / peak, 4)})
    line.update(extra)
    print(json.dumps(line), flush=True)


def run(iters: int = 200, warmup: int = 20) -> None:
    import torch

    from . import ops, workloads
    from ._lib import load

    load()
    peak = _peak_gbs()
    dev = torch.device("cuda")
    bf = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(0)

    # ---- K/V append: decode step of C2 (64 rows x 1024) and a 64k-row batch
    for name, rows, width, slots_total in (("C2 decode step", 64, 1024, 1 << 20),
                                           ("64k rows", 65536, 1024, 1 << 18)):
        k = torch.randn(rows, width, generator=g, device=dev).to(bf)
        v = torch.randn(rows, width, generator=g, device=dev).to(bf)
        kc = torch.empty(slots_total, width, dtype=bf, device=dev)
        vc = torch.empty_like(kc)
        slots = torch.randperm(slots_total, device=dev)[:rows].to(torch.int64)
        us = _time(lambda: ops.store(k, v, kc, vc, slots), iters, warmup)
        _emit("append", name, us, rows * (width * 2 * 2 * 2 + 8), peak)

    # ---- block copy (copy-on-write): C4 forks (64 partial tails, 48 layers)
    # and whole pages
    w4 = workloads.c4(seed=0)
    src, dst, ntok = (np.asarray(x, np.int32) for x in w4.cow)
    for name, layers, full in (("C4 CoW tails, 48 layers", 48, False),
                               ("256 whole pages, 48 layers", 48, True)):
        n = 256 if full else len(src)
        s_ = torch.from_numpy(np.arange(n, dtype=np.int32) if full else src).to(dev)
        d_ = torch.from_numpy((np.arange(n, dtype=np.int32) + 512) if full else dst).to(dev)
        t_ = torch.from_numpy(np.full(n, 16, np.int32) if full else ntok).to(dev)
        pages_total = int(max(int(d_.max()), int(s_.max()))) + 2
        pools_k = [torch.zeros(pages_total * 16, w4.width, dtype=bf, device=dev) for _ in range(layers)]
        pools_v = [torch.zeros_like(p) for p in pools_k]
        tok = int(t_.sum())
        us = _time(lambda: ops.copy_blocks(pools_k, pools_v, s_, d_, t_, 16, w4.width, pages_total),
                   iters, warmup)
        _emit("copy_blocks", name, us, layers * 2 * tok * w4.width * 2 * 2, peak)

    # ---- RoPE and fused RoPE + append (Qwen3-8B shape hq32/hkv8/d128)
    hq, hkv, dim, max_pos = 32, 8, 128, 8192
    inv = 1.0 / (1e6 ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    cache = torch.from_numpy(np.concatenate([np.cos(ang), np.sin(ang)], 1).astype(np.float32)).to(dev)
    for name, rows in (("C2 decode step", 64), ("C3 step, 2108 rows", 2108), ("64k rows", 65536)):
        q = torch.randn(rows, hq, dim, generator=g, device=dev).to(bf)
        k = torch.randn(rows, hkv, dim, generator=g, device=dev).to(bf)
        v = torch.randn(rows, hkv, dim, generator=g, device=dev).to(bf)
        slots_total = max(1 << 18, rows)
        kc = torch.empty(slots_total, hkv * dim, dtype=bf, device=dev)
        vc = torch.empty_like(kc)
        slots = torch.randperm(slots_total, device=dev)[:rows].to(torch.int64)
        pos = torch.randint(0, max_pos, (rows,), generator=g, device=dev)
        # q read + written, k and v read, both written to the pools, the cos |
        # sin row of each position read, slot and position read
        e = 2  # bytes per element
        fused = rows * (2 * hq * dim * e + 2 * hkv * dim * e + 2 * hkv * dim * e + dim * 4 + 16)
        us = _time(lambda: ops.rope_append(q, k, v, kc, vc, slots, pos, cache), iters, warmup)
        _emit("rope_append", name, us, fused, peak)
        # the reference's sequence: rope in place, then store from k and v
        us2 = _time(lambda: (ops.rope(q, k, pos, cache), ops.store(k, v, kc, vc, slots)), iters,
                    warmup)
        _emit("rope_then_append", name, us2, fused, peak,
              note="rope and append as two launches (the reference's order)")

    # ---- greedy accept (batch 64, 15 draft tokens)
    batch, kd = 64, 15
    draft = torch.randint(0, 1000, (batch, kd), generator=g, device=dev)
    verify = torch.randint(0, 1000, (batch, kd + 1), generator=g, device=dev)
    out = torch.zeros(batch, kd + 2, dtype=torch.int64, device=dev)
    us = _time(lambda: ops.accept(draft, verify, out), iters, warmup)
    _emit("accept", "batch 64, k 15", us, 0, peak)

    # ---- step preparation: host planner + H2D versus the device planner
    w2 = workloads.c2(seed=0, steps=2)
    md = w2.metadata(0)
    plan = ops.AttentionPlan(w2.hq, w2.hkv, 128, 16, w2.batch, w2.max_pages(2), True,
                             w2.num_blocks)
    us = _time(lambda: plan.prepare(md.qo, md.kv, md.pages, md.last, md.batch, md.rows, False,
                                    torch.cuda.current_stream()), iters, warmup, graph=False)
    _emit("prepare_host", "C2 decode step (64 seqs)", us, 0, peak,
          note="host planner + one H2D copy, as seen by the stream")
    stride = int(np.diff(md.kv).max()) + 1
    bt = np.zeros((w2.batch, stride), np.int32)
    for b, t in enumerate(w2.block_tables):
        bt[b, :len(t)] = t
    bt_d = torch.from_numpy(bt).to(dev)
    starts = torch.from_numpy(w2.cached.astype(np.int32)).to(dev)
    slots = torch.empty(w2.batch, dtype=torch.int64, device=dev)
    positions = torch.empty_like(slots)
    gplan = ops.AttentionPlan(w2.hq, w2.hkv, 128, 16, w2.batch, w2.max_pages(2), True,
                              w2.num_blocks)
    us = _time(lambda: gplan.step_prepare_device(bt_d, starts, 1, slots, positions,
                                                 torch.cuda.current_stream()), iters, warmup)
    _emit("prepare_device", "C2 decode step (64 seqs)", us, 0, peak,
          note="slot mapping + work lists built by one kernel from device block tables")
    plan.close()
    gplan.close()
    if ops.device_errors() != 0:
        raise RuntimeError("device error bits set during the op benchmark")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    a = ap.parse_args(argv)
    run(a.iters, a.warmup)
    return 0


if __name__ == "__main__":
    sys.exit(main())
