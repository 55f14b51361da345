"""Paged-KV decode benchmark (BASELINE metric: paged decode-attention achieved
TB/s and decode tokens/s at 1/2/4/8 B200).

One step = one decode step of the whole layer stack of the configured
workload: build the step's slot mapping and page tables on the host (the
reference's CudaModel::prepare), prepare the attention plan (one H2D copy),
then per layer append one K/V row per sequence and run paged decode attention.

Default workload: C2 (Qwen3-8B attention shape: hq32/hkv8/d128 bf16, 36
layers, 64 sequences, contexts U[512,4096], page 16). Under torchrun every
rank runs its own 64 sequences (weak scaling); NCCL is used only after the
timed loop to gather per-rank results (no collective on the hot path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c3|c4|c5|q35|draft]
  python bench.py --impl reference ...   # the reference's own CPU/ATen path

c3 / c4 time the chunked-prefill and verify steps (rows/s, tensor-core
roofline); q35 and draft are head_dim 256 steps (hybrid-model full-attention
decode, and 16-row draft blocks under the full mask).

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "flashengine.cpp_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "paged decode-attn achieved TB/s (% HBM peak); decode tokens/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def measured_peak_tflops():
    """Sustained bf16 dense peak (a kernel timed inside a long step)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


# DRAM bytes (read + write) per launch of each roofline kernel, from one
# `ncu --set full --clock-control none` capture of the same layer shape; the
# profile named beside each holds the command. Keyed by (workload, kernel) and
# checked against the algorithmic units (bytes or FLOPs) of the captured launch,
# so a changed workload reports null rather than a stale figure.
# The decode kernel streams every page once, so its traffic scales with the
# bytes a launch reads (the bench's contexts grow by one token per step); the
# tcgen05 kernel's DRAM bytes depend on L2 reuse of shared prefixes and are
# only reported for the captured launch itself.
NCU_TRAFFIC = {
    ("C2", "paged_decode_kernel"): (611757056, 603463680.0, True,
                                    "profiles/paged_decode_kernel_c2.md"),
    ("C4", "paged_prefill_tc_kernel"): (63075840, 75586338816.0, False,
                                        "profiles/paged_prefill_tc_kernel_c4.md"),
    ("DFL", "paged_prefill_tc_kernel"): (159589120, 155019264.0, True,
                                         "profiles/paged_prefill_tc_kernel_d256_draft.md"),
    ("Q35", "paged_decode_kernel"): (308690176, 302256128.0, True,
                                     "profiles/paged_decode_kernel_d256_q35.md"),
    ("C3", "paged_prefill_tc_kernel"): (42910208, 42966450176.0, False,
                                        "profiles/paged_prefill_tc_kernel_c3.md"),
}


def ncu_traffic(workload: str, kernel: str, units_per_launch: float):
    """(traffic bytes per launch, source) for the bench's launch, or (None, None)."""
    ent = NCU_TRAFFIC.get((workload, kernel))
    if ent is None:
        return None, None
    dram, units, proportional, src = ent
    ratio = units_per_launch / units
    if proportional and 0.9 < ratio < 1.1:
        return round(dram * ratio), f"ncu capture scaled by algorithmic bytes, {src}"
    if abs(ratio - 1.0) <= 1e-3:
        return dram, f"ncu capture, {src}"
    return None, None


def row_step_bound(block_tables, flops: float, nbytes: float, tpeak_tflops: float,
                   peak_gbs: float) -> str:
    """Roofline bound of a multi-row attention launch. With no page shared
    between sequences every K/V byte comes from HBM once per launch; below the
    ridge (FLOPs per byte < peak FLOP/s / peak B/s, e.g. 16-row draft blocks x
    a GQA group of 8 = 128 FLOP/B) the launch is bound by HBM, not by the
    tensor pipe. Shared pages (a common prefix) are served from L2, so such a
    step stays tensor-bound whatever its per-byte intensity."""
    all_pages = np.concatenate([np.asarray(t) for t in block_tables])
    shared = len(np.unique(all_pages)) < len(all_pages)
    ridge = tpeak_tflops * 1e12 / (peak_gbs * 1e9)
    return "hbm" if (not shared and flops / nbytes < ridge) else "tensor"


def measured_peak_gbs():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="fe_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.dev)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                    power.append(float(parts[3]))
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# distributed plumbing (one process per GPU; no collective on the hot path)
# ---------------------------------------------------------------------------

def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def gather_floats(values, world):
    """All-gather a small float64 vector per rank (after timing only)."""
    from fekv.dist import gather_floats as _gather

    return _gather(values, world, device="cuda")


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

def make_workload(config, rank, world, total_steps):
    from fekv import workloads

    if config == "c2":
        return workloads.c2(seed=1000 + rank, steps=total_steps)
    if config == "c5":
        return workloads.c5(rank=rank, world=world, steps=total_steps)
    if config == "c3":
        return workloads.c3(seed=1000 + rank)
    if config == "c4":
        return workloads.c4(seed=1000 + rank)
    if config == "q35":
        return workloads.q35(seed=1000 + rank, steps=total_steps)
    if config == "draft":
        return workloads.draft(seed=1000 + rank)
    raise ValueError(config)


def is_decode(config):
    return config in ("c2", "c5", "q35")


def attention_flops(w, md, select=None):
    """Useful FLOPs of one attention launch: 4 * hq * head_dim per visible
    (query row, key) pair (QK^T and PV), with the workload's mask; `select`
    (bool per sequence) restricts the sum."""
    lengths = md.lengths(w.page).astype(np.int64)
    q = (md.qo[1:] - md.qo[:-1]).astype(np.int64)
    if w.causal:
        pairs = q * (lengths - q + 1) + q * (q - 1) // 2
    else:
        pairs = q * lengths
    if select is not None:
        pairs = pairs[select]
    return float(4 * w.hq * w.dim * int(pairs.sum()))


def decode_rows_mask(w, md):
    """Sequences served by the decode kernel: query rows x GQA group <= 16
    (the rest run on the tcgen05 kernel)."""
    q = (md.qo[1:] - md.qo[:-1]).astype(np.int64)
    return q * (w.hq // w.hkv) <= 16


class DecodeState:
    """Device-resident pools and per-layer step inputs for one GPU."""

    def __init__(self, w, physical_layers, seed, rows):
        import torch

        self.w = w
        dt = torch.bfloat16 if w.bf16 else torch.float16
        self.dt = dt
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        self.kpools, self.vpools = [], []
        for _ in range(physical_layers):
            for lst in (self.kpools, self.vpools):
                t = torch.empty(w.cache_slots, w.width, dtype=dt, device="cuda")
                t.normal_(0.0, w.scale, generator=g)
                lst.append(t)
        L = w.layers
        self.q = torch.randn(L, rows, w.hq, w.dim, generator=g, device="cuda", dtype=dt) * w.scale
        self.knew = torch.randn(L, rows, w.width, generator=g, device="cuda", dtype=dt) * w.scale
        self.vnew = torch.randn(L, rows, w.width, generator=g, device="cuda", dtype=dt) * w.scale
        self.out = torch.empty_like(self.q)
        self.slots = torch.empty(rows, dtype=torch.int64, device="cuda")
        self.physical = physical_layers


def run_ours(args, rank, world, local):
    import torch

    import fekv
    from fekv.dist import job_rate

    fekv.load()
    peak, peak_kind = measured_peak_gbs()
    total_steps = args.warmup + args.steps + args.e2e_steps + 1
    w = make_workload(args.config, rank, world, total_steps)
    if args.layers:
        w.layers = args.layers
    # physical layer pools: all layers when they fit, else pools are reused
    per_layer = 2 * w.cache_slots * w.width * 2
    free, _ = torch.cuda.mem_get_info()
    budget = min(free * 0.85, args.pool_gb * 1e9)
    physical = int(min(w.layers, max(1, budget // per_layer)))
    rows = w.metadata(0).rows
    st = DecodeState(w, physical, seed=7 + rank, rows=rows)
    plan = fekv.AttentionPlan(w.hq, w.hkv, w.dim, w.page, w.batch, w.max_pages(total_steps),
                              w.bf16, w.num_blocks)
    stream = torch.cuda.current_stream()
    decode = is_decode(args.config)
    cow = None
    if w.cow is not None:
        cow = tuple(torch.from_numpy(np.asarray(x, np.int32)).cuda() for x in w.cow)

    attn_ev = []
    md0 = w.metadata(0)
    dmask0 = decode_rows_mask(w, md0)
    # a step with both decode rows and multi-row sequences is timed in two
    # parts (decode kernel + merge, then the tcgen05 kernel): the same kernels
    # in the same order as one fe_attn_run, with an event between them
    mixed = (not is_decode(args.config)) and bool(dmask0.any()) and bool((~dmask0).any())
    sample_layer = w.layers // 2

    def step(s, record=False, host_io=None):
        md = w.metadata(s if decode else 0)
        if host_io is not None:
            host_io["h2d"]()
        plan.prepare(md.qo, md.kv, md.pages, md.last, md.batch, md.rows, False, stream)
        st.slots.copy_(torch.from_numpy(md.slots).pin_memory(), non_blocking=True)
        if cow is not None:
            # copy-on-write of the forked sequences' shared partial tail pages,
            # every layer in one launch (idempotent, so it can repeat per step)
            for l0 in range(0, st.physical, fekv._lib.FE_MAX_LAYERS):
                l1 = min(st.physical, l0 + fekv._lib.FE_MAX_LAYERS)
                fekv.copy_blocks(st.kpools[l0:l1], st.vpools[l0:l1], cow[0], cow[1], cow[2],
                                 w.page, w.width, w.num_blocks + 1, None, stream)
        for layer in range(w.layers):
            p = layer % st.physical
            # kernel durations for the roofline come from events around one
            # sampled layer per step: an event between two kernels ends their
            # programmatic overlap, so the other layers run without them
            timed = record and layer == sample_layer
            if host_io is not None:
                host_io["before"](layer)
            fekv.store(st.knew[layer], st.vnew[layer], st.kpools[p], st.vpools[p], st.slots,
                       md.rows, w.width, w.bf16, stream, w.cache_slots)
            if timed:
                e0 = torch.cuda.Event(enable_timing=True)
                em = torch.cuda.Event(enable_timing=True) if mixed else None
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            if timed and mixed:
                plan.attention(st.q[layer], st.kpools[p], st.vpools[p], st.out[layer], w.causal,
                               stream, lists=fekv._lib.FE_ATTN_LISTS_DECODE)
                em.record(stream)
                plan.attention(st.q[layer], st.kpools[p], st.vpools[p], st.out[layer], w.causal,
                               stream, lists=fekv._lib.FE_ATTN_LISTS_ROWS)
            else:
                plan.attention(st.q[layer], st.kpools[p], st.vpools[p], st.out[layer], w.causal,
                               stream)
            if timed:
                e1.record(stream)
                attn_ev.append((e0, em, e1))
            if host_io is not None:
                host_io["after"](layer)
        return md

    # warm-up
    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    barrier(world)

    # timed region (device-resident inputs)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    keys = 0
    flops = 0.0
    rows_flops = 0.0
    dec_keys = 0
    dec_qrows = 0
    t0.record(stream)
    for i in range(args.steps):
        md = step(args.warmup + i, record=True)
        lengths = md.lengths(w.page)
        keys += int(lengths.sum())
        flops += attention_flops(w, md)
        dm = decode_rows_mask(w, md)
        rows_flops += attention_flops(w, md, ~dm)
        dec_keys += int(lengths[dm].sum())
        dec_qrows += int((md.qo[1:] - md.qo[:-1])[dm].sum())
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    attn_ms = [a.elapsed_time(b) for a, _, b in attn_ev]
    dec_part_ms = [a.elapsed_time(m) for a, m, _ in attn_ev] if mixed else [0.0]
    rows_part_ms = [m.elapsed_time(b) for _, m, b in attn_ev] if mixed else [0.0]
    barrier(world)

    # algorithmic bytes / FLOPs of one attention launch (averaged over steps)
    per_launch_bytes = (keys / args.steps) * 2 * w.width * 2 + 2 * rows * w.hq * w.dim * 2
    per_launch_flops = flops / args.steps
    attn_avg_ms = float(np.mean(attn_ms))
    achieved_gbs = per_launch_bytes / (attn_avg_ms * 1e-3) / 1e9
    achieved_tflops = per_launch_flops / (attn_avg_ms * 1e-3) / 1e12
    rows_ms = float(np.mean(rows_part_ms))
    dec_ms = float(np.mean(dec_part_ms))
    rows_tflops = (rows_flops / args.steps) / (rows_ms * 1e-3) / 1e12 if mixed else 0.0
    dec_bytes = ((dec_keys / args.steps) * 2 * w.width * 2 +
                 2 * (dec_qrows / args.steps) * w.hq * w.dim * 2)
    dec_gbs = dec_bytes / (dec_ms * 1e-3) / 1e9 if mixed else 0.0

    # end-to-end through the C ABI with host buffers: per step, H2D of every
    # layer's q/k/v from pinned memory and D2H of every layer's output, on a
    # copy stream and per layer, so layer l+1's inputs arrive while layer l
    # computes and layer l's output leaves during layer l+1 (events keep a
    # buffer from being overwritten before the copy or kernel reading it).
    hq_pin = torch.empty(st.q.shape, dtype=st.dt, pin_memory=True)
    hk_pin = torch.empty(st.knew.shape, dtype=st.dt, pin_memory=True)
    hv_pin = torch.empty(st.vnew.shape, dtype=st.dt, pin_memory=True)
    ho_pin = torch.empty(st.out.shape, dtype=st.dt, pin_memory=True)
    hq_pin.copy_(st.q)
    hk_pin.copy_(st.knew)
    hv_pin.copy_(st.vnew)
    copy_stream = torch.cuda.Stream()
    h2d_ev = [torch.cuda.Event() for _ in range(w.layers)]
    comp_ev = [torch.cuda.Event() for _ in range(w.layers)]
    d2h_ev = [torch.cuda.Event() for _ in range(w.layers)]
    io_started = [False]

    def io_h2d():
        with torch.cuda.stream(copy_stream):
            for layer in range(w.layers):
                if io_started[0]:
                    copy_stream.wait_event(comp_ev[layer])  # last step's layer done with them
                st.q[layer].copy_(hq_pin[layer], non_blocking=True)
                st.knew[layer].copy_(hk_pin[layer], non_blocking=True)
                st.vnew[layer].copy_(hv_pin[layer], non_blocking=True)
                h2d_ev[layer].record(copy_stream)

    def io_before(layer):
        stream.wait_event(h2d_ev[layer])
        if io_started[0]:
            stream.wait_event(d2h_ev[layer])  # last step's output of this layer has left

    def io_after(layer):
        comp_ev[layer].record(stream)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(comp_ev[layer])
            ho_pin[layer].copy_(st.out[layer], non_blocking=True)
            d2h_ev[layer].record(copy_stream)
        if layer == w.layers - 1:
            io_started[0] = True

    io = {"h2d": io_h2d, "before": io_before, "after": io_after}
    h2d_bytes = (hq_pin.numel() + hk_pin.numel() + hv_pin.numel()) * 2
    d2h_bytes = ho_pin.numel() * 2
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    base = args.warmup + args.steps
    e0.record(stream)
    copy_stream.wait_stream(stream)  # no copy starts before the timed region
    for i in range(args.e2e_steps):
        step(base + i, host_io=io)
    stream.wait_stream(copy_stream)  # the last outputs are on the host
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    # this repo's kernels per layer-step: the append, the decode kernel and its
    # split-K merge when the step has decode rows, the tcgen05 kernel when it
    # has multi-row sequences
    inf = plan.info()
    launches_per_layer = (1 + (1 if inf["decode_items"] else 0) +
                          (1 if inf["split_sequences"] else 0) + (1 if inf["prefill_items"] else 0))
    stats = gather_floats([ms, e2e_ms, attn_avg_ms, achieved_gbs, keys, achieved_tflops,
                           rows_ms, rows_tflops, dec_ms, dec_gbs], world)
    plan.close()
    if rank != 0:
        return None
    ms_max = float(stats[:, 0].max())
    e2e_max = float(stats[:, 1].max())
    value = job_rate([rows * args.steps] * world, stats[:, 0])
    e2e_value = job_rate([rows * args.e2e_steps] * world, stats[:, 1])
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if w.bf16 else "f16",
        "data": "synthetic (seeded N(0,1) x scale K/V/q; random non-contiguous pages)",
        "config": {
            "workload": f"{w.name}: hq{w.hq}/hkv{w.hkv}/d{w.dim} page{w.page}, {w.layers} layers, "
                        f"{w.batch} seqs/GPU, 1 appended token + decode attention per layer-step",
            "seqs_per_gpu": w.batch, "layers": w.layers, "physical_layer_pools": physical,
            "mean_context": float(np.mean(w.cached)),
            "kv_bytes_per_step": float(per_launch_bytes * w.layers),
            "l2": "inputs larger than L2 (each layer's KV pages exceed 126 MB)",
            "parallelism": f"sequence-sharded x{world}, no hot-path collective",
        },
        "decode_attn_tbs": round(float(stats[:, 3].sum()) / 1e3, 4),
        "decode_attn_frac_of_peak": round(float(stats[:, 3].mean()) / peak, 4),
        "roofline": {
            "bound": "hbm",
            "achieved": round(float(stats[0, 3]), 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(float(stats[0, 3]) / peak, 4),
            "peak_kind": peak_kind,
            "kernel": "paged_decode_kernel",
            "algorithmic_bytes_per_launch": float(per_launch_bytes),
            "avg_launch_ms": round(float(stats[0, 2]), 5),
            "traffic": None,
            "traffic_source": None,
        },
        "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": int(d2h_bytes),
                "steps": args.e2e_steps},
        "gpu_launches": launches_per_layer * w.layers * args.steps,
        "clocks": clk,
    }
    if not decode:
        # prefill / verify workloads: the attention is a tensor-core contraction
        tpeak, tkind = measured_peak_tflops()
        line["metric"] = f"{w.name} paged attention TFLOP/s (tensor pipe) and query rows/s"
        line["unit"] = "rows/s"
        line["config"]["workload"] = (
            f"{w.name}: hq{w.hq}/hkv{w.hkv}/d{w.dim} page{w.page}, {w.layers} layers, "
            f"{w.batch} seqs, {rows} query rows per layer-step, "
            f"{'causal' if w.causal else 'non-causal'}"
            + (", copy-on-write of shared tail pages each step" if w.cow is not None else ""))
        line["config"]["attention_flops_per_step"] = per_launch_flops * w.layers
        line.pop("decode_attn_tbs")
        line.pop("decode_attn_frac_of_peak")
        line["roofline"] = {
            "bound": "tensor", "achieved": round(float(stats[0, 5]), 2), "peak": tpeak,
            "unit": "TFLOP/s", "frac": round(float(stats[0, 5]) / tpeak, 4), "peak_kind": tkind,
            "kernel": "paged_prefill_tc_kernel",
            "algorithmic_flops_per_launch": per_launch_flops,
            "avg_launch_ms": round(float(stats[0, 2]), 5), "traffic": None,
            "traffic_source": None,
        }
        ridge = tpeak * 1e12 / (peak * 1e9)
        if not mixed and row_step_bound(w.block_tables, per_launch_flops, per_launch_bytes,
                                        tpeak, peak) == "hbm":
            line["roofline"] = {
                "bound": "hbm", "achieved": round(float(stats[0, 3]), 1), "peak": peak,
                "unit": "GB/s", "frac": round(float(stats[0, 3]) / peak, 4),
                "peak_kind": peak_kind, "kernel": "paged_prefill_tc_kernel",
                "algorithmic_bytes_per_launch": float(per_launch_bytes),
                "flops_per_byte": round(per_launch_flops / per_launch_bytes, 1),
                "ridge_flops_per_byte": round(ridge, 1),
                "avg_launch_ms": round(float(stats[0, 2]), 5), "traffic": None,
                "traffic_source": None,
            }
            line["tensor_tflops"] = round(float(stats[0, 5]), 2)
        if mixed:
            # the step's multi-row sequences on the tcgen05 kernel, and its
            # decode rows on the decode kernel, each against its own roof
            line["roofline"].update({
                "achieved": round(float(stats[0, 7]), 2),
                "frac": round(float(stats[0, 7]) / tpeak, 4),
                "algorithmic_flops_per_launch": rows_flops / args.steps,
                "avg_launch_ms": round(float(stats[0, 6]), 5),
            })
            line["roofline_decode_rows"] = {
                "bound": "hbm", "achieved": round(float(stats[0, 9]), 1), "peak": peak,
                "unit": "GB/s", "frac": round(float(stats[0, 9]) / peak, 4),
                "peak_kind": peak_kind, "kernel": "paged_decode_kernel + decode_merge_kernel",
                "algorithmic_bytes_per_launch": dec_bytes,
                "avg_launch_ms": round(float(stats[0, 8]), 5),
            }
            line["attention_call_tflops"] = round(float(achieved_tflops), 2)
        line["gpu_launches"] = launches_per_layer * w.layers * args.steps + (
            args.steps if w.cow is not None else 0)
    rl = line["roofline"]
    units = rl.get("algorithmic_bytes_per_launch", rl.get("algorithmic_flops_per_launch"))
    rl["traffic"], rl["traffic_source"] = ncu_traffic(w.name, rl["kernel"], float(units))
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w, args)
    return line


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own ATen path (oracle/_ref), all host threads
# ---------------------------------------------------------------------------

def _ref_layer_step(ref, w, md, pools, inputs):
    kp, vp = pools
    q, kn, vn = inputs
    ref.store(kn, vn, kp, vp, md.slots)
    ref.prepare(md.qo, md.kv, md.pages, md.last)
    return ref.attention(q, kp, vp, w.causal)


def cpu_reference_setup(w, steps):
    import oracle
    from fekv import workloads

    threads = os.cpu_count() or 1
    oracle.ref_set_threads(threads)
    rng = np.random.default_rng(5)
    kp = workloads.random_bits(rng, (w.cache_slots, w.width), w.bf16, w.scale)
    vp = workloads.random_bits(rng, (w.cache_slots, w.width), w.bf16, w.scale)
    rows = w.metadata(0).rows
    q = workloads.random_bits(rng, (rows, w.hq, w.dim), w.bf16, w.scale)
    kn = workloads.random_bits(rng, (rows, w.width), w.bf16, w.scale)
    vn = workloads.random_bits(rng, (rows, w.width), w.bf16, w.scale)
    ref = oracle.RefAten(w.hq, w.hkv, w.dim, w.page, w.batch, w.max_pages(steps), w.bf16,
                         w.num_blocks)
    return ref, (kp, vp), (q, kn, vn), oracle.ref_get_threads()


def cpu_baseline(w, args):
    """One layer-step of the workload (store + prepare_plan + attention for
    every sequence) through the reference library, repeated for ~10 s."""
    import oracle

    if not oracle.ref_available():
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": "oracle/_ref not built"}
    ref, pools, inputs, threads = cpu_reference_setup(w, 4)
    md = w.metadata(0)
    _ref_layer_step(ref, w, md, pools, inputs)  # warm
    times = []
    t_end = time.time() + args.cpu_seconds
    while time.time() < t_end or len(times) < 3:
        t = time.perf_counter()
        _ref_layer_step(ref, w, md, pools, inputs)
        times.append(time.perf_counter() - t)
    ref.close()
    layer_s = statistics.median(times)
    rows = md.rows
    return {"value": round(rows / (layer_s * w.layers), 3),
            "unit": "tokens/s" if rows == w.batch else "rows/s",
            "cores": threads, "kind": "reference",
            "sample": f"{len(times)} layer-steps of {w.name} ({w.batch} seqs, {rows} rows: store + prepare_plan "
                      f"+ attention), median {layer_s*1e3:.1f} ms/layer, scaled to {w.layers} layers",
            "cpu_model": _cpu_model()}


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU/ATen implementation of the path
    (FlashEngine.cpp src/portable_gpu_ops.cpp compiled for the CPU), all host
    threads. Each step = one layer-step of the workload; rank 0 only."""
    if rank != 0:
        return None
    import oracle

    w = make_workload(args.config, 0, 1, 4)
    if not oracle.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libfe_ref_aten.so not built"}
    ref, pools, inputs, threads = cpu_reference_setup(w, 4)
    md = w.metadata(0)
    for _ in range(args.warmup):
        _ref_layer_step(ref, w, md, pools, inputs)
    t = time.perf_counter()
    for _ in range(args.steps):
        _ref_layer_step(ref, w, md, pools, inputs)
    el = time.perf_counter() - t
    ref.close()
    layer_s = el / args.steps
    value = w.batch / (layer_s * w.layers)
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(layer_s * 1e3 * w.layers, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if w.bf16 else "f16",
        "data": "synthetic", "config": {"workload": f"{w.name} (one layer-step per step, scaled "
                                                    f"to {w.layers} layers)",
                                        "seqs": w.batch, "layers": w.layers},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads,
                         "kind": "reference",
                         "sample": f"{args.steps} layer-steps of {w.name}, all sequences"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c2", "c3", "c4", "c5", "q35", "draft"], default="c2")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--pool-gb", type=float, default=150.0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (profiling a small case only)")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        rank, world, local = dist_setup(args.gpus)
        line = run_ours(args, rank, world, local)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
