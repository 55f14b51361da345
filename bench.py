"""Paged-KV decode benchmark (BASELINE metric: paged decode-attention achieved
TB/s and decode tokens/s at 1/2/4/8 B200).

One step = one decode step of the whole layer stack of the configured
workload: build the step's slot mapping and page tables on the host (the
reference's CudaModel::prepare), prepare the attention plan (one H2D copy),
then per layer append one K/V row per sequence and run paged decode attention.

Headline workload: C2 (Qwen3-8B attention shape: hq32/hkv8/d128 bf16, 36
layers, 64 sequences per GPU, contexts U[512,4096], page 16). Under torchrun
every rank runs one of 8 shards of one seeded list of 512 sequences, split so
that every shard holds the same KV bytes to within 0.1% (weak scaling). NCCL
is used only after the timed loops: to gather per-rank stats, per-rank output
checksums, and one sampled sequence per rank (its K/V, query and output),
which rank 0 recomputes in fp32 (`results`). No collective runs on the hot
path.

The same JSON line carries sub-objects measured in the same process:
  c5   BASELINE config 5 (hq64/hkv8, 64 layers, 128 sequences per GPU from
       1024 log-normal contexts 2k-32k, split-K decode + append, 32 steps),
       at every N, with its own roofline, e2e and results check;
  c3   chunked prefill + decode rows (tcgen05 kernel roofline), N=1 only;
  c4   shared-prefix verify blocks + copy-on-write (tcgen05), N=1 only;
  q35  head_dim 256 decode (hybrid-model full-attention layers), N=1 only;
  draft head_dim 256 16-row draft blocks under the full mask, N=1 only;
  ops  append / block copy / fused RoPE+append / accept / merge-free
       preparation timings against the HBM roofline, N=1 only.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c3|c4|c5|q35|draft]
                  [--sub c5,c3,c4,q35,draft,ops|none] [--layers L]
  python bench.py --impl reference ...   # the reference's own CPU/ATen path

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
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "flashengine.cpp_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "paged decode-attn achieved TB/s (% HBM peak); decode tokens/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TFLOPS_SUSTAINED = 1400.0
C5_STEPS = 32  # split-K decode + append for 32 steps


def measured_peak_gbs():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def measured_peak_tflops():
    """Sustained bf16 dense peak (a kernel timed inside a long step)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return FALLBACK_TFLOPS_SUSTAINED, "fallback (sustained)"


# DRAM bytes (read + write) per launch of each roofline kernel, from one
# `ncu --set full --clock-control none` capture of the same layer shape; the
# profile named beside each holds the command. Keyed by (workload, kernel) and
# checked against the algorithmic units (bytes or FLOPs) of the captured launch,
# so a changed workload reports null rather than a stale figure.
# The decode kernel streams every page once, so its traffic scales with the
# bytes a launch reads (the bench's contexts grow by one token per step); the
# tcgen05 kernel's DRAM bytes depend on L2 reuse of shared prefixes and are
# only reported for the captured launch itself.
NOMINAL_HBM_GBS = 8000.0  # B200 HBM3e, nominal (the north star's "roughly 8 TB/s")

NCU_TRAFFIC = {
    ("C2", "paged_decode_kernel"): (632665344, 625496064.0, True,
                                    "profiles/paged_decode_kernel_c2.md"),
    ("C5", "paged_decode_kernel"): (4732976768, 4716232704.0, True,
                                    "profiles/paged_decode_kernel_c5.md"),
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


# ---------------------------------------------------------------------------
# clocks sampled during a timed region
# ---------------------------------------------------------------------------

# NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
_REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                "hw_thermal_slowdown": 0x40}


class ClockSampler:
    """SM clock, power and clock-event reasons of this rank's GPU, read every
    `period_ms` from a host thread through NVML while a timed region runs (a
    few-ms period gives a usable sample count even for a region of a tenth of
    a second). Falls back to `nvidia-smi -lms 200` when NVML is unavailable.
    Only reads the GPU's state; changes nothing."""

    def __init__(self, device_index: int, period_ms: float = 2.0):
        self.dev = device_index
        self.period = period_ms / 1e3
        self.samples = []
        self._stop = threading.Event()
        self._thread = None
        self._proc = None
        self._path = None
        self.source = None

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        try:
            import torch

            uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(
                uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def start(self):
        try:
            nv, h = self._nvml_handle()
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.source = f"nvml every {self.period * 1e3:.0f} ms"

            def loop():
                while not self._stop.is_set():
                    try:
                        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        pw = nv.nvmlDeviceGetPowerUsage(h) / 1e3
                        rs = reasons_fn(h)
                        self.samples.append((float(sm), float(mx), pw, int(rs)))
                    except Exception:
                        pass
                    time.sleep(self.period)

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
            return
        except Exception:
            pass
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        fd, self._path = tempfile.mkstemp(prefix="fe_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.dev)],
                stdout=open(self._path, "w"), stderr=subprocess.DEVNULL)
            self.source = "nvidia-smi every 200 ms"
        except Exception:
            self._proc = None

    def stop(self) -> dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join(2)
        elif self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            with open(self._path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 7:
                        continue
                    try:
                        bits = sum(_REASON_BITS[n] for n, v in zip(names, parts[3:7])
                                   if v.lower() == "active")
                        self.samples.append((float(parts[0]), float(parts[1]),
                                             float(parts[2]), bits))
                    except ValueError:
                        continue
            os.unlink(self._path)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0,
                    "reasons": ["no clock source"]}
        sm = [s[0] for s in self.samples]
        reasons = sorted(n for n, bit in _REASON_BITS.items()
                         if any(s[3] & bit for s in self.samples))
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(s[1] for s in self.samples),
                "sm_mhz_min": min(sm), "power_w_max": round(max(s[2] for s in self.samples), 1),
                "samples": len(sm), "source": self.source, "reasons": reasons}


# ---------------------------------------------------------------------------
# distributed plumbing (one process per GPU; no collective on the hot path)
# ---------------------------------------------------------------------------

def dist_setup():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch

    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def gather_floats(values, world, device="cuda"):
    """All-gather a small float64 vector per rank (after timing only)."""
    from fekv.dist import gather_floats as _gather

    return _gather(values, world, device=device)


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

def make_workload(config, rank, world, total_steps):
    from fekv import workloads

    if config == "c2":
        return workloads.c2_shard(shard=rank, nshards=max(world, 8), steps=total_steps)
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


def physical_pools(w, pool_gb, free_bytes=None):
    """Layer pools held on the GPU: all layers when they fit in the budget,
    else fewer, reused round-robin (layer l uses pool l mod P); each pool is
    far larger than L2, so reuse adds no cache effect."""
    per_layer = 2 * w.cache_slots * w.width * 2
    budget = pool_gb * 1e9 if free_bytes is None else min(free_bytes * 0.85, pool_gb * 1e9)
    return int(min(w.layers, max(1, budget // per_layer)))


def config_dict(w, world, physical):
    """The workload description both arms print (same dict, same config)."""
    return {
        "workload": f"{w.name}: hq{w.hq}/hkv{w.hkv}/d{w.dim} page{w.page}, {w.layers} layers, "
                    f"{w.batch} seqs/GPU, "
                    + ("1 appended token + decode attention per layer-step" if int(w.rows.max()) == 1
                       else f"{int(w.rows.sum())} query rows per layer-step, "
                            f"{'causal' if w.causal else 'non-causal'}"
                            + (", copy-on-write of shared tail pages each step"
                               if w.cow is not None else "")),
        "seqs_per_gpu": w.batch, "layers": w.layers, "physical_layer_pools": physical,
        "mean_context": round(float(np.mean(w.cached)), 2),
        "shard": w.notes.get("shard"),
        "l2": "inputs larger than L2 (each layer's KV pages exceed 126 MB)",
        "parallelism": f"sequence-sharded x{world}, no hot-path collective",
        "timed_step": "plan preparation (host planner + H2D), slot upload, then append + "
                      "attention per layer; the scheduler's per-step block tables and slot "
                      "mapping are built before timing",
    }


def dense_attention_f32(q, k, v, hq, hkv, causal):
    """fp32 softmax attention of one sequence (result check after timing):
    q [rows, hq, d], k/v [length, hkv, d] -> [rows, hq, d]; causal rows are
    bottom-right aligned as in src/portable_gpu_ops.cpp:31."""
    import torch

    rows, _, d = q.shape
    length = k.shape[0]
    G = hq // hkv
    kk = k.float().repeat_interleave(G, dim=1).permute(1, 2, 0)
    vv = v.float().repeat_interleave(G, dim=1).permute(1, 0, 2)
    logits = torch.bmm(q.float().permute(1, 0, 2), kk) / float(np.sqrt(d))
    if causal:
        t = torch.arange(length, device=q.device)
        r = torch.arange(rows, device=q.device).unsqueeze(1)
        logits = logits.masked_fill(~(t.unsqueeze(0) <= length - rows + r).unsqueeze(0),
                                    float("-inf"))
    return torch.bmm(torch.softmax(logits, -1), vv).permute(1, 0, 2)


def check_sample(q, k, v, out, hq, hkv, causal):
    """(ok, max_abs_err) of `out` against the fp32 recomputation: within 2e-3
    plus one output ulp, the parity tests' bar."""
    import torch

    ref = dense_attention_f32(q, k, v, hq, hkv, causal)
    ref16 = ref.to(out.dtype).float()
    mant = 7 if out.dtype == torch.bfloat16 else 10
    ulp = torch.exp2(torch.floor(torch.log2(ref16.abs().clamp_min(2.0 ** -126))) - mant)
    err = (out.float() - ref16).abs()
    return bool((err <= 2e-3 + ulp).all().item()), float(err.max().item())


# ---------------------------------------------------------------------------
# one GPU's share of a workload
# ---------------------------------------------------------------------------

class Runner:
    """Device-resident pools, per-layer step inputs and the attention plan of
    one rank. step(): host slot mapping + plan prepare, then per layer the
    append and the attention (and, for C4, the copy-on-write of the forked
    sequences' shared tail pages once per step)."""

    def __init__(self, config, rank, world, steps, warmup, e2e_steps, pool_gb, layers=0):
        import torch

        import fekv

        self.config, self.rank, self.world = config, rank, world
        self.steps, self.warmup, self.e2e_steps = steps, warmup, e2e_steps
        self.total_steps = warmup + steps + e2e_steps + 1
        w = make_workload(config, rank, world, self.total_steps)
        if layers:
            w.layers = layers
        self.w = w
        free, _ = torch.cuda.mem_get_info()
        self.physical = physical_pools(w, pool_gb, free)
        self.decode = is_decode(config)
        dt = torch.bfloat16 if w.bf16 else torch.float16
        self.dt = dt
        g = torch.Generator(device="cuda")
        g.manual_seed(7 + rank)
        self.kpools, self.vpools = [], []
        for _ in range(self.physical):
            for lst in (self.kpools, self.vpools):
                t = torch.empty(w.cache_slots, w.width, dtype=dt, device="cuda")
                t.normal_(0.0, w.scale, generator=g)
                lst.append(t)
        self.rows = w.metadata(0).rows
        L, rows = w.layers, self.rows
        self.q = torch.randn(L, rows, w.hq, w.dim, generator=g, device="cuda", dtype=dt) * w.scale
        self.knew = torch.randn(L, rows, w.width, generator=g, device="cuda", dtype=dt) * w.scale
        self.vnew = torch.randn(L, rows, w.width, generator=g, device="cuda", dtype=dt) * w.scale
        self.out = torch.empty_like(self.q)
        self.slots = torch.empty(rows, dtype=torch.int64, device="cuda")
        self.plan = fekv.AttentionPlan(w.hq, w.hkv, w.dim, w.page, w.batch,
                                       w.max_pages(self.total_steps), w.bf16, w.num_blocks)
        self.stream = torch.cuda.current_stream()
        self.cow = None
        if w.cow is not None:
            self.cow = tuple(torch.from_numpy(np.asarray(x, np.int32)).cuda() for x in w.cow)
        md0 = w.metadata(0)
        dm = decode_rows_mask(w, md0)
        # a step with both decode rows and multi-row sequences runs the decode
        # kernel and the tcgen05 kernel side by side (one fe_attn_run); the
        # per-kernel rooflines come from a serial full-width pass after timing
        self.mixed = (not self.decode) and bool(dm.any()) and bool((~dm).any())
        self.sample_layer = w.layers // 2
        self.attn_ev = []
        self.last_md = None
        self.side_by_side = False
        # The engine's per-step scheduler output (block tables and the slot
        # mapping of CudaModel::prepare, made here by the numpy stand-in
        # fekv.metadata, ~0.4 ms of Python per q35 step) is built before any
        # timing, each step's slots in their own pinned buffer; the timed step
        # is this library's work: plan preparation (host planner + one H2D
        # copy), the slots' upload, append and attention. With the stand-in
        # inside the loop the short q35 and draft steps were host-bound.
        keys = range(self.total_steps) if self.decode else [0]
        self.step_md = {k: w.metadata(k) for k in keys}
        self.step_slots = {k: torch.from_numpy(md.slots).pin_memory()
                           for k, md in self.step_md.items()}

    def step(self, s, record=False, host_io=None):
        import torch

        import fekv

        w = self.w
        key = s if self.decode else 0
        if key not in self.step_md:
            self.step_md[key] = w.metadata(key)
            self.step_slots[key] = torch.from_numpy(self.step_md[key].slots).pin_memory()
        md = self.step_md[key]
        self.plan.prepare(md.qo, md.kv, md.pages, md.last, md.batch, md.rows, False, self.stream)
        # a pinned buffer per step: the host runs steps ahead of the GPU (a
        # step's buffer is not rewritten while its copy may still be queued)
        self.slots.copy_(self.step_slots[key], non_blocking=True)
        if self.cow is not None:
            # copy-on-write of the forked sequences' shared partial tail pages,
            # every layer in one launch (idempotent, so it can repeat per step)
            for l0 in range(0, self.physical, fekv._lib.FE_MAX_LAYERS):
                l1 = min(self.physical, l0 + fekv._lib.FE_MAX_LAYERS)
                fekv.copy_blocks(self.kpools[l0:l1], self.vpools[l0:l1], *self.cow, w.page,
                                 w.width, w.num_blocks + 1, None, self.stream)
        if host_io is not None:
            host_io["start"]()
        for layer in range(w.layers):
            p = layer % self.physical
            # kernel durations for the roofline come from events around one
            # sampled layer per step: an event between two kernels ends their
            # programmatic overlap, so the other layers run without them
            timed = record and layer == self.sample_layer
            if host_io is not None:
                host_io["layer_start"](layer)
            fekv.store(self.knew[layer], self.vnew[layer], self.kpools[p], self.vpools[p],
                       self.slots, md.rows, w.width, w.bf16, self.stream, w.cache_slots)
            if timed:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
            self.plan.attention(self.q[layer], self.kpools[p], self.vpools[p], self.out[layer],
                                w.causal, self.stream)
            if timed:
                e1.record(self.stream)
                self.attn_ev.append((e0, e1))
            if host_io is not None:
                host_io["layer_end"](layer)
        if host_io is not None:
            host_io["end"]()
        self.last_md = md
        return md

    def run_device(self, clock_dev):
        """W untimed steps, then K timed steps between CUDA events on the
        launching stream, bracketed by barrier + synchronize; NVML clocks
        sampled throughout the timed region."""
        import torch

        w = self.w
        for s in range(self.warmup):
            self.step(s)
        torch.cuda.synchronize()
        if self.mixed:
            inf = self.plan.info()
            sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
            self.side_by_side = inf["grid_ctas"] <= sms
        barrier(self.world)
        clocks = ClockSampler(clock_dev)
        clocks.start()
        time.sleep(0.05)
        barrier(self.world)
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        keys = flops = rows_flops = 0.0
        dec_keys = dec_qrows = 0
        t0.record(self.stream)
        for i in range(self.steps):
            md = self.step(self.warmup + i, record=True)
            lengths = md.lengths(w.page)
            keys += int(lengths.sum())
            flops += attention_flops(w, md)
            dm = decode_rows_mask(w, md)
            rows_flops += attention_flops(w, md, ~dm)
            dec_keys += int(lengths[dm].sum())
            dec_qrows += int((md.qo[1:] - md.qo[:-1])[dm].sum())
        t1.record(self.stream)
        torch.cuda.synchronize()
        clk = clocks.stop()
        barrier(self.world)
        ms = t0.elapsed_time(t1)
        K = self.steps
        attn_ms = [a.elapsed_time(b) for a, b in self.attn_ev]
        attn_avg_ms = float(np.mean(attn_ms))
        per_launch_bytes = (keys / K) * 2 * w.width * 2 + 2 * self.rows * w.hq * w.dim * 2
        per_launch_flops = flops / K
        st = {"ms": ms, "attn_avg_ms": attn_avg_ms, "kv_bytes_per_launch": per_launch_bytes,
              "flops_per_launch": per_launch_flops,
              "gbs": per_launch_bytes / (attn_avg_ms * 1e-3) / 1e9,
              "tflops": per_launch_flops / (attn_avg_ms * 1e-3) / 1e12,
              "step_gbs": per_launch_bytes * w.layers * K / (ms * 1e-3) / 1e9,
              "rows_ms": 0.0, "rows_tflops": 0.0, "dec_ms": 0.0, "dec_gbs": 0.0,
              "rows_flops_per_launch": rows_flops / K, "dec_bytes_per_launch": 0.0}
        if self.mixed:
            rows_ms, dec_ms = self.time_parts()
            dec_bytes = (dec_keys / K) * 2 * w.width * 2 + 2 * (dec_qrows / K) * w.hq * w.dim * 2
            st.update({"rows_ms": rows_ms, "rows_tflops": (rows_flops / K) / (rows_ms * 1e-3) / 1e12,
                       "dec_ms": dec_ms, "dec_gbs": dec_bytes / (dec_ms * 1e-3) / 1e9,
                       "dec_bytes_per_launch": dec_bytes})
        self.clocks = clk
        return st

    def time_parts(self):
        """Per-kernel durations of a mixed step at full width: a plan
        prepared in graph mode runs the decode list (decode kernel + merge)
        and the row list (tcgen05 kernel) one after the other on every SM;
        K layer-calls of each, on the layer pools in turn, between CUDA
        events. Untimed by the step clock (after the timed region)."""
        import torch

        import fekv

        w = self.w
        md = w.metadata(0)
        plan = fekv.AttentionPlan(w.hq, w.hkv, w.dim, w.page, w.batch,
                                  w.max_pages(self.total_steps), w.bf16, w.num_blocks)
        plan.prepare(md.qo, md.kv, md.pages, md.last, md.batch, md.rows, True, self.stream)
        res = []
        for lists in (fekv._lib.FE_ATTN_LISTS_ROWS, fekv._lib.FE_ATTN_LISTS_DECODE):
            for i in range(3):
                p = i % self.physical
                plan.attention(self.q[0], self.kpools[p], self.vpools[p], self.out[0], w.causal,
                               self.stream, lists=lists)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            for i in range(self.steps):
                p = i % self.physical
                plan.attention(self.q[0], self.kpools[p], self.vpools[p], self.out[0], w.causal,
                               self.stream, lists=lists)
            e1.record(self.stream)
            torch.cuda.synchronize()
            res.append(e0.elapsed_time(e1) / self.steps)
        plan.close()
        return res[0], res[1]

    def run_e2e(self, device_ms_per_step):
        """The same steps through the C ABI with HOST buffers: per step, the
        H2D of every layer's q/k/v from pinned memory and the D2H of every
        layer's output, inside the timed region. Inputs and outputs are
        double-buffered on the device: a copy stream brings step i+1's inputs
        in while step i computes and takes step i's outputs out while step
        i+1 computes, and the compute stream waits once per step (a wait
        between two layers' kernels would end their programmatic overlap).
        Inputs and outputs get a stream each, so that the two directions of
        the host link run at once, unless a step's copies take under 30% of
        its kernel time: there one stream measured faster (C2: 4.03 ms per
        step against 4.13). The first step's inputs arrive and the last
        step's outputs leave in four layer chunks, the first step's layers
        waiting only for their own chunk, so one chunk of each stays exposed
        rather than a whole step's copies."""
        import torch

        w = self.w
        hq_pin = torch.empty(self.q.shape, dtype=self.dt, pin_memory=True)
        hk_pin = torch.empty(self.knew.shape, dtype=self.dt, pin_memory=True)
        hv_pin = torch.empty(self.vnew.shape, dtype=self.dt, pin_memory=True)
        ho_pin = torch.empty(self.out.shape, dtype=self.dt, pin_memory=True)
        hq_pin.copy_(self.q)
        hk_pin.copy_(self.knew)
        hv_pin.copy_(self.vnew)
        self.pins = (hq_pin, hk_pin, hv_pin, ho_pin)
        sets = [(self.q, self.knew, self.vnew, self.out),
                tuple(torch.empty_like(t) for t in (self.q, self.knew, self.vnew, self.out))]
        h2d_bytes = (hq_pin.numel() + hk_pin.numel() + hv_pin.numel()) * 2
        d2h_bytes = ho_pin.numel() * 2
        copy_ms = (h2d_bytes + d2h_bytes) / 50e9 * 1e3  # at ~50 GB/s per direction
        dual = copy_ms > 0.3 * device_ms_per_step
        in_stream = torch.cuda.Stream()
        out_stream = torch.cuda.Stream() if dual else in_stream
        h2d_ev = [torch.cuda.Event() for _ in range(2)]
        comp_ev = [torch.cuda.Event() for _ in range(2)]
        d2h_ev = [torch.cuda.Event() for _ in range(2)]
        n = self.e2e_steps
        state = {"i": 0}
        chunks = min(4, w.layers)
        bounds = [w.layers * c // chunks for c in range(chunks + 1)]
        first_ev = [torch.cuda.Event() for _ in range(chunks)]
        last_ev = [torch.cuda.Event() for _ in range(chunks)]

        def h2d_first():
            with torch.cuda.stream(in_stream):
                q, k, v, _ = sets[0]
                for c in range(chunks):
                    l0, l1 = bounds[c], bounds[c + 1]
                    q[l0:l1].copy_(hq_pin[l0:l1], non_blocking=True)
                    k[l0:l1].copy_(hk_pin[l0:l1], non_blocking=True)
                    v[l0:l1].copy_(hv_pin[l0:l1], non_blocking=True)
                    first_ev[c].record(in_stream)
                h2d_ev[0].record(in_stream)

        def d2h_chunk(b, c, ev):
            with torch.cuda.stream(out_stream):
                out_stream.wait_event(ev)
                l0, l1 = bounds[c], bounds[c + 1]
                ho_pin[l0:l1].copy_(sets[b][3][l0:l1], non_blocking=True)

        def h2d(b, after_compute):
            with torch.cuda.stream(in_stream):
                if after_compute:
                    in_stream.wait_event(comp_ev[b])  # the step before last is done with set b
                q, k, v, _ = sets[b]
                q.copy_(hq_pin, non_blocking=True)
                k.copy_(hk_pin, non_blocking=True)
                v.copy_(hv_pin, non_blocking=True)
                h2d_ev[b].record(in_stream)

        def io_start():
            i = state["i"]
            b = i % 2
            self.q, self.knew, self.vnew, self.out = sets[b]
            if i > 0:  # the first step waits per chunk (layer_start)
                self.stream.wait_event(h2d_ev[b])
            if i >= 2:
                self.stream.wait_event(d2h_ev[b])  # step i-2's outputs have left set b
            if i + 1 < n:
                h2d(1 - b, i >= 1)

        def layer_start(layer):
            if state["i"] == 0 and layer in bounds[:-1]:
                self.stream.wait_event(first_ev[bounds.index(layer)])

        def layer_end(layer):
            i = state["i"]
            if i == n - 1 and layer + 1 in bounds[1:-1]:
                c = bounds.index(layer + 1) - 1
                last_ev[c].record(self.stream)
                d2h_chunk(i % 2, c, last_ev[c])

        def io_end():
            i = state["i"]
            b = i % 2
            comp_ev[b].record(self.stream)
            if i == n - 1:  # earlier chunks left in layer_end
                d2h_chunk(b, chunks - 1, comp_ev[b])
            else:
                with torch.cuda.stream(out_stream):
                    out_stream.wait_event(comp_ev[b])
                    ho_pin.copy_(sets[b][3], non_blocking=True)
            d2h_ev[b].record(out_stream)
            state["i"] = i + 1

        io = {"start": io_start, "end": io_end, "layer_start": layer_start,
              "layer_end": layer_end}
        barrier(self.world)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        base = self.warmup + self.steps
        e0.record(self.stream)
        in_stream.wait_stream(self.stream)  # no copy starts before the timed region
        out_stream.wait_stream(self.stream)
        h2d_first()
        for i in range(n):
            self.step(base + i, host_io=io)
        self.stream.wait_stream(in_stream)
        self.stream.wait_stream(out_stream)  # the last outputs are on the host
        e1.record(self.stream)
        torch.cuda.synchronize()
        barrier(self.world)
        # the results check reads the last step's buffers
        self.q, self.knew, self.vnew, self.out = sets[(n - 1) % 2 if n > 0 else 0]
        return {"e2e_ms": e0.elapsed_time(e1), "h2d_bytes": float(h2d_bytes),
                "d2h_bytes": float(d2h_bytes), "copy_streams": 2.0 if dual else 1.0}

    def host_copy_rates(self):
        """One step's H2D inputs and D2H outputs copied alone (every rank at
        once, between barriers): the host-link rate each rank gets while all
        ranks copy, which bounds the end-to-end leg."""
        import torch

        hq_pin, hk_pin, hv_pin, ho_pin = self.pins
        res = {}
        for name, pairs in (("h2d", [(self.q, hq_pin), (self.knew, hk_pin),
                                     (self.vnew, hv_pin)]),
                            ("d2h", [(ho_pin, self.out)])):
            nbytes = sum(dst.numel() * 2 for dst, _ in pairs)
            best = None
            for _ in range(3):
                barrier(self.world)
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
                for dst, src in pairs:
                    dst.copy_(src, non_blocking=True)
                e1.record(self.stream)
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1)
                best = ms if best is None else min(best, ms)
            res[f"{name}_gbs"] = nbytes / (best * 1e-3) / 1e9
            res[f"{name}_ms"] = best
        barrier(self.world)
        return res

    def sample(self):
        """The longest sequence of this rank's shard in the last executed step:
        its K/V rows (gathered through its block table from the last layer's
        pool), query rows and output rows of that layer."""
        import torch

        w, md = self.w, self.last_md
        layer = w.layers - 1
        p = layer % self.physical
        lengths = md.lengths(w.page)
        b = int(np.argmax(lengths))
        n = int(lengths[b])
        t = np.arange(n)
        pages = md.pages[md.kv[b]:md.kv[b + 1]].astype(np.int64)
        slots = torch.from_numpy(pages[t // w.page] * w.page + t % w.page).cuda()
        k = self.kpools[p].index_select(0, slots).view(n, w.hkv, w.dim)
        v = self.vpools[p].index_select(0, slots).view(n, w.hkv, w.dim)
        q0, q1 = int(md.qo[b]), int(md.qo[b + 1])
        return n, k, v, self.q[layer, q0:q1].contiguous(), self.out[layer, q0:q1].contiguous()

    def checksums(self):
        o = self.out.float()
        return [float(o.sum().item()), float(o.abs().sum().item())]

    def launches_per_step(self):
        inf = self.plan.info()
        per_layer = (1 + (1 if inf["decode_items"] else 0) + (1 if inf["split_sequences"] else 0)
                     + (1 if inf["prefill_items"] else 0))
        return per_layer * self.w.layers + (1 if self.cow is not None else 0)

    def close(self):
        import torch

        self.plan.close()
        self.kpools = self.vpools = None
        self.q = self.knew = self.vnew = self.out = None
        self.pins = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def verify_results(runner, world):
    """After timing: every rank's output checksums, and one sampled sequence
    per rank (K/V, q, output) gathered over NCCL and recomputed in fp32 on
    rank 0. Returns the `results` object on rank 0 (None elsewhere)."""
    import torch

    n, k, v, q, out = runner.sample()
    sums = runner.checksums()
    info = gather_floats([float(n)] + sums, world, device=k.device.type)
    w = runner.w
    if world > 1:
        import torch.distributed as dist

        maxlen = int(info[:, 0].max())
        pad = lambda t: torch.cat([t, t.new_zeros((maxlen - t.shape[0],) + tuple(t.shape[1:]))])  # noqa: E731
        ks, vs = [torch.empty((maxlen,) + tuple(k.shape[1:]), dtype=k.dtype, device=k.device)
                  for _ in range(world)], \
                 [torch.empty((maxlen,) + tuple(v.shape[1:]), dtype=v.dtype, device=v.device)
                  for _ in range(world)]
        qs = [torch.empty_like(q) for _ in range(world)]
        os_ = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(ks, pad(k).contiguous())
        dist.all_gather(vs, pad(v).contiguous())
        dist.all_gather(qs, q)
        dist.all_gather(os_, out)
    else:
        ks, vs, qs, os_ = [k], [v], [q], [out]
    if runner.rank != 0:
        return None
    oks, errs = [], []
    for r in range(world):
        nr = int(info[r, 0])
        ok, err = check_sample(qs[r], ks[r][:nr], vs[r][:nr], os_[r], w.hq, w.hkv, w.causal)
        oks.append(ok)
        errs.append(err)
    return {"ok": bool(all(oks)), "ranks_checked": world, "per_rank_ok": oks,
            "max_abs_err": round(max(errs), 6),
            "checked": "the longest sequence of each rank's shard, last layer of the final step, "
                       "recomputed in fp32 on rank 0 from K/V gathered over NCCL "
                       "(bar: 2e-3 + 1 output ulp)",
            "checksums": [[round(float(x), 3) for x in info[r, 1:]] for r in range(world)]}


STAT_KEYS = ["ms", "attn_avg_ms", "kv_bytes_per_launch", "flops_per_launch", "gbs", "tflops",
             "step_gbs", "rows_ms", "rows_tflops", "dec_ms", "dec_gbs", "rows_flops_per_launch",
             "dec_bytes_per_launch", "e2e_ms", "h2d_bytes", "d2h_bytes", "h2d_gbs", "d2h_gbs",
             "h2d_ms", "d2h_ms", "copy_streams"]


def measure(config, args, rank, world, local, steps, with_e2e=True, verify=True):
    """Run one workload on every rank; returns (rank-0 section or None, runner
    stats table [world, len(STAT_KEYS)], runner) — the runner already closed."""
    r = Runner(config, rank, world, steps, args.warmup, args.e2e_steps if with_e2e else 0,
               args.pool_gb, args.layers if config == args.config else 0)
    st = r.run_device(local)
    if with_e2e:
        st.update(r.run_e2e(st["ms"] / r.steps))
        st.update(r.host_copy_rates())
    results = verify_results(r, world) if verify else None
    table = gather_floats([float(st.get(k, 0.0)) for k in STAT_KEYS], world)
    launches = r.launches_per_step()
    section = None
    if rank == 0:
        section = summarize(r, table, results, launches, with_e2e)
    r.close()
    return section, table, r


def summarize(r, table, results, launches, with_e2e):
    """The JSON fields of one workload from all ranks' stats."""
    from fekv.dist import job_rate

    w = r.w
    col = {k: table[:, i] for i, k in enumerate(STAT_KEYS)}
    world = table.shape[0]
    K = r.steps
    peak, peak_kind = measured_peak_gbs()
    tpeak, tkind = measured_peak_tflops()
    value = job_rate([r.rows * K] * world, col["ms"])
    sec = {
        "value": round(value, 2), "unit": "tokens/s" if r.decode else "rows/s",
        "steps": K, "ms_per_step": round(float(col["ms"].max()) / K, 4),
        "config": config_dict(w, world, r.physical),
        "per_rank": {
            "ms_per_step": [round(float(x) / K, 4) for x in col["ms"]],
            "kv_bytes_per_step": [float(x) * w.layers for x in col["kv_bytes_per_launch"]],
            "step_gbs": [round(float(x), 1) for x in col["step_gbs"]],
            "sampled_launch_gbs": [round(float(x), 1) for x in col["gbs"]],
        },
        # all ranks' algorithmic KV bytes over the slowest rank's time
        "job_kv_tbs": round(float((col["kv_bytes_per_launch"] * w.layers * K).sum())
                            / (float(col["ms"].max()) * 1e-3) / 1e12, 4),
        "gpu_launches": launches * K,
        "clocks": r.clocks,
    }
    if r.decode:
        sec["roofline"] = {
            "bound": "hbm", "achieved": round(float(col["gbs"][0]), 1), "peak": peak,
            "unit": "GB/s", "frac": round(float(col["gbs"][0]) / peak, 4),
            "peak_kind": peak_kind, "kernel": "paged_decode_kernel",
            "algorithmic_bytes_per_launch": float(col["kv_bytes_per_launch"][0]),
            "avg_launch_ms": round(float(col["attn_avg_ms"][0]), 5),
            "timing": "CUDA events around the attention call (decode kernel + split-K merge) "
                      "of one sampled layer per step",
            # the same bytes over the whole step's time (append, merge, PDL overlap included)
            "step_level_gbs": round(float(col["step_gbs"][0]), 1),
            "step_level_frac": round(float(col["step_gbs"][0]) / peak, 4),
            # against B200's nominal HBM3e rate, for context (`frac` is of the measured peak)
            "frac_nominal": round(float(col["gbs"][0]) / NOMINAL_HBM_GBS, 4),
        }
    else:
        per_launch_flops = float(col["flops_per_launch"][0])
        per_launch_bytes = float(col["kv_bytes_per_launch"][0])
        sec["roofline"] = {
            "bound": "tensor", "achieved": round(float(col["tflops"][0]), 2), "peak": tpeak,
            "unit": "TFLOP/s", "frac": round(float(col["tflops"][0]) / tpeak, 4),
            "peak_kind": tkind, "kernel": "paged_prefill_tc_kernel",
            "algorithmic_flops_per_launch": per_launch_flops,
            "avg_launch_ms": round(float(col["attn_avg_ms"][0]), 5),
        }
        if not r.mixed and row_step_bound(w.block_tables, per_launch_flops, per_launch_bytes,
                                          tpeak, peak) == "hbm":
            sec["roofline"] = {
                "bound": "hbm", "achieved": round(float(col["gbs"][0]), 1), "peak": peak,
                "unit": "GB/s", "frac": round(float(col["gbs"][0]) / peak, 4),
                "peak_kind": peak_kind, "kernel": "paged_prefill_tc_kernel",
                "algorithmic_bytes_per_launch": per_launch_bytes,
                "flops_per_byte": round(per_launch_flops / per_launch_bytes, 1),
                "ridge_flops_per_byte": round(tpeak * 1e12 / (peak * 1e9), 1),
                "avg_launch_ms": round(float(col["attn_avg_ms"][0]), 5),
            }
            sec["tensor_tflops"] = round(float(col["tflops"][0]), 2)
        if r.mixed:
            # the tcgen05 kernel on the step's prefill rows and the decode
            # kernel on its decode rows, each at full width one after the
            # other (graph-mode plan, after the timed steps)
            sec["roofline"].update({
                "achieved": round(float(col["rows_tflops"][0]), 2),
                "frac": round(float(col["rows_tflops"][0]) / tpeak, 4),
                "algorithmic_flops_per_launch": float(col["rows_flops_per_launch"][0]),
                "avg_launch_ms": round(float(col["rows_ms"][0]), 5),
                "timing": "tcgen05 kernel alone at full width (serial pass after the timed steps)",
            })
            sec["roofline_decode_rows"] = {
                "bound": "hbm", "achieved": round(float(col["dec_gbs"][0]), 1), "peak": peak,
                "unit": "GB/s", "frac": round(float(col["dec_gbs"][0]) / peak, 4),
                "peak_kind": peak_kind, "kernel": "paged_decode_kernel + decode_merge_kernel",
                "algorithmic_bytes_per_launch": float(col["dec_bytes_per_launch"][0]),
                "avg_launch_ms": round(float(col["dec_ms"][0]), 5),
                "timing": "decode list alone at full width (serial pass after the timed steps)",
            }
            # the call the timed steps make: both kernels side by side
            call_ms = float(col["attn_avg_ms"][0])
            sec["attention_call"] = {
                "avg_ms": round(call_ms, 5),
                "side_by_side": bool(r.side_by_side),
                "serial_parts_ms": round(float(col["rows_ms"][0] + col["dec_ms"][0]), 5),
                "tflops": round(float(col["tflops"][0]), 2),
                "kv_gbs": round(float(col["gbs"][0]), 1),
                "timing": "CUDA events around fe_attn_run of one sampled layer per timed step",
            }
            sec["attention_call_tflops"] = round(float(col["tflops"][0]), 2)
    rl = sec["roofline"]
    units = rl.get("algorithmic_bytes_per_launch", rl.get("algorithmic_flops_per_launch"))
    rl["traffic"], rl["traffic_source"] = ncu_traffic(w.name, rl["kernel"], float(units))
    if with_e2e:
        e2e_value = job_rate([r.rows * r.e2e_steps] * world, col["e2e_ms"])
        sec["e2e"] = {
            "value": round(e2e_value, 2), "unit": sec["unit"],
            "h2d_bytes_per_step": int(col["h2d_bytes"][0]),
            "d2h_bytes_per_step": int(col["d2h_bytes"][0]), "steps": r.e2e_steps,
            "per_rank_ms_per_step": [round(float(x) / r.e2e_steps, 4) for x in col["e2e_ms"]],
            "copy_streams": int(col["copy_streams"][0]),
            # one step's copies alone, all ranks copying at once
            "host_copy": {
                "h2d_gbs": [round(float(x), 1) for x in col["h2d_gbs"]],
                "d2h_gbs": [round(float(x), 1) for x in col["d2h_gbs"]],
                "h2d_ms_per_step": [round(float(x), 3) for x in col["h2d_ms"]],
                "d2h_ms_per_step": [round(float(x), 3) for x in col["d2h_ms"]],
            },
        }
    if results is not None:
        sec["results"] = results
    return sec


# ---------------------------------------------------------------------------
# small operators (append, block copy, fused RoPE + append, accept, prepare)
# ---------------------------------------------------------------------------

def _graph_time_us(fn, iters, warmup):
    """Mean device time per call: `iters` calls captured in one CUDA graph and
    replayed between CUDA events (host-side argument handling stays out)."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / iters


def ops_suite(iters=50, warmup=5, only=None):
    """Timings of the path's smaller operators on one GPU; each entry gives
    the mean time per call and, where the operator moves data, its
    algorithmic bytes (every byte it must read or write once) against the HBM
    copy peak. Cases larger than L2 show the kernel's bandwidth; the
    decode-step cases are bound by launch latency. `only` runs one case."""
    import torch

    import fekv
    from fekv import workloads

    peak, peak_kind = measured_peak_gbs()
    dev = torch.device("cuda")
    bf = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    out = {"peak_gbs": peak, "peak_kind": peak_kind, "iters": iters,
           "timing": "CUDA-graph replay of `iters` calls between CUDA events"}

    def entry(us, nbytes, **kw):
        e = {"us": round(us, 2)}
        if nbytes:
            gbs = nbytes / (us * 1e-6) / 1e9
            e.update({"bytes": int(nbytes), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                      "frac_nominal": round(gbs / NOMINAL_HBM_GBS, 4)})
        e.update(kw)
        return e

    def append_case(rows, slots_total, width=1024):
        k = torch.randn(rows, width, generator=g, device=dev).to(bf)
        v = torch.randn(rows, width, generator=g, device=dev).to(bf)
        kc = torch.empty(slots_total, width, dtype=bf, device=dev)
        vc = torch.empty_like(kc)
        slots = torch.randperm(slots_total, device=dev)[:rows].to(torch.int64)
        us = _graph_time_us(lambda: fekv.store(k, v, kc, vc, slots), iters, warmup)
        return entry(us, rows * (width * 2 * 2 * 2 + 8), kernel="append_kernel", rows=rows,
                     width=width)

    def copy_case(full, sets):
        # C4's copy-on-write tails move 78 MB, less than L2: they cycle over
        # four copies of the pools so that each call finds its pages evicted
        w4 = workloads.c4(seed=0)
        src, dst, ntok = (np.asarray(x, np.int32) for x in w4.cow)
        n = 256 if full else len(src)
        s_ = torch.from_numpy(np.arange(n, dtype=np.int32) if full else src).to(dev)
        d_ = torch.from_numpy((np.arange(n, dtype=np.int32) + 512) if full else dst).to(dev)
        t_ = torch.from_numpy(np.full(n, 16, np.int32) if full else ntok).to(dev)
        pages_total = int(max(int(d_.max()), int(s_.max()))) + 2
        pools = []
        for _ in range(sets):
            kp = [torch.zeros(pages_total * 16, w4.width, dtype=bf, device=dev) for _ in range(48)]
            pools.append((kp, [torch.zeros_like(p) for p in kp]))
        turn = [0]

        def call():
            kp, vp = pools[turn[0] % sets]
            turn[0] += 1
            fekv.copy_blocks(kp, vp, s_, d_, t_, 16, w4.width, pages_total)

        us = _graph_time_us(call, iters, warmup)
        tok = int(t_.sum())
        return entry(us, 48 * 2 * tok * w4.width * 2 * 2, kernel="copy_blocks_kernel", copies=n,
                     tokens=tok, pool_sets=sets)

    def gather_case():
        # a C2 layer's K gathered densely (the ATen path's index_select
        # without its max_context padding)
        w2 = workloads.c2(seed=0)
        md = w2.metadata(0)
        lengths = md.lengths(w2.page)
        pool = torch.randn(w2.cache_slots, w2.width, generator=g, device=dev).to(bf)
        dense = torch.empty(int(lengths.sum()), w2.width, dtype=bf, device=dev)
        kv_d, pages_d, last_d = (torch.from_numpy(a).to(dev) for a in (md.kv, md.pages, md.last))
        roff = torch.from_numpy(np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
                                ).to(dev)
        us = _graph_time_us(lambda: fekv.gather(pool, dense, kv_d, pages_d, last_d, roff,
                                                md.batch, int(lengths.max()), w2.page, w2.width),
                            iters, warmup)
        return entry(us, int(lengths.sum()) * w2.width * 2 * 2, kernel="gather_kernel",
                     tokens=int(lengths.sum()))

    def clear_case():
        pages = torch.arange(256, dtype=torch.int32, device=dev)
        pools = [torch.empty(300 * 16, 1024, dtype=bf, device=dev) for _ in range(96)]
        us = _graph_time_us(lambda: fekv.clear_pages(pools, pages, 16, 1024, 300), iters, warmup)
        return entry(us, 96 * 256 * 16 * 1024 * 2, kernel="clear_pages_kernel", pools=96,
                     pages=256)

    def rope_case(rows, hq=32, hkv=8, dim=128, max_pos=8192):
        # fused RoPE + append (Qwen3-8B shape), and the reference's order:
        # rope in place, then the append
        inv = 1.0 / (1e6 ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
        ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
        cache = torch.from_numpy(np.concatenate([np.cos(ang), np.sin(ang)], 1).astype(np.float32)
                                 ).to(dev)
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
        nbytes = rows * (2 * hq * dim * 2 + 2 * hkv * dim * 2 + 2 * hkv * dim * 2 + dim * 4 + 16)
        us = _graph_time_us(lambda: fekv.rope_append(q, k, v, kc, vc, slots, pos, cache), iters,
                            warmup)
        us2 = _graph_time_us(lambda: (fekv.rope(q, k, pos, cache),
                                      fekv.store(k, v, kc, vc, slots)), iters, warmup)
        return entry(us, nbytes, kernel="rope_vec_kernel (fused append)", rows=rows,
                     rope_then_append_us=round(us2, 2))

    def accept_case():
        draft = torch.randint(0, 1000, (64, 15), generator=g, device=dev)
        verify = torch.randint(0, 1000, (64, 16), generator=g, device=dev)
        acc = torch.zeros(64, 17, dtype=torch.int64, device=dev)
        return entry(_graph_time_us(lambda: fekv.accept(draft, verify, acc), iters, warmup), 0,
                     kernel="accept_kernel")

    def prepare_host_case():
        w2 = workloads.c2(seed=0, steps=2)
        md = w2.metadata(0)
        plan = fekv.AttentionPlan(w2.hq, w2.hkv, 128, 16, w2.batch, w2.max_pages(2), True,
                                  w2.num_blocks)
        stream = torch.cuda.current_stream()
        torch.cuda.synchronize()
        t = time.perf_counter()
        for _ in range(iters):
            plan.prepare(md.qo, md.kv, md.pages, md.last, md.batch, md.rows, False, stream)
        torch.cuda.synchronize()
        us = (time.perf_counter() - t) * 1e6 / iters
        plan.close()
        return entry(us, 0, note="host planner + one H2D copy, wall clock")

    def prepare_device_case():
        w2 = workloads.c2(seed=0, steps=2)
        md = w2.metadata(0)
        stride = int(np.diff(md.kv).max()) + 1
        bt = np.zeros((w2.batch, stride), np.int32)
        for b, tb in enumerate(w2.block_tables):
            bt[b, :len(tb)] = tb
        bt_d = torch.from_numpy(bt).to(dev)
        starts = torch.from_numpy(w2.cached.astype(np.int32)).to(dev)
        sl = torch.empty(w2.batch, dtype=torch.int64, device=dev)
        ps = torch.empty_like(sl)
        plan = fekv.AttentionPlan(w2.hq, w2.hkv, 128, 16, w2.batch, w2.max_pages(2), True,
                                  w2.num_blocks)
        us = _graph_time_us(lambda: plan.step_prepare_device(bt_d, starts, 1, sl, ps), iters,
                            warmup)
        plan.close()
        return entry(us, 0, kernel="plan_device_kernel",
                     note="slot mapping + work lists of a C2 step, one kernel")

    cases = {
        "append_c2_step": lambda: append_case(64, 1 << 20),
        "append_c3_step": lambda: append_case(2108, 1 << 20),
        "append_64k_rows": lambda: append_case(65536, 1 << 18),
        "copy_blocks_c4_cow_48_layers": lambda: copy_case(False, 4),
        "copy_blocks_256_pages_48_layers": lambda: copy_case(True, 1),
        "gather_c2_layer": gather_case,
        "clear_pages_256_pages_96_pools": clear_case,
        "rope_append_c2_step": lambda: rope_case(64),
        "rope_append_c3_step": lambda: rope_case(2108),
        "rope_append_64k_rows": lambda: rope_case(65536),
        "accept_batch64_k15": accept_case,
        "prepare_host_c2_step": prepare_host_case,
        "prepare_device_c2_step": prepare_device_case,
    }
    if only is not None and only not in cases:
        raise ValueError(f"unknown operator case {only}; one of {sorted(cases)}")
    for name, fn in cases.items():
        if only is None or name == only:
            out[name] = fn()
            torch.cuda.empty_cache()
    if fekv.device_errors() != 0:
        raise RuntimeError("device error bits set during the operator timings")
    return out


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own ATen path (oracle/_ref), all host threads
# ---------------------------------------------------------------------------

def _ref_layer_step(ref, w, md, pools, inputs):
    kp, vp = pools
    q, kn, vn = inputs
    ref.store(kn, vn, kp, vp, md.slots)
    ref.prepare(md.qo, md.kv, md.pages, md.last)
    return ref.attention(q, kp, vp, w.causal)


def cpu_reference_setup(w):
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
    # max_pages sized to this step's longest context (the ATen path's gather
    # is padded to max_pages)
    ref = oracle.RefAten(w.hq, w.hkv, w.dim, w.page, w.batch, w.max_pages(1), w.bf16,
                         w.num_blocks)
    return ref, (kp, vp), (q, kn, vn), oracle.ref_get_threads()


def time_reference_layer_steps(w, count=None, seconds=None, warmup=1):
    """Per-layer-step wall times of the reference library on this workload's
    first step (store + prepare_plan + attention of every sequence):
    `count` steps, or as many as fit in `seconds`. Returns (times, threads)."""
    ref, pools, inputs, threads = cpu_reference_setup(w)
    md = w.metadata(0)
    for _ in range(warmup):
        _ref_layer_step(ref, w, md, pools, inputs)
    times = []
    t_end = time.time() + (seconds or 0)
    while (count is not None and len(times) < count) or \
            (count is None and (time.time() < t_end or len(times) < 3)):
        t = time.perf_counter()
        _ref_layer_step(ref, w, md, pools, inputs)
        times.append(time.perf_counter() - t)
    ref.close()
    return times, threads


def cpu_baseline(w, args):
    """The bench workload's first layer-step through the reference library,
    repeated for ~args.cpu_seconds, median time scaled to the layer count."""
    import oracle

    if not oracle.ref_available():
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": "oracle/_ref not built"}
    times, threads = time_reference_layer_steps(w, seconds=args.cpu_seconds)
    layer_s = statistics.median(times)
    rows = w.metadata(0).rows
    return {"value": round(rows / (layer_s * w.layers), 3),
            "unit": "tokens/s" if rows == w.batch else "rows/s",
            "cores": threads, "kind": "reference",
            "sample": f"{len(times)} layer-steps of {w.name} ({w.batch} seqs, {rows} rows: store + "
                      f"prepare_plan + attention), median {layer_s*1e3:.1f} ms/layer, scaled to "
                      f"{w.layers} layers",
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


# Layers timed back to back by both arms (`layer_calls` in this repository's
# line, `reference_gpu` in the reference arm's): name, workload, pool copies.
LAYER_CALLS = (("c2_decode_layer", "c2", 8), ("c3_mixed_layer", "c3", 8),
               ("c4_verify_layer", "c4", 8), ("c5_decode_layer", "c5", 3))


def time_layer_calls(args, world, make_impl):
    """Times one implementation's attention call on one layer of each of
    LAYER_CALLS (shard 0): the call back to back in one stream, each launch
    reading the next of several layer pools (each larger than L2, so no
    launch finds its pages there), CUDA events around the timed launches.
    `make_impl(w, md, total_steps)` returns (attention(q, k, v, o), close)."""
    import torch

    peak, peak_kind = measured_peak_gbs()
    tpeak, tkind = measured_peak_tflops()
    out = {}
    total_steps = args.warmup + args.steps + args.e2e_steps + 1
    for name, config, npools in LAYER_CALLS:
        w = make_workload(config, 0, world, total_steps)
        md = w.metadata(args.warmup if is_decode(config) else 0)
        g = torch.Generator(device="cuda")
        g.manual_seed(11)
        pools = []
        for _ in range(npools):
            kc = torch.empty(w.cache_slots, w.width, dtype=torch.bfloat16, device="cuda")
            vc = torch.empty_like(kc)
            kc.normal_(0.0, w.scale, generator=g)
            vc.normal_(0.0, w.scale, generator=g)
            pools.append((kc, vc))
        q = (torch.randn(md.rows, w.hq, w.dim, generator=g, device="cuda") * w.scale).to(
            torch.bfloat16)
        o = torch.empty_like(q)
        attention, close = make_impl(w, md, total_steps)
        for i in range(max(args.warmup, 3)):
            attention(q, *pools[i % npools], o)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        n = max(args.steps, 8)
        e0.record()
        for i in range(n):
            attention(q, *pools[i % npools], o)
        e1.record()
        torch.cuda.synchronize()
        close()
        ms = e0.elapsed_time(e1) / n
        keys = int(md.lengths(w.page).sum())
        nbytes = keys * 2 * w.width * 2 + 2 * md.rows * w.hq * w.dim * 2
        flops = attention_flops(w, md)
        ent = {"avg_launch_ms": round(ms, 5), "launches": n, "pools": npools,
               "algorithmic_bytes_per_launch": float(nbytes),
               "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
               "frac_of_hbm_peak": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4),
               "algorithmic_flops_per_launch": flops,
               "tflops": round(flops / (ms * 1e-3) / 1e12, 2),
               "frac_of_tensor_peak": round(flops / (ms * 1e-3) / 1e12 / tpeak, 4)}
        out[name] = ent
        del pools, q, o
        torch.cuda.empty_cache()
    out["peaks"] = {"hbm_gbs": peak, "hbm_kind": peak_kind, "bf16_tflops": tpeak,
                    "bf16_kind": tkind}
    return out


def layer_calls(args, world):
    """This repository's attention call (plan prepared on the host, not in
    graph mode) timed like the reference arm's `reference_gpu`."""
    import torch

    import fekv

    stream = torch.cuda.current_stream().cuda_stream

    def make_impl(w, md, total_steps):
        plan = fekv.AttentionPlan(w.hq, w.hkv, w.dim, w.page, w.batch, w.max_pages(total_steps),
                                  w.bf16, w.num_blocks)
        plan.prepare(md.qo, md.kv, md.pages, md.last, md.batch, md.rows, False, stream)
        return (lambda q, k, v, o: plan.attention(q, k, v, o, w.causal, stream)), plan.close

    out = {"method": "the attention call back to back in one stream, host-prepared plan; "
                     "the reference arm's reference_gpu times the reference's FlashInfer path "
                     "on the same inputs the same way"}
    out.update(time_layer_calls(args, world, make_impl))
    return out


def reference_gpu(args, world):
    """The reference's own GPU attention (src/flashinfer_attention.cu: FlashInfer's
    FA2 paged kernel, split-KV disabled, built for sm_100a from the reference
    source by oracle/build_oracle.py) timed on one GPU, on the same layer
    inputs and in the same way as this repository's `layer_calls`: a C2
    decode layer (shard 0, the headline), a C3 mixed layer (prefill chunks and
    decode rows, causal), a C4 verify layer and a C5 long-context decode
    layer."""
    import torch

    import oracle

    if not torch.cuda.is_available():
        return {"unavailable": "no GPU"}
    if not oracle.ref_flashinfer_available():
        return {"unavailable": "oracle/_ref/libfe_ref_flashinfer.so not built"}
    stream = torch.cuda.current_stream().cuda_stream

    def make_impl(w, md, total_steps):
        fi = oracle.RefFlashInfer(w.hq, w.hkv, w.dim, w.page, w.batch, w.max_pages(total_steps),
                                  True, w.num_blocks)
        fi.prepare(md.qo, md.kv, md.pages, md.last, stream)
        return (lambda q, k, v, o: fi.attention(q, k, v, o, w.causal, stream)), fi.close

    out = {"kernel": "FlashInfer BatchPrefillWithPagedKVCache (FA2, split-KV off), "
                     "src/flashinfer_attention.cu built for sm_100a",
           "flashinfer_headers": "flashinfer wheel 0.6.11.post2 (the reference pins 0.6.14)"}
    out.update(time_layer_calls(args, world, make_impl))
    return out


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU/ATen implementation of the path
    (FlashEngine.cpp src/portable_gpu_ops.cpp compiled for the CPU), all host
    threads, on the same workload as this repository's headline (shard 0).
    Each timed step is one layer-step (store + prepare_plan + attention of
    all sequences); `ms_per_step` is that measured time, `value` converts it
    to decode tokens/s of the whole layer stack. Rank 0 only."""
    if rank != 0:
        return None
    import oracle

    total_steps = args.warmup + args.steps + args.e2e_steps + 1
    w = make_workload(args.config, 0, world, total_steps)
    if not oracle.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libfe_ref_aten.so not built"}
    times, threads = time_reference_layer_steps(w, count=args.steps, warmup=args.warmup)
    layer_s = statistics.median(times)
    rows = w.metadata(0).rows
    value = rows / (layer_s * w.layers)
    unit = "tokens/s" if rows == w.batch else "rows/s"
    sample = (f"{args.steps} layer-steps of {w.name} shard 0 ({w.batch} seqs, {rows} rows: "
              f"store + prepare_plan + attention), median {layer_s * 1e3:.1f} ms, "
              f"scaled to {w.layers} layers")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(layer_s * 1e3, 3),
        "step": "one layer-step (the timed unit)",
        "ms_per_model_step_extrapolated": round(layer_s * 1e3 * w.layers, 3),
        "timed_region_s": round(float(sum(times)), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if w.bf16 else "f16",
        "data": "synthetic (seeded N(0,1) x scale K/V/q; random non-contiguous pages)",
        "config": config_dict(w, world, physical_pools(w, args.pool_gb)),
        "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": threads,
                         "kind": "reference", "sample": sample, "cpu_model": _cpu_model()},
        "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    # the reference's own GPU attention on the same layer inputs (one GPU)
    if not args.no_reference_gpu:
        try:
            line["reference_gpu"] = reference_gpu(args, world)
        except Exception as e:  # reported, not fatal: the CPU arm above stands
            line["reference_gpu"] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    return line


# ---------------------------------------------------------------------------
# this repository's arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, local):
    import fekv

    fekv.load()
    head, table, runner = measure(args.config, args, rank, world, local, args.steps)
    w = runner.w
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if w.bf16 else "f16",
            "data": "synthetic (seeded N(0,1) x scale K/V/q; random non-contiguous pages)",
        }
        line.update({k: v for k, v in head.items() if k not in ("value", "unit", "ms_per_step",
                                                               "steps")})
        if runner.decode:
            line["decode_attn_tbs"] = round(float(table[:, STAT_KEYS.index("gbs")].sum()) / 1e3, 4)
        else:
            line["metric"] = f"{w.name} paged attention TFLOP/s (tensor pipe) and query rows/s"
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w, args)
    subs = [s for s in args.sub.split(",") if s and s != "none"] if args.config == "c2" else []
    for sub in subs:
        if sub == "c5":
            sec, _, _ = measure("c5", args, rank, world, local, C5_STEPS)
        elif sub in ("c3", "c4", "q35", "draft") and world == 1:
            sec, _, _ = measure(sub, args, rank, world, local, args.steps,
                                verify=sub == "q35")
        elif sub == "ops" and world == 1:
            sec = ops_suite(args.ops_iters)
        elif sub == "calls" and world == 1:
            sec = layer_calls(args, world)
        else:
            continue
        if rank == 0:
            line[sub] = sec
    return line


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c2", "c3", "c4", "c5", "q35", "draft", "ops"],
                    default="c2",
                    help="headline workload; `ops` prints only the small-operator timings "
                         "(profiling one operator: --ops-case)")
    ap.add_argument("--ops-case", default=None, help="with --config ops: one operator case")
    ap.add_argument("--ops-iters", type=int, default=50)
    ap.add_argument("--sub", default="c5,c3,c4,q35,draft,ops,calls",
                    help="workloads measured beside the c2 headline (comma list, or none)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--pool-gb", type=float, default=150.0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="reference arm: skip timing the reference's FlashInfer GPU path")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count of --config (profiling a small case only)")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.config == "ops":
        import torch

        import fekv

        fekv.load()
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        line = {"ops": ops_suite(args.ops_iters, min(5, args.ops_iters), args.ops_case)}
    elif args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        rank, world, local = dist_setup()
        line = run_ours(args, rank, world, local)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
