"""Multi-rank host logic on the CPU with two gloo ranks (no GPU): the
sequence-sharded C5 workload gives each rank its own balanced shard of the
global sequence list, the post-timing stats gather returns the same [world, k]
table on every rank, the whole-job rate is all ranks' units over the slowest
rank's time, the results check gathers one sampled sequence per rank and
flags a rank whose output is wrong, and a rank that leaves before the
collective is reported as an error on its peer within the process-group
timeout instead of hanging it."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PER_RANK = 8


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir, mode):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "flashengine.cpp_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch.distributed as dist

    from fekv import dist as fdist
    from fekv import workloads

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=15))
    if mode in ("verify", "verify_bad"):
        _verify_worker(rank, world, out_dir, plant=(mode == "verify_bad"))
        dist.destroy_process_group()
        return
    w = workloads.c5(rank=rank, world=world, steps=2, per_gpu=PER_RANK)
    if mode == "leave" and rank == 1:
        os._exit(3)  # leaves between steps, before the stats collective
    try:
        stats = fdist.gather_floats([float(w.batch), 10.0 + rank], world, device="cpu")
        ctx = fdist.gather_floats(w.cached.astype(np.float64), world, device="cpu")
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), stats=stats, ctx=ctx)
    except Exception as e:  # the peer left: report, do not hang
        with open(os.path.join(out_dir, f"r{rank}.err"), "w") as f:
            f.write(type(e).__name__ + ": " + str(e)[:200])
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


class _FakeRunner:
    """Stands in for bench.Runner's sample/checksum interface on the CPU: one
    sequence of `n` keys per rank (different lengths on the two ranks), with
    the output computed by the fp32 check itself, optionally corrupted."""

    def __init__(self, rank, plant):
        import torch

        from fekv import workloads
        self.rank = rank
        self.w = workloads.decode_workload("T", 8, 2, [40], False, 3)
        g = torch.Generator().manual_seed(rank)
        self.n = 37 + 20 * rank
        self.k = torch.randn(self.n, 2, 128, generator=g).to(torch.float16)
        self.v = torch.randn(self.n, 2, 128, generator=g).to(torch.float16)
        self.q = torch.randn(1, 8, 128, generator=g).to(torch.float16)
        import bench
        self.out = bench.dense_attention_f32(self.q, self.k, self.v, 8, 2, True).to(torch.float16)
        if plant and rank == 1:
            self.out[0, 3, 5] += 0.01

    def sample(self):
        return self.n, self.k, self.v, self.q, self.out

    def checksums(self):
        return [float(self.out.float().sum()), float(self.out.float().abs().sum())]


def _verify_worker(rank, world, out_dir, plant):
    import json

    import bench
    res = bench.verify_results(_FakeRunner(rank, plant), world)
    if rank == 0:
        with open(os.path.join(out_dir, "verify.json"), "w") as f:
            json.dump(res, f)


def _launch(tmp_path, mode, world=2, timeout=90):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:  # only the processes started here
        p.kill()
        p.join(5)
    assert not alive, "a rank hung"
    return [p.exitcode for p in procs]


def test_sharded_workload_and_job_rate(tmp_path):
    from fekv import workloads
    from fekv.dist import job_rate

    codes = _launch(tmp_path, "ok")
    assert codes == [0, 0]
    r0 = np.load(tmp_path / "r0.npz")
    r1 = np.load(tmp_path / "r1.npz")
    # every rank holds the same gathered table
    np.testing.assert_array_equal(r0["stats"], r1["stats"])
    np.testing.assert_array_equal(r0["ctx"], r1["ctx"])
    # each rank holds its own balanced shard of the global list
    from fekv.dist import balanced_shards
    glob = workloads.c5_contexts(0, PER_RANK * 8)
    shards = balanced_shards(glob, 8, PER_RANK)
    np.testing.assert_array_equal(r0["ctx"][0], glob[shards[0]])
    np.testing.assert_array_equal(r0["ctx"][1], glob[shards[1]])
    assert not set(shards[0]) & set(shards[1])
    # whole-job rate: 16 sequences over the slower rank's 11 ms
    rate = job_rate(r0["stats"][:, 0], r0["stats"][:, 1])
    assert rate == pytest.approx(2 * PER_RANK / 11e-3)


def test_rank_leaving_is_reported_not_hung(tmp_path):
    codes = _launch(tmp_path, "leave")
    assert codes[1] == 3
    assert (tmp_path / "r0.err").exists(), "the surviving rank did not see the failure"
    assert not (tmp_path / "r0.npz").exists()


def test_balanced_shards_equalise_kv_bytes():
    from fekv import workloads
    from fekv.dist import balanced_shards
    rng = np.random.default_rng(0)
    costs = rng.integers(512, 4097, size=512)
    shards = balanced_shards(costs, 8, 64)
    assert sorted(np.concatenate(shards).tolist()) == list(range(512))
    assert all(len(s) == 64 for s in shards)
    sums = np.array([costs[s].sum() for s in shards])
    assert (sums.max() - sums.min()) / sums.mean() < 0.001
    # the bench's C2 and C5 shards
    c2 = [workloads.c2_shard(r, 8).cached.sum() for r in range(8)]
    c5 = [workloads.c5(r, 8).cached.sum() for r in range(8)]
    for sums in (np.array(c2), np.array(c5)):
        assert (sums.max() - sums.min()) / sums.mean() < 0.001


def test_results_check_gathers_samples(tmp_path):
    import json
    assert _launch(tmp_path, "verify") == [0, 0]
    res = json.loads((tmp_path / "verify.json").read_text())
    assert res["ok"] and res["ranks_checked"] == 2 and len(res["checksums"]) == 2


def test_results_check_flags_a_wrong_rank(tmp_path):
    import json
    assert _launch(tmp_path, "verify_bad") == [0, 0]
    res = json.loads((tmp_path / "verify.json").read_text())
    assert not res["ok"] and res["per_rank_ok"] == [True, False]
