"""Multi-rank host logic on the CPU with two gloo ranks (no GPU): the
sequence-sharded C5 workload gives each rank a disjoint slice of the global
sequence list, the post-timing stats gather returns the same [world, k] table
on every rank, the whole-job rate is all ranks' units over the slowest rank's
time, and a rank that leaves before the collective is reported as an error on
its peer within the process-group timeout instead of hanging it."""
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
    # the shards are the first two disjoint slices of the global list
    glob = workloads.c5_contexts(0, PER_RANK * 8)
    np.testing.assert_array_equal(r0["ctx"][0], glob[:PER_RANK])
    np.testing.assert_array_equal(r0["ctx"][1], glob[PER_RANK:2 * PER_RANK])
    # whole-job rate: 16 sequences over the slower rank's 11 ms
    rate = job_rate(r0["stats"][:, 0], r0["stats"][:, 1])
    assert rate == pytest.approx(2 * PER_RANK / 11e-3)


def test_rank_leaving_is_reported_not_hung(tmp_path):
    codes = _launch(tmp_path, "leave")
    assert codes[1] == 3
    assert (tmp_path / "r0.err").exists(), "the surviving rank did not see the failure"
    assert not (tmp_path / "r0.npz").exists()
