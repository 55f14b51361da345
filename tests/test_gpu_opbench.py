"""The small-operator benchmark (fekv.opbench) runs end to end on the GPU:
every case prints a JSON line with a positive time, and no device error is
raised (a short run: two timed calls per case)."""
import json

import pytest

pytestmark = pytest.mark.gpu


def test_opbench_runs(capsys):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from fekv import opbench
    opbench.run(iters=2, warmup=1)
    lines = [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    ops = {l["op"] for l in lines}
    assert {"append", "copy_blocks", "rope_append", "rope_then_append", "accept",
            "prepare_host", "prepare_device"} <= ops
    assert all(l["us"] > 0 for l in lines)
