"""bench.py's small-operator timings (append, block copy, gather, page clear,
fused RoPE + append, accept, host and device step preparation) run end to end
on the GPU:
every entry has a positive time and no device error is raised (a short run:
two timed calls per case)."""
import pytest

pytestmark = pytest.mark.gpu


def test_ops_suite_runs():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import bench
    out = bench.ops_suite(iters=2, warmup=1)
    cases = {k: v for k, v in out.items() if isinstance(v, dict)}
    assert {"append_c2_step", "append_c3_step", "append_64k_rows",
            "copy_blocks_c4_cow_48_layers", "copy_blocks_256_pages_48_layers", "gather_c2_layer",
            "clear_pages_256_pages_96_pools", "rope_append_c2_step", "rope_append_c3_step",
            "rope_append_64k_rows", "accept_batch64_k15", "prepare_host_c2_step",
            "prepare_device_c2_step"} == set(cases)
    assert all(v["us"] > 0 for v in cases.values())
