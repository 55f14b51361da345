"""bench.py's roofline helpers, without a GPU: the DRAM traffic taken from a
committed ncu capture (scaled only where traffic grows with the bytes read)
and the choice of bound for multi-row attention steps."""
import numpy as np

import bench


def test_traffic_from_capture_scales_only_for_streaming_kernels():
    dram, units, _, _ = bench.NCU_TRAFFIC[("C2", "paged_decode_kernel")]
    t, src = bench.ncu_traffic("C2", "paged_decode_kernel", units * 1.01)
    assert t == round(dram * 1.01) and "scaled" in src
    t, src = bench.ncu_traffic("C4", "paged_prefill_tc_kernel",
                               bench.NCU_TRAFFIC[("C4", "paged_prefill_tc_kernel")][1])
    assert t == bench.NCU_TRAFFIC[("C4", "paged_prefill_tc_kernel")][0] and "scaled" not in src
    # a launch that is not the captured one reports no traffic
    assert bench.ncu_traffic("C4", "paged_prefill_tc_kernel", 1.0) == (None, None)
    assert bench.ncu_traffic("C3", "paged_prefill_tc_kernel", 1.0) == (None, None)
    assert bench.ncu_traffic("C2", "paged_decode_kernel", units * 2) == (None, None)


def test_row_step_bound():
    own = [np.arange(0, 10), np.arange(10, 20)]
    shared = [np.arange(0, 10), np.concatenate([np.arange(0, 5), np.arange(20, 25)])]
    tpeak, peak = 1382.0, 6552.0  # ridge ~211 FLOP/B
    assert bench.row_step_bound(own, 128.0e6, 1.0e6, tpeak, peak) == "hbm"
    assert bench.row_step_bound(own, 400.0e6, 1.0e6, tpeak, peak) == "tensor"
    # a shared prefix is served from L2: tensor-bound at any intensity
    assert bench.row_step_bound(shared, 128.0e6, 1.0e6, tpeak, peak) == "tensor"
