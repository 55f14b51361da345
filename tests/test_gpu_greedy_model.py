"""Greedy-token identity on a seeded synthetic Qwen3-style model: the same
generation run with the reference's paged-KV operators (torch restatement of
the CUDA store and the fp32 ATen attention, src/cuda_kernels.cu:24,34 and
src/portable_gpu_ops.cpp:27-44) and with this repository's operators through
the C ABI must produce identical tokens. Covers chunked prefill, decode, a
copy-on-write fork and speculative verify rows (see tests/synth_model.py)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(seed, prompts, steps, num_blocks=160):
    import fekv
    from synth_model import FekvBackend, PagedKV, SynthQwen3, TorchBackend, generate

    model = SynthQwen3(seed=seed)
    kv_ref = PagedKV(model, num_blocks, seed=seed + 1)
    toks_ref, gap_ref, acc_ref = generate(model, kv_ref, TorchBackend(model, kv_ref), prompts,
                                          steps=steps, seed=seed)
    kv_our = PagedKV(model, num_blocks, seed=seed + 1)
    ours = FekvBackend(model, kv_our)
    try:
        toks_our, gap_our, acc_our = generate(model, kv_our, ours, prompts, steps=steps, seed=seed)
    finally:
        ours.close()
    assert fekv.device_errors() == 0
    return toks_ref, toks_our, gap_ref


@pytest.mark.parametrize("seed", [3, 11])
def test_greedy_tokens_identical(seed):
    rng = np.random.default_rng(seed)
    # edge lengths: one token, exactly one page, a page plus one, > 8 pages
    lengths = [37, 16, 1, 70, 129, 17]
    prompts = [rng.integers(0, 512, n) for n in lengths]
    toks_ref, toks_our, gap = _run(seed, prompts, steps=24)
    assert len(toks_ref) == len(lengths) + 1  # the forked sequence
    for b, (r, o) in enumerate(zip(toks_ref, toks_our)):
        assert r == o, (f"sequence {b}: tokens diverge at {next(i for i, (x, y) in enumerate(zip(r, o)) if x != y)}"
                        f" (smallest reference top-2 logit gap {gap:.3g})")
