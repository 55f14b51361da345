"""The greedy-token check itself, on the CPU with the torch reference
operators: it is deterministic, and it notices a planted off-by-one in the
attention (every row missing its last visible key). Test infrastructure only;
the GPU test (test_gpu_greedy_model.py) compares this repository's kernels."""
import numpy as np


def _gen(backend_kw, seed=3, steps=8):
    from synth_model import PagedKV, SynthQwen3, TorchBackend, generate

    model = SynthQwen3(seed=seed, device="cpu")
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, 512, n) for n in (21, 16, 1, 40)]
    kv = PagedKV(model, 64, seed=seed + 1)
    toks, gap, _ = generate(model, kv, TorchBackend(model, kv, **backend_kw), prompts,
                            steps=steps, verify_at=(3,), seed=seed)
    return toks, gap


def test_greedy_check_is_deterministic():
    a, gap = _gen({})
    b, _ = _gen({})
    assert a == b
    assert gap > 0.0  # fp32 logits: no exact ties


def test_greedy_check_detects_a_planted_attention_error():
    good, _ = _gen({})
    bad, _ = _gen({"drop_last_key": True})
    assert any(g != b for g, b in zip(good, bad))
