"""RoPE, fused RoPE + append and greedy accept on the GPU, bit-exact against
both the C restatement (oracle/fe_oracle.c) and the reference's own CUDA
kernels compiled from its source (oracle/_ref/libfe_ref_cuda.so:
src/cuda_kernels.cu rope_kernel, store_kernel, accept_kernel) on the same
device inputs."""
import ctypes

import numpy as np
import pytest

import oracle
from fe_testutil import to_device, to_host_bits

pytestmark = pytest.mark.gpu

DIM = 128


def rope_cache(max_pos, dim=DIM, theta=1.0e6):
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _bits(rng, shape, dtype, scale=2.0):
    return oracle.from_float(rng.standard_normal(shape).astype(np.float32) * scale, dtype)


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _errors():
    import fekv
    return fekv.device_errors()


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("rows,hq,hkv", [(1, 32, 8), (64, 32, 8), (37, 8, 2), (200, 64, 8),
                                         (5, 0, 4)])
def test_rope_bit_exact(dtype, rows, hq, hkv):
    import fekv
    import torch
    rng = np.random.default_rng(rows * 7 + hq + dtype)
    max_pos = 8192
    cache = rope_cache(max_pos)
    q = _bits(rng, (rows, hq, DIM), dtype)
    k = _bits(rng, (rows, hkv, DIM), dtype)
    pos = rng.integers(0, max_pos, rows).astype(np.int64)
    qd, kd = to_device(q, dtype == 1), to_device(k, dtype == 1)
    posd, cd = _dev(pos), _dev(cache)
    fekv.rope(qd if hq else None, kd, posd, cd)
    qo, ko = oracle.rope(q, k, pos, cache, dtype)
    np.testing.assert_array_equal(to_host_bits(qd), qo)
    np.testing.assert_array_equal(to_host_bits(kd), ko)
    # the reference kernel on the same inputs
    qr, kr = to_device(q, dtype == 1), to_device(k, dtype == 1)
    rc = oracle.ref_cuda().ref_cuda_rope(qr.data_ptr() if hq else None, kr.data_ptr(),
                                         posd.data_ptr(), cd.data_ptr(), rows, hq, hkv, DIM,
                                         int(dtype == 1), _stream(), max_pos)
    assert rc == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_host_bits(qd), to_host_bits(qr))
    np.testing.assert_array_equal(to_host_bits(kd), to_host_bits(kr))
    assert _errors() == 0


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("rows,hq,hkv,in_place", [(64, 32, 8, False), (300, 8, 2, True),
                                                  (16, 32, 4, False)])
def test_rope_append_equals_reference_rope_then_store(dtype, rows, hq, hkv, in_place):
    import fekv
    import torch
    rng = np.random.default_rng(11 * rows + dtype)
    max_pos, page, blocks = 4096, 16, 64
    cache_slots = (blocks + 1) * page
    width = hkv * DIM
    cache = rope_cache(max_pos)
    q = _bits(rng, (rows, hq, DIM), dtype)
    k = _bits(rng, (rows, hkv, DIM), dtype)
    v = _bits(rng, (rows, hkv, DIM), dtype)
    pool_k = _bits(rng, (cache_slots, width), dtype)
    pool_v = _bits(rng, (cache_slots, width), dtype)
    slots = rng.permutation(cache_slots)[:rows].astype(np.int64)
    slots[::5] = -1  # graph padding rows
    pos = rng.integers(0, max_pos, rows).astype(np.int64)
    posd, cd, sd = _dev(pos), _dev(cache), _dev(slots)
    bf = dtype == 1
    # ours: one fused launch
    qd, kd, vd = to_device(q, bf), to_device(k, bf), to_device(v, bf)
    kcd, vcd = to_device(pool_k, bf), to_device(pool_v, bf)
    k_out = kd if in_place else torch.empty_like(kd)
    fekv.rope_append(qd, kd, vd, kcd, vcd, sd, posd, cd, k_out=k_out)
    # reference: rope, then store
    qr, kr, vr = to_device(q, bf), to_device(k, bf), to_device(v, bf)
    kcr, vcr = to_device(pool_k, bf), to_device(pool_v, bf)
    lib = oracle.ref_cuda()
    assert lib.ref_cuda_rope(qr.data_ptr(), kr.data_ptr(), posd.data_ptr(), cd.data_ptr(), rows,
                             hq, hkv, DIM, int(bf), _stream(), max_pos) == 0
    assert lib.ref_cuda_store(kr.data_ptr(), vr.data_ptr(), kcr.data_ptr(), vcr.data_ptr(),
                              sd.data_ptr(), rows, width, int(bf), _stream(), cache_slots) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_host_bits(qd), to_host_bits(qr))
    np.testing.assert_array_equal(to_host_bits(k_out), to_host_bits(kr))
    np.testing.assert_array_equal(to_host_bits(kcd), to_host_bits(kcr))
    np.testing.assert_array_equal(to_host_bits(vcd), to_host_bits(vcr))
    if not in_place:
        np.testing.assert_array_equal(to_host_bits(kd), k)  # k itself is read only
    # and the oracle: rope then append (skip semantics)
    qo, ko = oracle.rope(q, k, pos, cache, dtype)
    pk, pv = pool_k.copy(), pool_v.copy()
    oracle.append(ko.reshape(rows, width), v.reshape(rows, width), pk, pv, slots, cache_slots)
    np.testing.assert_array_equal(to_host_bits(kcd), pk)
    np.testing.assert_array_equal(to_host_bits(vcd), pv)
    assert _errors() == 0


def _shifted(a, bf, shift):
    """A device copy of bit array `a` that starts `shift` elements into its
    allocation (shift 2: 4-byte but not 16-byte aligned)."""
    import torch
    flat = to_device(np.concatenate([np.zeros(shift, np.uint16), a.reshape(-1)]), bf)
    return flat[shift:].view(*a.shape)


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("rot,shift", [(128, 0), (48, 0), (36, 0), (128, 2), (64, 2)])
def test_rope_kernel_forms_bit_exact(dtype, rot, shift):
    """Both kernel forms -- 16-byte (rotary_dim a multiple of 16, 16-byte
    aligned buffers) and 4-byte (any other rotary_dim that is a multiple of 4,
    or buffers only 4-byte aligned) -- against the C restatement, for RoPE
    alone and fused with the append, full and partial rotary."""
    import fekv
    import torch
    rng = np.random.default_rng(rot * 3 + shift + dtype)
    rows, hq, hkv, max_pos, page, blocks = 45, 16, 4, 2048, 16, 16
    cache_slots = (blocks + 1) * page
    bf = dtype == 1
    cache = rope_cache(max_pos, dim=rot)
    q = _bits(rng, (rows, hq, DIM), dtype)
    k = _bits(rng, (rows, hkv, DIM), dtype)
    v = _bits(rng, (rows, hkv, DIM), dtype)
    pos = rng.integers(0, max_pos, rows).astype(np.int64)
    slots = rng.permutation(cache_slots)[:rows].astype(np.int64)
    slots[::7] = -1
    posd, cd, sd = _dev(pos), _dev(cache), _dev(slots)
    qo, ko = oracle.rope(q, k, pos, cache, dtype)
    # RoPE alone, in place
    qd, kd = _shifted(q, bf, shift), _shifted(k, bf, shift)
    fekv.rope(qd, kd, posd, cd)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_host_bits(qd), qo)
    np.testing.assert_array_equal(to_host_bits(kd), ko)
    # fused with the append, keys also written to k_out
    pool = _bits(rng, (cache_slots, hkv * DIM), dtype)
    qd, kd, vd = _shifted(q, bf, shift), _shifted(k, bf, shift), _shifted(v, bf, shift)
    kcd, vcd = _shifted(pool, bf, shift), _shifted(pool, bf, shift)
    k_out = _shifted(np.zeros_like(k), bf, shift)
    fekv.rope_append(qd, kd, vd, kcd, vcd, sd, posd, cd, k_out=k_out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_host_bits(qd), qo)
    np.testing.assert_array_equal(to_host_bits(k_out), ko)
    np.testing.assert_array_equal(to_host_bits(kd), k)  # k itself is read only
    pk, pv = pool.copy(), pool.copy()
    oracle.append(ko.reshape(rows, -1), v.reshape(rows, -1), pk, pv, slots, cache_slots)
    np.testing.assert_array_equal(to_host_bits(kcd), pk)
    np.testing.assert_array_equal(to_host_bits(vcd), pv)
    assert _errors() == 0


def test_rope_append_out_of_range_position_and_slot():
    """Invalid rows are skipped and flagged (the reference would read or write
    out of bounds there, so it is not run on these inputs)."""
    import fekv
    import torch
    from fekv._lib import FE_DEVERR_POS_RANGE, FE_DEVERR_SLOT_RANGE
    rng = np.random.default_rng(3)
    rows, hq, hkv, max_pos, cache_slots = 6, 8, 2, 128, 64
    cache = rope_cache(max_pos)
    q = _bits(rng, (rows, hq, DIM), 1)
    k = _bits(rng, (rows, hkv, DIM), 1)
    v = _bits(rng, (rows, hkv, DIM), 1)
    pool = np.zeros((cache_slots, hkv * DIM), np.uint16)
    pos = np.array([3, max_pos, -2, 7, 9, 11], np.int64)
    slots = np.array([1, 2, 3, cache_slots, 5, -1], np.int64)
    qd, kd, vd = to_device(q, True), to_device(k, True), to_device(v, True)
    kcd, vcd = to_device(pool, True), to_device(pool, True)
    fekv.rope_append(qd, kd, vd, kcd, vcd, _dev(slots), _dev(pos), _dev(cache))
    torch.cuda.synchronize()
    assert _errors() == FE_DEVERR_POS_RANGE | FE_DEVERR_SLOT_RANGE
    qo, ko = oracle.rope(q, k, pos, cache, 1)
    np.testing.assert_array_equal(to_host_bits(qd), qo)  # rows 1, 2 unrotated
    kc = to_host_bits(kcd)
    np.testing.assert_array_equal(kc[1], ko[0].reshape(-1))
    np.testing.assert_array_equal(kc[5], ko[4].reshape(-1))
    assert not kc[[2, 3]].any()  # rows with a bad position wrote nothing
    assert not kc[6:].any()


def test_accept_reference_matrix_with_graph_replay():
    """The reference's own test (tests/gpu_ops_tests.cpp:55-79): batch 1/2/4/8,
    k 1..15, every accepted length, guard bands around the output, direct
    launches and CUDA-graph replays."""
    import fekv
    import torch
    checks = replays = 0
    side = torch.cuda.Stream()
    for batch in (1, 2, 4, 8):
        for k in range(1, 16):
            draft = torch.zeros(batch, k, dtype=torch.int64, device="cuda")
            verify = torch.zeros(batch, k + 1, dtype=torch.int64, device="cuda")
            out = torch.full((batch * (k + 2) + 16,), -999, dtype=torch.int64, device="cuda")
            view = out[8:8 + batch * (k + 2)].view(batch, k + 2)

            def execute():
                fekv.accept(draft, verify, view)

            with torch.cuda.stream(side):
                execute()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                execute()
            for first in range(k + 1):
                d = np.zeros((batch, k), np.int64)
                v = np.zeros((batch, k + 1), np.int64)
                for b in range(batch):
                    acc = (first + b) % (k + 1)
                    d[b] = 10 + np.arange(k)
                    v[b, :k] = 10 + np.arange(k)
                    v[b, acc] = 99
                draft.copy_(torch.from_numpy(d))
                verify.copy_(torch.from_numpy(v))
                for captured in (False, True):
                    out.fill_(-999)
                    if captured:
                        g.replay()
                        replays += 1
                    else:
                        with torch.cuda.stream(side):
                            execute()
                    torch.cuda.synchronize()
                    ids = out.cpu().numpy()
                    assert (ids[:8] == -999).all() and (ids[8 + batch * (k + 2):] == -999).all()
                    for b in range(batch):
                        acc = (first + b) % (k + 1)
                        row = ids[8 + b * (k + 2):8 + (b + 1) * (k + 2)]
                        assert row[k + 1] == acc + 1 and row[acc] == 99
                        assert list(row[:acc]) == list(range(10, 10 + acc))
                        checks += 1
            del g
    assert checks == 2 * (1 + 2 + 4 + 8) * sum(k + 1 for k in range(1, 16))
    assert replays == 4 * sum(k + 1 for k in range(1, 16))


def test_accept_random_vs_reference_kernel():
    import fekv
    import torch
    rng = np.random.default_rng(9)
    lib = oracle.ref_cuda()
    for batch, k in ((1, 0), (3, 1), (64, 4), (128, 15), (300, 7)):
        draft = rng.integers(0, 4, (batch, k)).astype(np.int64)
        verify = rng.integers(0, 4, (batch, k + 1)).astype(np.int64)
        verify[::3, :k] = draft[::3]  # some rows accept everything
        dd, vd = _dev(draft), _dev(verify)
        ours = torch.full((batch, k + 2), -1, dtype=torch.int64, device="cuda")
        ref = torch.full((batch, k + 2), -1, dtype=torch.int64, device="cuda")
        fekv.accept(dd, vd, ours)
        assert lib.ref_cuda_accept(dd.data_ptr() if k else None, vd.data_ptr(), ref.data_ptr(),
                                   batch, k, _stream()) == 0
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ours.cpu().numpy(), ref.cpu().numpy())
        np.testing.assert_array_equal(ours.cpu().numpy(), oracle.accept(draft, verify))
