"""The allocation-free attention entry point (nemo_op_attention_tc_noalloc).

It exists for hosts that cannot allocate device memory where attention runs
(device memory owned by another allocator or reserved up front, or a server
that cannot afford cudaFree's device-wide synchronisation). Its scratch is a
fixed device array inside the library, so these checks call it through the C
ABI twice in a row and compare each result with the regular entry point
(nemo_op_attention_tc, which allocates its scratch per call) on the same
inputs, with the attention tolerance of the other GPU tests. The file is named
to be collected last: a run that stops at the first failure has run every
other test before reaching it.
"""
import numpy as np
import pytest

from gpu_util import dev, empty, f16_bits, f16_of_bits, host, ptr, rel_err
from nemo_b200.runtime import NemoError, check, load_library

pytestmark = pytest.mark.gpu

ATTN_TOL = 2e-3  # same bound as tests/test_gpu_ops.py::test_attention


def _inputs(rng, lengths):
    import torch
    T = sum(lengths)
    qkv = f16_bits(rng.normal(0, 1, (T, 5120)))
    q = f16_bits(rng.normal(0, 1.5, (T, 3072)))
    k = f16_bits(rng.normal(0, 1.5, (T, 1024)))
    lens = np.asarray(lengths, np.uint32)
    d_len = dev(lens)
    d_meta = torch.zeros(load_library().nemo_op_meta_bytes(), dtype=torch.uint8, device="cuda")
    check(load_library().nemo_op_meta(ptr(d_len), lens.size, max(lengths), ptr(d_meta)))
    return T, dev(q.view(np.float16)), dev(k.view(np.float16)), dev(qkv.view(np.float16)), d_len, d_meta


@pytest.mark.parametrize("lengths", [[2100, 300], [40, 3, 17]], ids=["stride3", "ragged"])
def test_noalloc_matches_allocating_entry_point_twice(lengths):
    import torch
    L = load_library()
    rng = np.random.default_rng(2024)
    T, d_q, d_k, d_qkv, d_len, d_meta = _inputs(rng, lengths)
    seq = max(lengths)
    ref = empty((T, 3072), torch.float16)
    check(L.nemo_op_attention_tc(ptr(d_q), ptr(d_k), ptr(d_qkv), ptr(d_meta), 0, len(lengths), seq, T, ptr(ref)))
    want = f16_of_bits(host(ref).view(np.uint16))
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        out = empty((T, 3072), torch.float16)
        check(L.nemo_op_attention_tc_noalloc(ptr(d_q), ptr(d_k), ptr(d_qkv), ptr(d_meta), 0, len(lengths), seq, T,
                                             ptr(out)))
        got = f16_of_bits(host(out).view(np.uint16))
        assert rel_err(got, want) < ATTN_TOL


def test_noalloc_stale_rows_do_not_leak_into_a_later_call():
    """A first call leaves non-finite V values in the shared array beyond the
    rows a shorter second call samples; the second call's last 128-row K/V
    tile still loads those rows (with zero key weight), so they must have been
    cleared: its result still matches the allocating entry point."""
    import torch
    L = load_library()
    rng = np.random.default_rng(77)
    T1, q1, k1, qkv1, _, m1 = _inputs(rng, [2700])  # 900 sampled rows
    qkv1[:, 4096:] = float("nan")
    out1 = empty((T1, 3072), torch.float16)
    check(L.nemo_op_attention_tc_noalloc(ptr(q1), ptr(k1), ptr(qkv1), ptr(m1), 0, 1, 2700, T1, ptr(out1)))
    T2, q2, k2, qkv2, _, m2 = _inputs(rng, [2100])  # 700 sampled rows: the last tile covers rows 640..767
    ref = empty((T2, 3072), torch.float16)
    check(L.nemo_op_attention_tc(ptr(q2), ptr(k2), ptr(qkv2), ptr(m2), 0, 1, 2100, T2, ptr(ref)))
    out2 = empty((T2, 3072), torch.float16)
    check(L.nemo_op_attention_tc_noalloc(ptr(q2), ptr(k2), ptr(qkv2), ptr(m2), 0, 1, 2100, T2, ptr(out2)))
    got = f16_of_bits(host(out2).view(np.uint16))
    assert np.isfinite(got).all()
    assert rel_err(got, f16_of_bits(host(ref).view(np.uint16))) < ATTN_TOL


def test_noalloc_calls_allocate_no_device_memory():
    """The property the entry point exists for: after a first call (which looks
    up the array's address), further calls leave the device's free memory
    unchanged."""
    import torch
    L = load_library()
    rng = np.random.default_rng(5)
    lengths = [2100, 300]
    T, d_q, d_k, d_qkv, _, d_meta = _inputs(rng, lengths)
    outs = [empty((T, 3072), torch.float16) for _ in range(3)]
    check(L.nemo_op_attention_tc_noalloc(ptr(d_q), ptr(d_k), ptr(d_qkv), ptr(d_meta), 0, 2, 2100, T, ptr(outs[0])))
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for o in outs[1:]:
        check(L.nemo_op_attention_tc_noalloc(ptr(d_q), ptr(d_k), ptr(d_qkv), ptr(d_meta), 0, 2, 2100, T, ptr(o)))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.equal(outs[1], outs[2])


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    L = load_library()
    # one 6200-token request keeps ceil(6200 / 3) = 2067 sampled keys > 2048:
    # rejected on the host, from the run's metadata, before any device work.
    rows = 6200
    lens = dev(np.array([rows], np.uint32))
    meta = torch.zeros(L.nemo_op_meta_bytes(), dtype=torch.uint8, device="cuda")
    check(L.nemo_op_meta(ptr(lens), 1, rows, ptr(meta)))
    q = torch.zeros((rows, 3072), dtype=torch.float16, device="cuda")
    k = torch.zeros((rows, 1024), dtype=torch.float16, device="cuda")
    qkv = torch.zeros((rows, 5120), dtype=torch.float16, device="cuda")
    out = torch.zeros((rows, 3072), dtype=torch.float16, device="cuda")
    with pytest.raises(NemoError, match="2067 sampled key rows"):
        check(L.nemo_op_attention_tc_noalloc(ptr(q), ptr(k), ptr(qkv), ptr(meta), 0, 1, rows, rows, ptr(out)))
