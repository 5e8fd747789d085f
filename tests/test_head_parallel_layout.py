"""The data movement of the head-parallel path (csrc/headpar.cu) on CPU, with
the routing functions the kernels use (hp_qkv_route in the QKV GEMM epilogue,
hp_row_owner in the attention epilogue), exported host-callable as
nemo_hp_qkv_route / nemo_hp_row_owner.

N devices hold contiguous token shards of ceil(S/N) rows (the last one fewer).
Each device's QKV epilogue stores every row chunk at global row row0 + r of the
owning device's Q / K / V buffer and, for every third position, at row pos / 3
of its compact K / V buffers. Afterwards every device must hold the whole
sequence of its own head group (q heads j*24/N.., kv heads j*8/N.., so each
GQA group of 3 stays together) and the sampled keys in order. The attention
epilogue then stores each output row into the attention buffer of the row's
owner at the group's columns: every device must end with its token shard of
the full attention output. The merge / pool gathers place shard j at row
j * ceil(S/N), which must give the rows in token order."""
import ctypes

import numpy as np
import pytest

from nemo_b200.runtime import NemoError, check, load_library

QW, KVW, QKVW = 3072, 1024, 5120


def _routes(n):
    lib = load_library()
    dev, buf, col = (np.zeros(QKVW, np.int32) for _ in range(3))
    check(lib.nemo_hp_qkv_route(n, *(a.ctypes.data_as(ctypes.c_void_p) for a in (dev, buf, col))))
    return dev, buf, col


def _owners(n, rows_per_dev, s):
    out = np.zeros(s, np.int32)
    check(load_library().nemo_hp_row_owner(n, rows_per_dev, s, out.ctypes.data_as(ctypes.c_void_p)))
    return out


@pytest.mark.parametrize("n", [2, 4, 8])
def test_qkv_route_keeps_gqa_groups_together(n):
    dev, buf, col = _routes(n)
    gq, gk = QW // n, KVW // n
    for j in range(n):
        q = np.where((dev == j) & (buf == 0))[0]
        k = np.where((dev == j) & (buf == 1))[0]
        v = np.where((dev == j) & (buf == 2))[0]
        assert np.array_equal(q, np.arange(j * gq, (j + 1) * gq))
        assert np.array_equal(k, QW + np.arange(j * gk, (j + 1) * gk))
        assert np.array_equal(v, QW + KVW + np.arange(j * gk, (j + 1) * gk))
        assert np.array_equal(col[q], np.arange(gq)) and np.array_equal(col[k], np.arange(gk))
        # q head h uses kv head h // 3: every q head of the group finds its kv head there
        assert set(q // 128 // 3) == set((k - QW) // 128)
    # whole 32-column chunks (the epilogue's store unit) never straddle devices or buffers
    for c in range(0, QKVW, 32):
        assert len(set(zip(dev[c:c + 32], buf[c:c + 32]))) == 1
        assert np.array_equal(col[c:c + 32], col[c] + np.arange(32))


@pytest.mark.parametrize("n,s", [(2, 37), (2, 5000), (4, 513), (4, 2049), (8, 64), (8, 3203)])
def test_head_parallel_scatter_round_trip(n, s):
    dev, buf, col = _routes(n)
    sh = (s + n - 1) // n
    shard = lambda i: max(0, min(sh, s - i * sh))
    gq, gk = QW // n, KVW // n
    rng = np.random.default_rng(s + n)
    full_qkv = rng.integers(0, 1 << 15, (s, QKVW)).astype(np.int32)
    full_att = rng.integers(0, 1 << 15, (s, QW)).astype(np.int32)
    sample = s > 2048
    # per-device buffers the epilogues store into
    q = [np.full((s, gq), -1, np.int32) for _ in range(n)]
    k = [np.full((s, gk), -1, np.int32) for _ in range(n)]
    v = [np.full((s, gk), -1, np.int32) for _ in range(n)]
    kc = [np.full(((s + 2) // 3, gk), -1, np.int32) for _ in range(n)]
    vc = [np.full(((s + 2) // 3, gk), -1, np.int32) for _ in range(n)]
    bufs = (q, k, v)
    for r in range(n):
        row0 = r * sh
        for t in range(shard(r)):
            pos = row0 + t
            for c in range(0, QKVW, 32):
                j, b, dc = dev[c], buf[c], col[c]
                bufs[b][j][pos, dc:dc + 32] = full_qkv[pos, c:c + 32]
                if sample and b > 0 and pos % 3 == 0:
                    (kc, vc)[b - 1][j][pos // 3, dc:dc + 32] = full_qkv[pos, c:c + 32]
    for j in range(n):
        assert np.array_equal(q[j], full_qkv[:, j * gq:(j + 1) * gq])
        assert np.array_equal(k[j], full_qkv[:, QW + j * gk:QW + (j + 1) * gk])
        assert np.array_equal(v[j], full_qkv[:, QW + KVW + j * gk:QW + KVW + (j + 1) * gk])
        if sample:  # the compact rows the single-device gather would make (every third key)
            assert np.array_equal(kc[j], k[j][::3]) and np.array_equal(vc[j], v[j][::3])

    # attention epilogue: device j's head group, every row, to the row's owner
    owner = _owners(n, sh, s)
    attn = [np.full((sh, QW), -1, np.int32) for _ in range(n)]
    for j in range(n):
        for pos in range(s):
            o = owner[pos]
            attn[o][pos - o * sh, j * gq:(j + 1) * gq] = full_att[pos, j * gq:(j + 1) * gq]
    for r in range(n):
        assert np.array_equal(attn[r][:shard(r)], full_att[r * sh:r * sh + shard(r)])
        assert (attn[r][shard(r):] == -1).all()

    # merge / pool gathers: shard j's rows at row j * sh give token order
    gathered = np.full(n * sh, -1)
    for j in range(n):
        gathered[j * sh:j * sh + shard(j)] = np.arange(j * sh, j * sh + shard(j))
    assert np.array_equal(gathered[:s], np.arange(s))


def test_routing_rejects_bad_device_counts():
    lib = load_library()
    a = np.zeros(QKVW, np.int32)
    p = a.ctypes.data_as(ctypes.c_void_p)
    for n in (0, 1, 3, 16):
        with pytest.raises(NemoError):
            check(lib.nemo_hp_qkv_route(n, p, p, p))
        with pytest.raises(NemoError):
            check(lib.nemo_hp_row_owner(n, 4, 8, p))
    with pytest.raises(NemoError):
        check(lib.nemo_hp_row_owner(2, 0, 8, p))
