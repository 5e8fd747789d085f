"""The exchange pattern of the head-parallel path (csrc/headpar.cu) on CPU: two
gloo ranks hold contiguous token shards of ceil(S/N) rows (the last one
fewer), pack the Q/K/V columns of each head group, swap them with point-to-point
send/recv as the grouped NCCL calls do, and must end up with the whole
sequence of their own head group, in token order. The attention output goes
back the same way, and the in-place all-gather of padded shards must give the
rows in token order. The pack uses the column map of hp_pack_kernel itself
(nemo_hp_pack_columns, host-callable), checked first against the head-group
column sets."""
import os
import socket
import subprocess
import sys
import textwrap

import pytest

from conftest import REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


WORKER = textwrap.dedent("""
    import os
    import numpy as np
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method="env://", timeout=__import__("datetime").timedelta(seconds=60))
    r, N = dist.get_rank(), dist.get_world_size()
    QW, KVW, QKVW = 3072, 1024, 5120
    gw, gq, gk = QKVW // N, QW // N, KVW // N
    S = int(os.environ["SEQ"])
    sh = (S + N - 1) // N
    shard = lambda i: max(0, min(sh, S - i * sh))
    rng = np.random.default_rng(5)
    full_qkv = rng.standard_normal((S, QKVW)).astype(np.float32)
    full_att = rng.standard_normal((S, QW)).astype(np.float32)
    T = shard(r)
    mine = full_qkv[r * sh:r * sh + T]

    def expected_cols(j):  # Q, K, V columns of head group j
        return np.concatenate([np.arange(j * gq, (j + 1) * gq), QW + np.arange(j * gk, (j + 1) * gk),
                               QW + KVW + np.arange(j * gk, (j + 1) * gk)])

    import ctypes
    import sys
    sys.path.insert(0, os.path.join(os.getcwd(), "nemotron-3-embed-webgpu_b200"))
    from nemo_b200.runtime import check, load_library
    cmap = np.zeros(QKVW, np.int32)
    check(load_library().nemo_hp_pack_columns(N, cmap.ctypes.data_as(ctypes.c_void_p)))
    for j in range(N):
        assert np.array_equal(cmap[j * gw:(j + 1) * gw], expected_cols(j)), "pack column map"
    group_cols = lambda j: cmap[j * gw:(j + 1) * gw]  # the map hp_pack_kernel applies

    # pack: block j = this shard's rows, head group j's columns
    send = [mine[:, group_cols(j)] for j in range(N)]
    recv = [np.zeros((shard(j), gw), np.float32) for j in range(N)]
    reqs = []
    for j in range(N):
        if j == r:
            recv[j][:] = send[j]
            continue
        if T:
            reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(send[j])), j))
        if shard(j):
            buf = torch.from_numpy(recv[j])
            reqs.append(dist.irecv(buf, j))
    for q in reqs:
        q.wait()
    grp = np.concatenate(recv, axis=0)  # rows in token order
    assert grp.shape == (S, gw)
    assert np.array_equal(grp, full_qkv[:, group_cols(r)]), "head-sharded layout"

    # back: this head group's attention rows of shard i -> rank i
    att_g = full_att[:, r * gq:(r + 1) * gq]
    back = [np.zeros((T, gq), np.float32) for _ in range(N)]
    reqs = []
    for i in range(N):
        rows = att_g[i * sh:i * sh + shard(i)]
        if i == r:
            back[i][:] = rows
            continue
        if shard(i):
            reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(rows)), i))
        if T:
            reqs.append(dist.irecv(torch.from_numpy(back[i]), i))
    for q in reqs:
        q.wait()
    attn = np.zeros((T, QW), np.float32)  # unpack: block j -> columns of head group j
    for j in range(N):
        attn[:, j * gq:(j + 1) * gq] = back[j]
    assert np.array_equal(attn, full_att[r * sh:r * sh + T]), "token-sharded attention output"

    # merge / pool: all-gather of padded shards gives the rows in token order
    pad = np.zeros((sh, 8), np.float32)
    pad[:T] = np.arange(r * sh, r * sh + T)[:, None]
    outs = [torch.zeros(sh, 8) for _ in range(N)]
    dist.all_gather(outs, torch.from_numpy(pad))
    rows = torch.cat(outs).numpy()[:S, 0]
    assert np.array_equal(rows, np.arange(S)), "gathered row order"
    dist.destroy_process_group()
    print("rank", r, "ok")
""")


@pytest.mark.parametrize("seq", [37, 64])
def test_head_parallel_exchange_two_ranks(seq):
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), SEQ=str(seq))
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, cwd=REPO, text=True))
    outs = [p.communicate(timeout=180)[0] for p in procs]
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, o
        assert f"rank {r} ok" in o
