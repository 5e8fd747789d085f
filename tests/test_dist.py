"""The N>1 request-sharded path on CPU: two gloo ranks run the same rank
plumbing bench.py uses (barrier, max-over-ranks timing, whole-job throughput)
and the request split of multi-device plans."""
import os
import socket
import subprocess
import sys
import textwrap

from conftest import PKG_DIR, REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


WORKER = textwrap.dedent("""
    import sys, time
    sys.path.insert(0, {pkg!r})
    from nemo_b200 import dist as nd
    info = nd.init("gloo", 60.0)
    assert info.world == 2
    # rank 1 is slower: the job time is the max over ranks
    t0 = time.perf_counter()
    time.sleep(0.05 + 0.15 * info.rank)
    nd.barrier(info)
    local = time.perf_counter() - t0 if info.rank == 0 else 0.2
    worst = nd.max_over_ranks(info, 0.2 if info.rank == 1 else 0.05)
    assert abs(worst - 0.2) < 1e-12, worst
    v = nd.throughput(info.world, 10, 1, worst)
    assert abs(v - 100.0) < 1e-9, v
    nd.shutdown(info)
    print("rank", info.rank, "ok")
""")


def test_two_gloo_ranks():
    port = _free_port()
    code = WORKER.format(pkg=PKG_DIR)
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, cwd=REPO, text=True))
    outs = [p.communicate(timeout=120)[0] for p in procs]
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, o
        assert f"rank {r} ok" in o


def test_shard_requests_balances_tokens():
    from nemo_b200.dist import shard_requests
    lengths = [1500, 15, 150, 1500, 40, 700, 5, 5]
    shards = shard_requests(lengths, 3)
    assert sorted(i for s in shards for i in s) == list(range(len(lengths)))
    loads = [sum(lengths[i] for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(lengths)
    assert shard_requests([7], 4) == [[0], [], [], []]
