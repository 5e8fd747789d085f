"""Request sharding inside the C ABI: a model loaded on two devices splits each
micro-batch's requests across them (longest first onto the least-loaded
device); the embeddings must match the single-device run. Skipped with fewer
than two GPUs."""
import numpy as np
import pytest

from nemo_b200 import synth
from nemo_b200.runtime import NemotronB200Model

pytestmark = pytest.mark.gpu


def test_two_device_plan_matches_single_device():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = synth.cached_model_pack(3, "kquant", 5)
    with open(path, "rb") as f:
        data = f.read()
    reqs = synth.make_requests(8, [15, 40, 7, 33, 2], vocab=synth.VOCAB)
    ids, lens, seq = synth.pad_batch(reqs)
    one = NemotronB200Model(data, devices=[0])
    two = NemotronB200Model(data, devices=[0, 1])
    try:
        assert two.info().n_devices == 2
        a = one.create_plan(len(reqs), seq).run_array(ids, lens).copy()
        b = two.create_plan(len(reqs), seq).run_array(ids, lens).copy()
    finally:
        one.destroy()
        two.destroy()
    for i in range(len(reqs)):
        cos = float(a[i] @ b[i] / (np.linalg.norm(a[i]) * np.linalg.norm(b[i])))
        assert cos >= 0.9999, (i, cos)


@pytest.mark.parametrize("n_dev", [2, 4, 8])
@pytest.mark.parametrize("length", [700, 2300])
def test_head_parallel_matches_single_device(length, n_dev, monkeypatch):
    """One long request on a 2-, 4- or 8-device plan runs head-parallel (token-sharded
    projections; the QKV GEMM epilogue stores Q/K/V into the devices owning each
    head group and the attention epilogue stores rows into the devices owning
    them, over peer memory; peer copies gather rows for the merge and the
    pool); 2300 tokens also samples every third key before the merge. The
    embedding must match the single-device run, and the directly issued first
    run, the captured second run and the replayed third run must agree bit for
    bit."""
    import torch
    if torch.cuda.device_count() < n_dev:
        pytest.skip(f"needs {n_dev} GPUs")
    path = synth.cached_model_pack(3, "kquant", 5)
    with open(path, "rb") as f:
        data = f.read()
    reqs = synth.make_requests(9, [length], vocab=synth.VOCAB)
    ids, lens, seq = synth.pad_batch(reqs)
    one = NemotronB200Model(data, devices=[0])
    two = NemotronB200Model(data, devices=list(range(n_dev)))
    try:
        monkeypatch.setenv("NEMO_HEAD_PARALLEL_MIN", "512")
        plan2 = two.create_plan(1, seq)
        assert plan2.head_parallel_min == 512
        b = plan2.run_array(ids, lens).copy()   # issued directly
        b2 = plan2.run_array(ids, lens).copy()  # captured as one multi-device CUDA graph, then launched
        b3 = plan2.run_array(ids, lens).copy()  # graph replay
        plan1 = one.create_plan(1, seq)
        assert plan1.head_parallel_min == 0
        a = plan1.run_array(ids, lens).copy()
    finally:
        one.destroy()
        two.destroy()
    assert np.array_equal(b, b2) and np.array_equal(b, b3)
    cos = float(a[0] @ b[0] / (np.linalg.norm(a[0]) * np.linalg.norm(b[0])))
    assert cos >= 0.9999, cos
    assert abs(np.linalg.norm(b[0]) - 1) < 1e-3
