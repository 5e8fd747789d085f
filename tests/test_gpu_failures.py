"""Failure paths of the C ABI, made to happen without faulting the GPU.

* A bounded device-side wait that runs out: with test knobs set at plan
  creation, one grid barrier of the single-launch forward waits for one
  arrival more than the grid has, gives up at a 50 ms bound, and every CTA
  unwinds through the error word. nemo_plan_run returns NEMO_ERR_TIMEOUT and
  the same plan then runs normally, bit-identical to a plan without knobs.
* A device that fails its share of a micro-batch (host-side injection): the
  whole micro-batch is rejected, and the reference's engine rejects every
  request of that batch (src/webgpu/embedding-engine.ts:84-89) while other
  batches succeed.
* The host-side deadline on waiting for a device: nemo_plan_run returns
  NEMO_ERR_TIMEOUT instead of blocking past it; the device work still ends
  and the plan can be synchronised.
"""
import asyncio
import time

import numpy as np
import pytest

from nemo_b200 import synth
from nemo_b200.engine import NemotronEmbeddingEngine
from nemo_b200.runtime import NemoError, NemotronB200Model

pytestmark = pytest.mark.gpu

ERR_TIMEOUT = -5


@pytest.fixture(scope="module")
def pack5():
    with open(synth.cached_model_pack(2, "kquant", 5), "rb") as f:
        return f.read()


def _request(n, seed=3):
    reqs = synth.make_requests(seed, [n])
    ids, lens, seq = synth.pad_batch(reqs)
    return ids, lens, seq


def test_device_wait_bound_expires_and_plan_recovers(pack5, monkeypatch):
    model = NemotronB200Model(pack5)
    try:
        ids, lens, seq = _request(15)
        ref_plan = model.create_plan(1, seq)
        want = ref_plan.run_array(ids, lens).copy()
        monkeypatch.setenv("NEMO_TEST_FAULTS", "1")
        monkeypatch.setenv("NEMO_TEST_WAIT_LIMIT_MS", "50")
        plan = model.create_plan(1, seq)
        monkeypatch.delenv("NEMO_TEST_FAULTS")
        monkeypatch.delenv("NEMO_TEST_WAIT_LIMIT_MS")
        assert plan.fused
        for barrier in (1, 3, 9):
            monkeypatch.setenv("NEMO_TEST_STALL_BARRIER", str(barrier))
            t0 = time.perf_counter()
            with pytest.raises(NemoError, match="bounded wait") as e:
                plan.run_array(ids, lens)
            assert e.value.status == ERR_TIMEOUT
            assert time.perf_counter() - t0 < 1.5  # gave up at the 50 ms bound, not 2 s
            monkeypatch.setenv("NEMO_TEST_STALL_BARRIER", "0")
            got = plan.run_array(ids, lens)
            assert np.array_equal(got, want)
    finally:
        model.destroy()


class _Tok:
    def __init__(self, vocab):
        self.rng = np.random.default_rng(9)
        self.vocab = vocab

    def __call__(self, text):
        n = int(text)
        return {"input_ids": np.array([[1] + self.rng.integers(0, self.vocab, n - 1).tolist()])}


def test_failed_device_share_rejects_the_whole_batch(pack5, monkeypatch):
    # two replicas on one GPU stand in for two devices: the split and the
    # failure handling are host logic
    model = NemotronB200Model(pack5, devices=[0, 0])
    try:
        vocab = model.info().vocab
        monkeypatch.setenv("NEMO_TEST_FAIL_DEVICE", "1")
        plan = model.create_plan(4, 20)
        reqs = synth.make_requests(4, [20, 18, 7, 3], vocab=vocab)
        ids, lens, seq = synth.pad_batch(reqs)
        with pytest.raises(NemoError, match="injected failure"):
            plan.run(ids, lens)
        # the engine rejects every request of the failing batch
        engine = NemotronEmbeddingEngine(model, _Tok(vocab), 4, 0, 1)

        async def batch():
            return await asyncio.gather(*[engine.embed(str(n)) for n in (12, 9, 5, 3)], return_exceptions=True)

        res = asyncio.run(batch())
        assert all(isinstance(r, NemoError) and "injected failure" in str(r) for r in res)
        monkeypatch.delenv("NEMO_TEST_FAIL_DEVICE")
        ok_engine = NemotronEmbeddingEngine(model, _Tok(vocab), 4, 0, 1)

        async def ok_batch():
            return await asyncio.gather(*[ok_engine.embed(str(n)) for n in (12, 9, 5, 3)])

        for e in asyncio.run(ok_batch()):
            assert abs(np.linalg.norm(e) - 1) < 1e-3
    finally:
        model.destroy()


def test_host_deadline_returns_timeout(pack5, monkeypatch):
    model = NemotronB200Model(pack5)
    try:
        ids, lens, seq = _request(4000)
        monkeypatch.setenv("NEMO_HOST_DEADLINE_MS", "1")
        plan = model.create_plan(1, seq)
        monkeypatch.delenv("NEMO_HOST_DEADLINE_MS")
        with pytest.raises(NemoError, match="host deadline") as e:
            plan.run_array(ids, lens)
        assert e.value.status == ERR_TIMEOUT
        plan.synchronize()  # the device work itself ends
        ok = model.create_plan(1, seq)
        out = ok.run_array(ids, lens)
        assert abs(np.linalg.norm(out[0]) - 1) < 1e-3
    finally:
        model.destroy()
