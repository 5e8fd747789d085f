"""Distinct plans run concurrently (the reference's main.ts:292,303 awaits
Promise.all over plans): a single-launch plan (one cooperative grid over all
SMs) and a per-op plan, driven from two host threads on one GPU, give the same
embeddings as when run one after the other, and no bounded wait gives up."""
import threading

import numpy as np
import pytest

from nemo_b200 import synth
from nemo_b200.runtime import NemotronB200Model

pytestmark = pytest.mark.gpu


def test_fused_and_per_op_plans_concurrently():
    path = synth.cached_model_pack(0, "kquant", 16)
    with open(path, "rb") as f:
        data = f.read()
    model = NemotronB200Model(data, devices=[0])
    try:
        small = synth.make_requests(3, [15])
        big = synth.make_requests(4, [300, 120])
        ids_s, lens_s, seq_s = synth.pad_batch(small)
        ids_b, lens_b, seq_b = synth.pad_batch(big)
        plan_s = model.create_plan(1, seq_s)
        plan_b = model.create_plan(2, seq_b)
        assert plan_s.fused and not plan_b.fused
        want_s = plan_s.run_array(ids_s, lens_s).copy()
        want_b = plan_b.run_array(ids_b, lens_b).copy()
        errors = []

        def loop(plan, ids, lens, want, n):
            try:
                for _ in range(n):
                    got = plan.run_array(ids, lens)
                    if not np.array_equal(got, want):
                        errors.append("embeddings differ under concurrency")
                        return
            except Exception as e:  # a NemoError from a bounded wait, a CUDA error
                errors.append(repr(e))

        threads = [threading.Thread(target=loop, args=(plan_s, ids_s, lens_s, want_s, 200)),
                   threading.Thread(target=loop, args=(plan_b, ids_b, lens_b, want_b, 40))]
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=300)
        assert not any(t.is_alive() for t in threads), "a plan did not finish"
        assert not errors, errors
    finally:
        model.destroy()
