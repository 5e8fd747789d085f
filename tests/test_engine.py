"""The reference's engine tests (tests/embedding-engine.test.ts:5-50) against
the Python restatement of NemotronEmbeddingEngine."""
import asyncio

import numpy as np
import pytest

from nemo_b200.engine import NemotronEmbeddingEngine


class _Ids:
    def __init__(self, rows):
        self.rows = rows

    def tolist(self):
        return self.rows


class _Tok:
    def __init__(self, fn):
        self.fn = fn

    def __call__(self, text):
        return {"input_ids": _Ids(self.fn(text))}


def test_coalesces_sixteen_requests_and_preserves_order(golden):
    case = golden["engine"]["coalesce"]
    calls = []

    class Runtime:
        def create_plan(self, batch, sequence):
            class Plan:
                async def run(self, ids, lengths):
                    calls.append({"batch": batch, "sequence": sequence, "ids": list(ids), "lengths": list(lengths)})
                    return [np.array([ids[i * sequence + 1]], np.float32) for i in range(batch)]
            return Plan()

    engine = NemotronEmbeddingEngine(Runtime(), _Tok(lambda t: [[int(t)]]), 16, 0, case["bos"])

    async def main():
        return await asyncio.gather(*[engine.embed(str(i + 1)) for i in range(case["requests"])])

    results = asyncio.run(main())
    assert len(calls) == case["expect_calls"]
    assert calls[0]["batch"] == case["expect_batch"] and calls[0]["sequence"] == case["expect_sequence"]
    assert calls[0]["lengths"] == case["expect_lengths"]
    assert [float(r[0]) for r in results] == [float(i + 1) for i in range(16)]


def test_pads_mixed_length_requests_after_final_token(golden):
    case = golden["engine"]["padding"]
    recorded = []

    class Runtime:
        def create_plan(self, batch, sequence):
            class Plan:
                async def run(self, ids, lengths):
                    recorded[:] = list(ids)
                    return [np.zeros(1, np.float32) for _ in range(batch)]
            return Plan()

    engine = NemotronEmbeddingEngine(Runtime(), _Tok(lambda t: [[int(x) for x in t.split(",")]]), 16, 0,
                                     case["bos"], case["pad"])

    async def main():
        await asyncio.gather(*[engine.embed(t) for t in case["texts"]])

    asyncio.run(main())
    assert recorded == case["expect_ids"]


def test_splits_batches_for_storage_limit(golden):
    case = golden["engine"]["storage_split"]
    batches = []

    class Runtime:
        max_storage_buffer_binding_size = case["max_storage"]

        def create_plan(self, batch, sequence):
            class Plan:
                async def run(self, ids, lengths):
                    batches.append(batch)
                    return [np.zeros(1, np.float32) for _ in range(batch)]
            return Plan()

    engine = NemotronEmbeddingEngine(Runtime(), _Tok(lambda t: [[1]]), 16, 0, 1)

    async def main():
        await asyncio.gather(*[engine.embed("x") for _ in range(case["requests"])])

    asyncio.run(main())
    assert batches == case["expect_batches"]


def test_long_requests_cap_at_eight_and_failures_reject_the_batch():
    sizes = []

    class Runtime:
        def create_plan(self, batch, sequence):
            class Plan:
                def run(self, ids, lengths):  # blocking runtime: runs on a worker thread
                    sizes.append(batch)
                    if sequence == 3:
                        raise RuntimeError("device lost")
                    return [np.zeros(1, np.float32) for _ in range(batch)]
            return Plan()

    engine = NemotronEmbeddingEngine(Runtime(), _Tok(lambda t: [[1] * int(t)]), 16, 0, 1)

    async def main():
        ok = await asyncio.gather(*[engine.embed("1500") for _ in range(10)])
        bad = await asyncio.gather(*[engine.embed("3") for _ in range(2)], return_exceptions=True)
        return ok, bad

    ok, bad = asyncio.run(main())
    assert sizes[:2] == [8, 2] and len(ok) == 10
    assert all(isinstance(b, RuntimeError) for b in bad)


def test_rejects_bad_batch_size():
    with pytest.raises(ValueError):
        NemotronEmbeddingEngine(object(), lambda t: None, 17)


def test_micro_batches_follow_the_engines_flush():
    """micro_batches (the bench's split of a request queue) takes the same
    batches as the engine's flush: <= 16, <= 8 when the longest candidate has
    >= 1500 tokens."""
    from nemo_b200.engine import micro_batches
    assert micro_batches([15] * 16) == [list(range(16))]
    assert micro_batches([1500] * 16) == [list(range(8)), list(range(8, 16))]
    assert micro_batches([5000] * 10) == [list(range(8)), [8, 9]]
    assert micro_batches([15] * 20) == [list(range(16)), [16, 17, 18, 19]]
    assert micro_batches([10, 1499, 1500, 3]) == [[0, 1, 2, 3]]  # one candidate >= 1500 caps at 8
    sizes = []

    class Runtime:
        def create_plan(self, batch, sequence):
            class Plan:
                def run(self, ids, lengths):
                    sizes.append(batch)
                    return [np.zeros(1, np.float32) for _ in range(batch)]
            return Plan()

    lengths = [20] * 3 + [1600] * 9 + [7] * 20
    engine = NemotronEmbeddingEngine(Runtime(), _Tok(lambda t: [[1] * int(t)]), 16, 0, 1)

    async def main():
        return await asyncio.gather(*[engine.embed(str(n)) for n in lengths])

    asyncio.run(main())
    assert sizes == [len(b) for b in micro_batches(lengths)]
