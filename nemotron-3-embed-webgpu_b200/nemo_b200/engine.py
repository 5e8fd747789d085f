"""The reference's micro-batching embedding engine, restated for Python hosts.

``NemotronEmbeddingEngine`` follows src/webgpu/embedding-engine.ts:22-96 line by
line in behaviour: requests are queued, coalesced up to ``max_batch_size`` (16)
per micro-batch, capped by the runtime's storage-binding size and to 8 when the
longest request has >= 1500 tokens, padded after each request's last token,
and run serially on a plan cached per ``batch:sequence``; a failing batch
rejects every request in it. ``runtime`` is any object with
``create_plan(batch, sequence)`` and optional ``max_storage_buffer_binding_size``
(the B200 ``NemotronB200Model`` or a fake). A plan's ``run`` may be a coroutine
function or a blocking call (run on a worker thread, as the N-API addon does
with napi_async_work).
"""
from __future__ import annotations

import asyncio
import inspect
import math

import numpy as np


def micro_batches(lengths: list[int], max_batch_size: int = 16) -> list[list[int]]:
    """The engine's split of a queue of requests (token counts, BOS included)
    into micro-batches, as ``_flush`` takes them with no storage cap (the B200
    runtime has none): up to ``max_batch_size`` per batch, at most 8 when the
    longest candidate has >= 1500 tokens (embedding-engine.ts:62-69). Returns
    lists of request indices in queue order."""
    out, i = [], 0
    while i < len(lengths):
        candidates = lengths[i:i + max_batch_size]
        take = min(max_batch_size, 8 if max(candidates) >= 1500 else max_batch_size)
        out.append(list(range(i, min(i + take, len(lengths)))))
        i += take
    return out


class NemotronEmbeddingEngine:
    def __init__(self, runtime, tokenizer, max_batch_size: int = 16, batch_window_ms: float = 0,
                 bos_token: int = 1, pad_token: int = 11):
        if max_batch_size < 1 or max_batch_size > 16:
            raise ValueError("maxBatchSize must be between 1 and 16")
        self.runtime = runtime
        self.tokenizer = tokenizer
        self.max_batch_size = max_batch_size
        self.batch_window_ms = batch_window_ms
        self.bos_token = bos_token
        self.pad_token = pad_token
        self._pending: list[tuple[list[int], asyncio.Future]] = []
        self._plans: dict[str, object] = {}
        self._scheduled = False
        self._flushing = False

    def _tokens(self, text: str) -> list[int]:
        res = self.tokenizer(text)
        input_ids = res["input_ids"] if isinstance(res, dict) else res.input_ids
        rows = input_ids.tolist() if hasattr(input_ids, "tolist") else input_ids
        return [int(t) for t in rows[0]]

    async def embed(self, text: str) -> np.ndarray:
        """embedding-engine.ts:40-47: tokenise, prepend BOS if missing, queue."""
        tokens = self._tokens(text)
        if not tokens or tokens[0] != self.bos_token:
            tokens.insert(0, self.bos_token)
        fut = asyncio.get_running_loop().create_future()
        self._pending.append((tokens, fut))
        self._schedule()
        return await fut

    def _schedule(self) -> None:
        if self._scheduled or self._flushing:
            return
        self._scheduled = True
        loop = asyncio.get_running_loop()

        def fire():
            self._scheduled = False
            asyncio.ensure_future(self._flush())

        loop.call_later(self.batch_window_ms / 1000.0, fire)

    async def _run_plan(self, plan, ids: np.ndarray, lengths: np.ndarray):
        run = plan.run
        if inspect.iscoroutinefunction(run):
            return await run(ids, lengths)
        result = await asyncio.get_running_loop().run_in_executor(None, run, ids, lengths)
        if inspect.isawaitable(result):
            result = await result
        return result

    async def _flush(self) -> None:
        """embedding-engine.ts:58-95."""
        if self._flushing:
            return
        self._flushing = True
        try:
            while self._pending:
                candidates = self._pending[:self.max_batch_size]
                candidate_sequence = max(len(t) for t, _ in candidates)
                limit = getattr(self.runtime, "max_storage_buffer_binding_size", None)
                storage_limit = math.inf if limit is None else limit
                bytes_per_request = candidate_sequence * 6144 * 2 * 2
                storage_cap = max(1, int(storage_limit // bytes_per_request)) if storage_limit != math.inf else math.inf
                long_cap = 8 if candidate_sequence >= 1500 else self.max_batch_size
                take = int(min(self.max_batch_size, storage_cap, long_cap))
                requests = self._pending[:take]
                del self._pending[:take]
                sequence = max(len(t) for t, _ in requests)
                ids = np.full(len(requests) * sequence, self.pad_token, dtype=np.uint32)
                lengths = np.zeros(len(requests), dtype=np.uint32)
                for i, (tokens, _) in enumerate(requests):
                    ids[i * sequence:i * sequence + len(tokens)] = tokens
                    lengths[i] = len(tokens)
                key = f"{len(requests)}:{sequence}"
                plan = self._plans.get(key)
                if plan is None:
                    plan = self.runtime.create_plan(len(requests), sequence)
                    self._plans[key] = plan
                try:
                    embeddings = await self._run_plan(plan, ids, lengths)
                    for i, (_, fut) in enumerate(requests):
                        if not fut.done():
                            fut.set_result(embeddings[i])
                except Exception as error:  # every request of the failing batch is rejected
                    for _, fut in requests:
                        if not fut.done():
                            fut.set_exception(error)
        finally:
            self._flushing = False
            if self._pending:
                self._schedule()
