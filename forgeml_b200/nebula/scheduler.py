"""Asynchronous micro-batching in front of the serving engine.

Public surface of the reference AsyncBatcher (src/nebula/scheduler.py:20-199):
``AsyncBatcher(engine, *, max_batch_size, max_queue_size, batch_window_ms)``,
``await submit(prompt, max_new_tokens, timeout_s=)``, ``pending``,
``healthy``, ``close`` (also as an async context manager); QueueFull when
admission is bounded out, ServiceClosed after close, EngineFailed once a
batch failed.  Behaviour kept: requests are grouped into cohorts that one
``Engine.generate`` call can serve, the oldest waiting request's cohort goes
next, a batching window is waited only when that cohort cannot fill a batch
yet, the engine runs on a worker thread, and a failed batch fails every
waiting request (no retry).

Cohorts.  The reference's engine decodes a batch at one position, so a
cohort is (prompt length, max_new_tokens).  With ``mix_prompt_lengths=True``
(for an engine with ``generate_mixed``: this package's Engine) a cohort is
max_new_tokens alone: requests of different prompt lengths are prefilled in
their own groups and then decoded together, each at its own position.
Replica routing (the reference's RequestRouter) is not part of this path.
"""

from __future__ import annotations

import asyncio
import itertools
import logging
import math
from collections import deque
from dataclasses import dataclass, field

from forgeml_b200.nebula.engine import EngineFailed, _validate_prompt

_log = logging.getLogger(__name__)


class QueueFull(RuntimeError):
    pass


class ServiceClosed(RuntimeError):
    pass


@dataclass
class _Waiting:
    prompt: list
    max_new: int
    future: asyncio.Future
    order: int = field(default=0)


class AsyncBatcher:
    def __init__(self, engine, *, max_batch_size: int = 8, max_queue_size: int = 64, batch_window_ms: float = 5.0,
                 mix_prompt_lengths: bool = False):
        for name, v in (("max_batch_size", max_batch_size), ("max_queue_size", max_queue_size)):
            if not isinstance(v, int) or isinstance(v, bool) or v <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if (isinstance(batch_window_ms, bool) or not isinstance(batch_window_ms, (int, float))
                or not math.isfinite(batch_window_ms) or batch_window_ms < 0):
            raise ValueError("batch_window_ms must be a finite non-negative number")
        if max_batch_size > engine.max_requests:
            raise ValueError("max_batch_size exceeds engine max_requests")
        if mix_prompt_lengths and not hasattr(engine, "generate_mixed"):
            raise ValueError("mix_prompt_lengths needs an engine with generate_mixed")
        self.engine = engine
        self.max_batch_size, self.max_queue_size = max_batch_size, max_queue_size
        self.batch_window_ms = batch_window_ms
        self.mix_prompt_lengths = mix_prompt_lengths
        self._cohorts: dict[tuple, deque[_Waiting]] = {}
        self._arrivals = itertools.count()
        self._in_system = 0  # queued + being decoded
        self._closed = False
        self._failed = False
        self._engine_closed = False
        self._dispatcher: asyncio.Task | None = None
        self._work: asyncio.Event | None = None

    # ------------------------------------------------------------ state
    @property
    def pending(self) -> int:
        return self._in_system

    @property
    def healthy(self) -> bool:
        return not self._failed and not self._closed and self.engine.healthy

    def _cohort_key(self, prompt: list, max_new: int) -> tuple:
        return (max_new,) if self.mix_prompt_lengths else (len(prompt), max_new)

    # ------------------------------------------------------------ admission
    async def submit(self, prompt: list[int], max_new_tokens: int, *, timeout_s: float | None = None) -> list[int]:
        if self._closed:
            raise ServiceClosed("batcher is closed")
        if self._failed or not self.engine.healthy:
            raise EngineFailed("batcher engine is not healthy")
        if not isinstance(prompt, (list, tuple)):
            raise TypeError("prompt must be a list of token ids")
        if timeout_s is not None and (isinstance(timeout_s, bool) or not isinstance(timeout_s, (int, float))
                                      or not math.isfinite(timeout_s) or timeout_s <= 0):
            raise ValueError("timeout_s must be a finite positive number")
        prompt = list(prompt)
        _validate_prompt(self.engine.config, prompt, max_new_tokens)
        if self._in_system >= self.max_queue_size:
            raise QueueFull("request queue is full")
        loop = asyncio.get_running_loop()
        item = _Waiting(prompt, max_new_tokens, loop.create_future(), next(self._arrivals))
        self._cohorts.setdefault(self._cohort_key(prompt, max_new_tokens), deque()).append(item)
        self._in_system += 1
        if self._dispatcher is None or self._dispatcher.done():
            self._work = asyncio.Event()
            self._dispatcher = loop.create_task(self._dispatch_loop())
        self._work.set()
        waiter = asyncio.shield(item.future)
        try:
            return await (waiter if timeout_s is None else asyncio.wait_for(waiter, timeout_s))
        except (TimeoutError, asyncio.CancelledError):
            item.future.cancel()
            raise

    # ------------------------------------------------------------ dispatch
    def _queued(self) -> int:
        return sum(len(q) for q in self._cohorts.values())

    def _oldest_cohort(self) -> tuple:
        return min(self._cohorts, key=lambda k: self._cohorts[k][0].order)

    def _take(self, key: tuple) -> list[_Waiting]:
        q = self._cohorts[key]
        batch = [q.popleft() for _ in range(min(len(q), self.max_batch_size))]
        if not q:
            del self._cohorts[key]
        return batch

    def _settle(self, items, *, results=None, error=None) -> None:
        for i, it in enumerate(items):
            if not it.future.done():
                if error is not None:
                    it.future.set_exception(error)
                else:
                    it.future.set_result(results[i])
            self._in_system -= 1

    def _fail_queued(self, error) -> None:
        queued = [it for q in self._cohorts.values() for it in q]
        self._cohorts.clear()
        self._settle(queued, error=error)

    async def _dispatch_loop(self) -> None:
        try:
            while True:
                if not self._cohorts:
                    if self._closed:
                        return
                    self._work.clear()
                    await self._work.wait()
                    continue
                key = self._oldest_cohort()
                if len(self._cohorts[key]) < self.max_batch_size and self.batch_window_ms > 0:
                    await asyncio.sleep(self.batch_window_ms / 1000.0)
                    if key not in self._cohorts:  # closed meanwhile
                        continue
                batch = self._take(key)
                live = [it for it in batch if not it.future.cancelled()]
                self._settle([it for it in batch if it.future.cancelled()])
                if not live:
                    continue
                if not await self._run_batch(live):
                    return
        except Exception as exc:  # the loop itself broke: nothing queued may wait forever
            _log.exception("Nebula batch dispatcher failed")
            self._failed = True
            self._fail_queued(exc)
            raise

    async def _run_batch(self, live: list[_Waiting]) -> bool:
        prompts, max_new = [it.prompt for it in live], live[0].max_new
        call = self.engine.generate_mixed if self.mix_prompt_lengths else self.engine.generate
        try:
            results = await asyncio.to_thread(call, prompts, max_new)
            if not isinstance(results, list) or len(results) != len(live):
                raise EngineFailed("engine result count does not match the submitted batch")
        except Exception as exc:
            _log.exception("Nebula batch execution failed")
            self._failed = True
            self._settle(live, error=exc)
            self._fail_queued(exc)
            return False
        self._settle(live, results=results)
        return not (self._closed and not self._cohorts)

    # ------------------------------------------------------------ shutdown
    async def close(self) -> None:
        if not self._closed:
            self._closed = True
            self._fail_queued(ServiceClosed("batcher closed"))
            if self._work is not None:
                self._work.set()
        try:
            if self._dispatcher is not None:
                await asyncio.shield(self._dispatcher)
                self._dispatcher = None
        finally:
            if not self._engine_closed:
                self._engine_closed = True
                await asyncio.to_thread(self.engine.close)

    async def __aenter__(self):
        return self

    async def __aexit__(self, *exc):
        await self.close()
