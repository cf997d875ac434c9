"""AsyncBatcher host logic with a fake engine (the reference's
tests/test_nebula_scheduler.py approach): coalescing by (prompt length,
max_new), no mixing of cohorts unless asked for, bounded admission, failure
fan-out without retry, close semantics."""

import asyncio
import threading

import pytest

from forgeml_b200.nebula import AsyncBatcher, DecoderConfig, EngineFailed, QueueFull, ServiceClosed


class FakeEngine:
    max_requests = 64

    def __init__(self, delay=None, fail=None):
        self.batches = []
        self.delay, self.fail = delay, fail
        self.healthy = True
        self.closed = False
        self.config = DecoderConfig(vocab_size=64, hidden_size=16, num_heads=4, num_layers=2, intermediate_size=32,
                                    max_seq_len=32)

    def generate(self, prompts, max_new_tokens):
        self.batches.append((tuple(tuple(p) for p in prompts), max_new_tokens))
        if self.delay is not None:
            self.delay.wait(5)
        if self.fail is not None:
            raise self.fail
        return [[len(p)] * max_new_tokens for p in prompts]

    def close(self):
        self.closed = True


def run(coro):
    return asyncio.run(coro)


def test_coalesces_compatible_requests():
    async def go():
        e = FakeEngine()
        b = AsyncBatcher(e, max_batch_size=4, batch_window_ms=20)
        outs = await asyncio.gather(b.submit([1, 2], 2), b.submit([3, 4], 2), b.submit([5, 6], 2))
        assert outs == [[2, 2]] * 3
        assert len(e.batches) == 1 and len(e.batches[0][0]) == 3
        assert b.pending == 0
        await b.close()
        assert e.closed

    run(go())


def test_cohorts_are_not_mixed():
    async def go():
        e = FakeEngine()
        b = AsyncBatcher(e, max_batch_size=4, batch_window_ms=10)
        outs = await asyncio.gather(b.submit([1, 2], 2), b.submit([1, 2], 5), b.submit([1, 2, 3], 2))
        assert outs == [[2, 2], [2] * 5, [3, 3]]
        assert len(e.batches) == 3
        await b.close()

    run(go())


def test_batch_cap_and_queue_full():
    async def go():
        gate = threading.Event()
        e = FakeEngine(delay=gate)
        b = AsyncBatcher(e, max_batch_size=2, max_queue_size=3, batch_window_ms=0)
        tasks = [asyncio.create_task(b.submit([i, i], 1)) for i in range(3)]
        await asyncio.sleep(0.05)
        with pytest.raises(QueueFull):
            await b.submit([9, 9], 1)
        gate.set()
        outs = await asyncio.gather(*tasks)
        assert outs == [[2]] * 3
        assert all(len(batch[0]) <= 2 for batch in e.batches)
        await b.close()

    run(go())


def test_failure_fails_all_pending_without_retry():
    async def go():
        e = FakeEngine(fail=RuntimeError("boom"))
        b = AsyncBatcher(e, max_batch_size=4, batch_window_ms=5)
        res = await asyncio.gather(b.submit([1], 1), b.submit([2], 1), return_exceptions=True)
        assert all(isinstance(r, RuntimeError) for r in res)
        assert not b.healthy
        assert len(e.batches) == 1
        with pytest.raises(EngineFailed):
            await b.submit([1], 1)
        await b.close()

    run(go())


def test_close_rejects_and_validation():
    async def go():
        e = FakeEngine()
        b = AsyncBatcher(e)
        with pytest.raises(ValueError):
            await b.submit([1] * 40, 1)  # exceeds max_seq_len
        with pytest.raises(TypeError):
            await b.submit("abc", 1)
        await b.close()
        with pytest.raises(ServiceClosed):
            await b.submit([1], 1)

    run(go())
    with pytest.raises(ValueError):
        AsyncBatcher(FakeEngine(), max_batch_size=65)


class MixingEngine(FakeEngine):
    def generate_mixed(self, prompts, max_new_tokens):
        return self.generate(prompts, max_new_tokens)


def test_mixed_prompt_lengths_share_a_batch():
    async def go():
        e = MixingEngine()
        b = AsyncBatcher(e, max_batch_size=4, batch_window_ms=10, mix_prompt_lengths=True)
        outs = await asyncio.gather(b.submit([1, 2], 2), b.submit([1, 2, 3], 2), b.submit([1], 5))
        assert outs == [[2, 2], [3, 3], [1] * 5]
        assert sorted(len(batch[0]) for batch in e.batches) == [1, 2]  # max_new still splits cohorts
        await b.close()

    run(go())
    with pytest.raises(ValueError):
        AsyncBatcher(FakeEngine(), mix_prompt_lengths=True)


def test_oldest_request_goes_first():
    async def go():
        gate = threading.Event()
        e = FakeEngine(delay=gate)
        b = AsyncBatcher(e, max_batch_size=1, batch_window_ms=0)
        tasks = [asyncio.create_task(b.submit(p, 1)) for p in ([1], [1, 2], [3], [1, 2, 3])]
        await asyncio.sleep(0.05)
        gate.set()
        await asyncio.gather(*tasks)
        assert [batch[0][0] for batch in e.batches] == [(1,), (1, 2), (3,), (1, 2, 3)]
        await b.close()

    run(go())
