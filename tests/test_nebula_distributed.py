"""Multi-rank engine protocol on Gloo CPU processes (reference
tests/test_nebula_distributed.py pattern): TP2, PP2 and TP2xPP2 leaders drive
workers in ``serve()`` through the command broadcasts; results must equal the
monolithic model; a dying worker must surface as EngineFailed on the leader
with a cleared cache.  The CPU sharded decoder harness stands in for the
CUDA-only product decoder; the engine, protocol and ParallelContext are the
product's."""

import tempfile
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.distributed,
              pytest.mark.skipif(not (dist.is_available() and dist.is_gloo_available()), reason="no gloo")]

CFG = dict(vocab_size=32, hidden_size=16, num_heads=4, num_layers=4, intermediate_size=32, max_seq_len=16, seed=17)


def _ref_generate(model, prompt, n):
    out, cur = [], list(prompt)
    for _ in range(n):
        with torch.no_grad():
            nxt = int(model(torch.tensor([cur], dtype=torch.long))[0, -1].argmax())
        out.append(nxt)
        cur.append(nxt)
    return out


def _worker(rank, world, tp, pp, store):
    from forgeml_b200.nebula import DecoderConfig, Engine, ParallelContext, TinyDecoder
    from tests.cpu_engine import CpuShardedDecoder

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=20))
    cfg = DecoderConfig(**CFG)
    ctx = ParallelContext.from_env(tp_size=tp, pp_size=pp, timeout_s=20)
    engine = Engine(cfg, context=ctx, max_requests=4, decoder_factory=CpuShardedDecoder)
    try:
        if rank == 0:
            ref = TinyDecoder(cfg).eval()
            toks = torch.tensor([[1, 2, 3], [4, 5, 6]])
            with torch.no_grad():
                want = ref(toks)
            torch.testing.assert_close(engine.forward(toks, (21, 22), 0), want, rtol=1e-4, atol=1e-5)
            got2 = engine.forward(torch.tensor([[7], [8]]), (21, 22), 3)
            with torch.no_grad():
                want2 = ref(torch.tensor([[1, 2, 3, 7], [4, 5, 6, 8]]))[:, -1:, :]
            torch.testing.assert_close(got2, want2, rtol=1e-4, atol=1e-5)
            engine.release((21, 22))
            assert engine.decoder.cache.active_requests == 0
            prompts = [[1, 2, 3], [5, 6]]
            assert engine.generate(prompts, 3) == [_ref_generate(ref, p, 3) for p in prompts]
            assert engine.decoder.cache.active_requests == 0
            # prompts of different lengths decoded in one batch (STEP_AT on the wire)
            mixed = [[1, 2, 3, 4], [5, 6], [7]]
            assert engine.generate_mixed(mixed, 4) == [_ref_generate(ref, p, 4) for p in mixed]
            assert engine.decoder.cache.active_requests == 0
        else:
            engine.serve()
            assert engine.decoder.cache.active_requests == 0
    finally:
        engine.close()
        ctx.close()
        if dist.is_initialized():
            dist.destroy_process_group()


def _spawn(fn, args, nprocs, limit):
    procs = mp.start_processes(fn, args=args, nprocs=nprocs, join=False, start_method="spawn")
    deadline = time.time() + limit
    while time.time() < deadline and not all(p.exitcode is not None for p in procs.processes):
        time.sleep(0.2)
    for p in procs.processes:
        if p.is_alive():
            p.terminate()
    for p in procs.processes:
        p.join()
    return procs


def _run(world, tp, pp):
    with tempfile.TemporaryDirectory() as d:
        procs = _spawn(_worker, (world, tp, pp, f"{d}/store"), world, 90)
        assert [p.exitcode for p in procs.processes] == [0] * world


def test_tp2_pp1():
    _run(2, 2, 1)


def test_tp1_pp2():
    _run(2, 1, 2)


def test_tp2_pp2():
    _run(4, 2, 2)


def _failing(rank, store):
    from forgeml_b200.nebula import DecoderConfig, Engine, EngineFailed, ParallelContext
    from tests.cpu_engine import CpuShardedDecoder

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=10))
    ctx = ParallelContext.from_env(tp_size=2, pp_size=1, timeout_s=10)
    engine = Engine(DecoderConfig(**CFG), context=ctx, max_requests=4, decoder_factory=CpuShardedDecoder)
    if rank == 0:
        try:
            engine.forward(torch.tensor([[1, 2, 3]]), (1,), 0)
        except EngineFailed:
            assert not engine.healthy and engine.decoder.cache.active_requests == 0
            return
        raise AssertionError("forward did not fail after peer death")
    raise RuntimeError("deliberate worker failure")


def test_worker_failure_propagates():
    with tempfile.TemporaryDirectory() as d:
        procs = _spawn(_failing, (f"{d}/store",), 2, 60)
        assert procs.processes[0].exitcode == 0
        assert procs.processes[1].exitcode != 0


def _dying_in_prefill(rank, store):
    """TP1 x PP2: the second stage dies inside a pipelined PREFILL command."""
    from forgeml_b200.nebula import DecoderConfig, Engine, EngineFailed, ParallelContext
    from tests.cpu_engine import CpuShardedDecoder

    class _Dying(CpuShardedDecoder):
        def forward(self, *args, defer_broadcast=False, **kw):
            if defer_broadcast:
                raise RuntimeError("deliberate stage failure during prefill")
            return super().forward(*args, defer_broadcast=defer_broadcast, **kw)

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=10))
    ctx = ParallelContext.from_env(tp_size=1, pp_size=2, timeout_s=10)
    engine = Engine(DecoderConfig(**CFG), context=ctx, max_requests=4,
                    decoder_factory=CpuShardedDecoder if rank == 0 else _Dying)
    if rank == 0:
        assert engine.pipelined_prefill
        try:
            engine.generate_mixed([[1, 2, 3], [4, 5]], 2)
        except EngineFailed:
            assert not engine.healthy and engine.decoder.cache.active_requests == 0
            try:
                engine.generate_mixed([[1, 2]], 1)
            except EngineFailed:
                return
            raise AssertionError("a failed engine accepted another request")
        raise AssertionError("generate_mixed did not fail after a stage died in prefill")
    engine.serve()


def test_stage_failure_in_pipelined_prefill_poisons_the_leader():
    with tempfile.TemporaryDirectory() as d:
        procs = _spawn(_dying_in_prefill, (f"{d}/store",), 2, 60)
        assert procs.processes[0].exitcode == 0
        assert procs.processes[1].exitcode != 0


def _batcher_worker(rank, store):
    """TP2 x PP2 serving as in config 5: an AsyncBatcher that mixes prompt
    lengths in front of the leader; workers in serve()."""
    import asyncio

    from forgeml_b200.nebula import AsyncBatcher, DecoderConfig, Engine, ParallelContext, TinyDecoder
    from tests.cpu_engine import CpuShardedDecoder

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=4,
                            timeout=timedelta(seconds=20))
    cfg = DecoderConfig(**CFG)
    ctx = ParallelContext.from_env(tp_size=2, pp_size=2, timeout_s=20)
    engine = Engine(cfg, context=ctx, max_requests=4, decoder_factory=CpuShardedDecoder)
    try:
        if rank == 0:
            ref = TinyDecoder(cfg).eval()
            prompts = [[1, 2, 3], [4], [5, 6, 7, 8], [9, 10]]
            batches = []
            mixed = engine.generate_mixed

            def recording(ps, n):
                batches.append(sorted(len(p) for p in ps))
                return mixed(ps, n)

            engine.generate_mixed = recording

            async def go():
                async with AsyncBatcher(engine, max_batch_size=4, batch_window_ms=50,
                                        mix_prompt_lengths=True) as b:
                    return await asyncio.gather(*(b.submit(p, 3) for p in prompts))

            assert asyncio.run(go()) == [_ref_generate(ref, p, 3) for p in prompts]
            # every request served once, and prompts of different lengths shared a batch
            assert sorted(n for b in batches for n in b) == [1, 2, 3, 4]
            assert max(len(set(b)) for b in batches) > 1
            assert engine.decoder.cache.active_requests == 0
        else:
            engine.serve()
            assert engine.decoder.cache.active_requests == 0
    finally:
        engine.close()
        ctx.close()
        if dist.is_initialized():
            dist.destroy_process_group()


def test_batcher_mixing_prompt_lengths_on_tp2_pp2():
    with tempfile.TemporaryDirectory() as d:
        procs = _spawn(_batcher_worker, (f"{d}/store",), 4, 90)
        assert [p.exitcode for p in procs.processes] == [0] * 4


def _preflight_all(rank, store):
    """A command the cache replicas reject (a reserved id at position 0)
    fails on every rank at once: the leader and the worker both end poisoned
    with their caches cleared, none waiting on the other."""
    from forgeml_b200.nebula import DecoderConfig, Engine, EngineFailed, ParallelContext
    from tests.cpu_engine import CpuShardedDecoder

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=20))
    ctx = ParallelContext.from_env(tp_size=1, pp_size=2, timeout_s=20)
    engine = Engine(DecoderConfig(**CFG), context=ctx, max_requests=4, decoder_factory=CpuShardedDecoder)
    if rank == 0:
        engine.forward(torch.tensor([[1, 2, 3]]), (5,), 0)
        t0 = time.monotonic()
        try:
            engine.forward(torch.tensor([[4, 5]]), (5,), 0)
        except EngineFailed as exc:
            assert "preflight" in str(exc.__cause__)
            assert not engine.healthy and engine.decoder.cache.active_requests == 0
            assert time.monotonic() - t0 < 10  # no collective timeout was waited out
            return
        raise AssertionError("a reserved id was admitted again")
    try:
        engine.serve()
    except EngineFailed:
        assert not engine.healthy and engine.decoder.cache.active_requests == 0
        return
    raise AssertionError("the worker served past a failed preflight")


def test_preflight_failure_fails_every_rank_together():
    with tempfile.TemporaryDirectory() as d:
        procs = _spawn(_preflight_all, (f"{d}/store",), 2, 60)
        assert [p.exitcode for p in procs.processes] == [0, 0]
