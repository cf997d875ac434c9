"""Tensor/pipeline parallel engine on several B200s (NCCL over NVLink).

One process per GPU; the leader drives workers in ``serve()`` through the
reference command protocol.  fp32 results must match the monolithic CPU
oracle (rtol 1e-5, atol 1e-5) and greedy tokens must match exactly; bf16 runs
must agree with the single-GPU native engine on the same weights
(rtol 2e-2, atol 2e-2 * max|logits|).  Skipped when the box has fewer GPUs
than ranks.
"""

import tempfile
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(vocab_size=512, hidden_size=256, num_heads=8, num_layers=4, intermediate_size=512, max_seq_len=64, seed=17)


def _worker(rank, world, tp, pp, store, dtype_name):
    import os

    from forgeml_b200.nebula import DecoderConfig, Engine, ParallelContext, TinyDecoder
    from oracle import nebula as orc

    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    dtype = getattr(torch, dtype_name)
    cfg = DecoderConfig(**CFG)
    ctx = ParallelContext.from_env(tp_size=tp, pp_size=pp, device="cuda", timeout_s=60)
    engine = Engine(cfg, context=ctx, dtype=dtype, max_requests=4)
    try:
        if rank == 0:
            ref = TinyDecoder(cfg).eval()
            w = orc.weights_from_state_dict({k: v.to(dtype).float() for k, v in ref.state_dict().items()},
                                            cfg.num_layers)
            g = torch.Generator().manual_seed(5)
            toks = torch.randint(0, cfg.vocab_size, (2, 9), generator=g)
            got = engine.forward(toks, (21, 22), 0).float().cpu()
            want = orc.forward(w, toks, cfg.num_heads, cfg.num_layers)
            if dtype == torch.float32:
                torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
            else:
                torch.testing.assert_close(got, want, rtol=2e-2, atol=2e-2 * float(want.abs().max()))
            step = got[:, -1].argmax(-1, keepdim=True)
            got_d = engine.forward(step, (21, 22), 9).float().cpu()
            want_d = orc.forward(w, torch.cat([toks, step], 1), cfg.num_heads, cfg.num_layers)[:, -1:]
            tol = (1e-5, 1e-5) if dtype == torch.float32 else (2e-2, 2e-2 * float(want_d.abs().max()))
            torch.testing.assert_close(got_d, want_d, rtol=tol[0], atol=tol[1])
            engine.release((21, 22))
            prompts = toks.tolist()
            gen = engine.generate(prompts, 4)
            if dtype == torch.float32:
                assert gen == [orc.greedy(w, p, 4, cfg.num_heads, cfg.num_layers) for p in prompts]
            assert engine.decoder.cache.active_requests == 0
        else:
            engine.serve()
    finally:
        engine.close()
        torch.cuda.synchronize()
        dist.barrier()
        ctx.close()
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, tp, pp, dtype_name="float32"):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        procs = mp.start_processes(_worker, args=(world, tp, pp, f"{d}/store", dtype_name), nprocs=world,
                                   join=False, start_method="spawn")
        deadline = time.time() + 240
        while time.time() < deadline and not all(p.exitcode is not None for p in procs.processes):
            time.sleep(0.2)
        for p in procs.processes:
            if p.is_alive():
                p.terminate()
        for p in procs.processes:
            p.join()
        assert [p.exitcode for p in procs.processes] == [0] * world


def test_tp2_fp32():
    _run(2, 2, 1)


def test_tp2_bf16():
    _run(2, 2, 1, "bfloat16")


def test_pp2_fp32():
    _run(2, 1, 2)


def test_tp2_pp2_bf16():
    _run(4, 2, 2, "bfloat16")


def test_tp4_bf16():
    _run(4, 4, 1, "bfloat16")


def test_tp8_bf16():
    _run(8, 8, 1, "bfloat16")


def _ar_worker(rank, world, store, dtype_name, proto="auto"):
    import os

    from forgeml_b200.nebula import ParallelContext
    from forgeml_b200.nebula.peer import PeerAllReduce

    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    ctx = ParallelContext.from_env(tp_size=world, pp_size=1, device="cuda", timeout_s=60)
    dtype = getattr(torch, dtype_name)
    dev = ctx.device
    ar = PeerAllReduce(ctx, max_bytes=1 << 20, protocol=proto)
    try:
        for it, n in enumerate((2048 * 32, 8, 4096, 2048 * 32)):
            g = torch.Generator().manual_seed(1000 * it + rank)
            part = torch.randn(n, generator=g).to(dtype)
            res = torch.randn(n, generator=torch.Generator().manual_seed(77 + it)).to(dtype)  # same on all ranks
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather_object(parts, part)
            acc = torch.zeros(n, dtype=torch.float32)
            for p in parts:  # rank order, fp32
                acc += p.float()
            want = (acc.to(dtype).float() + res.float()).to(dtype)
            out = torch.empty(n, dtype=dtype, device=dev)
            ar(part.to(dev), res.to(dev), out)
            assert torch.equal(out.cpu(), want), f"rank {rank} iteration {it}"
            want_plain = acc.to(dtype)
            ar(part.to(dev), None, out)
            assert torch.equal(out.cpu(), want_plain)
        # replay inside a CUDA graph: epochs advance on the device
        part = torch.full((4096,), float(rank + 1), dtype=dtype, device=dev)
        res = torch.ones(4096, dtype=dtype, device=dev)
        out = torch.empty_like(part)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ar(part, res, out)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            ar(part, res, out)
        for _ in range(5):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.all(out.float() == 1 + world * (world + 1) / 2)
        del graph
        from forgeml_b200 import _native
        assert _native.device_status() == 0
    finally:
        ar.close()
        torch.cuda.synchronize()
        dist.barrier()
        ctx.close()
        if dist.is_initialized():
            dist.destroy_process_group()


def _run_ar(world, dtype_name, proto="auto"):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        procs = mp.start_processes(_ar_worker, args=(world, f"{d}/store", dtype_name, proto), nprocs=world,
                                   join=False, start_method="spawn")
        deadline = time.time() + 180
        while time.time() < deadline and not all(p.exitcode is not None for p in procs.processes):
            time.sleep(0.2)
        for p in procs.processes:
            if p.is_alive():
                p.terminate()
        for p in procs.processes:
            p.join()
        assert [p.exitcode for p in procs.processes] == [0] * world


def test_peer_all_reduce_2_bf16():
    _run_ar(2, "bfloat16")


def test_peer_all_reduce_2_bf16_two_shot():
    _run_ar(2, "bfloat16", "two_shot")


def test_peer_all_reduce_4_bf16_two_shot():
    _run_ar(4, "bfloat16", "two_shot")


def test_peer_all_reduce_8_bf16_two_shot():
    _run_ar(8, "bfloat16", "two_shot")


def test_peer_all_reduce_8_bf16_one_shot():
    _run_ar(8, "bfloat16", "one_shot")


def test_peer_all_reduce_2_fp32():
    _run_ar(2, "float32")


def test_peer_all_reduce_8_bf16():
    _run_ar(8, "bfloat16")


def _far_worker(rank, world, store):
    """Row-parallel linear with the all-reduce fused into the GEMM epilogue:
    every rank holds its own K slice of x and W; the result must equal the
    rank-ordered fp32 sum of the ranks' rounded partials (each partial computed
    by the same kernel without the exchange), rounded, plus the residual."""
    import os

    from forgeml_b200 import _native
    from forgeml_b200.linear import PackedLinear
    from forgeml_b200.nebula import ParallelContext
    from forgeml_b200.nebula.peer import PeerAllReduce

    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    ctx = ParallelContext.from_env(tp_size=world, pp_size=1, device="cuda", timeout_s=60)
    dev = ctx.device
    bf = torch.bfloat16
    ar = PeerAllReduce(ctx, max_bytes=4096 * 64)
    try:
        for it, (n, k_total, m) in enumerate(((2048, 2048, 32), (2048, 8192, 32), (4096, 4096, 7), (2048, 2048, 1))):
            k = k_total // world
            g = torch.Generator().manual_seed(100 * it + rank)
            w = (torch.randn(n, k, generator=g) * 0.02).to(bf).to(dev)
            x = torch.randn(m, k, generator=g).to(bf).to(dev)
            res = torch.randn(m, n, generator=torch.Generator().manual_seed(9 + it)).to(bf).to(dev)  # same on all ranks
            lin = PackedLinear(w)
            assert lin.fused_ok(m)
            part = lin.fused(x, torch.empty(m, n, dtype=bf, device=dev)).cpu()
            parts = [None] * world
            dist.all_gather_object(parts, part)
            acc = torch.zeros(m, n, dtype=torch.float32)
            for p in parts:  # rank order, fp32
                acc += p.float()
            want = (acc.to(bf).float() + res.cpu().float()).to(bf)
            for _ in range(2):
                got = lin.fused(x, torch.empty(m, n, dtype=bf, device=dev), residual=res, ar_ctx=ar.handle)
                assert torch.equal(got.cpu(), want), f"rank {rank} case {it}"
            got = lin.fused(x, torch.empty(m, n, dtype=bf, device=dev), ar_ctx=ar.handle)
            assert torch.equal(got.cpu(), acc.to(bf))
        # CUDA-graph replay (epochs advance on the device)
        n, k, m = 2048, 2048 // world, 32
        w = torch.zeros((n, k), dtype=bf, device=dev)
        w[:, 0] = 1.0
        x = torch.zeros(m, k, dtype=bf, device=dev)
        x[:, 0] = float(rank + 1)
        lin = PackedLinear(w)
        res = torch.ones(m, n, dtype=bf, device=dev)
        out = torch.empty(m, n, dtype=bf, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            lin.fused(x, out, residual=res, ar_ctx=ar.handle)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            lin.fused(x, out, residual=res, ar_ctx=ar.handle)
        for _ in range(5):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.all(out.float() == 1 + world * (world + 1) / 2)
        del graph
        assert _native.device_status() == 0
    finally:
        ar.close()
        torch.cuda.synchronize()
        dist.barrier()
        ctx.close()
        if dist.is_initialized():
            dist.destroy_process_group()


def _run_far(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        procs = mp.start_processes(_far_worker, args=(world, f"{d}/store"), nprocs=world, join=False,
                                   start_method="spawn")
        deadline = time.time() + 180
        while time.time() < deadline and not all(p.exitcode is not None for p in procs.processes):
            time.sleep(0.2)
        for p in procs.processes:
            if p.is_alive():
                p.terminate()
        for p in procs.processes:
            p.join()
        assert [p.exitcode for p in procs.processes] == [0] * world


def test_fused_all_reduce_linear_2():
    _run_far(2)


def test_fused_all_reduce_linear_8():
    _run_far(8)
