"""Benchmark: Nebula greedy-decode tokens/s (config 4) on the sm_100a kernels.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

Workload: 12-layer pre-LN decoder, d_model 2048, 16 heads
x 128, FFN 8192 tanh-GELU, vocab 32000, max context 2048, weights ~ N(0,0.02)
(seed 3), bf16; batch of 32 prompts x 512 token ids uniform in [0, 32000)
(seeded); tensor parallel degree = N (one process per GPU, NCCL).  A "step" is
one greedy decode step of the whole batch (32 tokens).  Prefill runs before
the timed region; the W warm-up steps and K timed steps continue the same
sequences (context 513 .. 512+W+K).  Every step streams > 3 GB of weights and
KV cache, far more than the 126 MB L2, so no flush is needed between steps.

JSON line keys (one line on rank 0):
  value        decode tokens/s, device-timed (CUDA events, max over ranks)
  e2e          the same metric through Engine.forward with the step's tokens
               copied from pinned host memory and the argmax ids read back
  generate     the workload's whole 128-token generation through
               Engine.generate (prefill + contexts 513..640), wall clock
  roofline     the decode step's dominant kernel family (HBM): algorithmic bytes /
               CUDA-event time of that family's launches replayed from a graph;
               roofline_other the other family, roofline_step the whole step
  parity       16 greedy steps of the full model checked before timing against
               the reference's TinyDecoder (fp32 CPU, bf16-rounded weights):
               max relative logit error, greedy agreement; failing exits 1
  budget       the step's time split among the GEMM, attention and (all ranks
               at once) TP all-reduce families
  gemm         fused linear+GELU GEMM TFLOP/s at 8192^3 bf16 (N=1), output
               rows checked against torch fp32
  forgeml      configs 1-3 on the native kernels: compiled MLP and encoder
               block, GEMM sweep (N=1)
  cpu_baseline the reference's own CPU implementation of the decode step (its
               Engine from baseline/_ref, fp32, all host cores; N=1), or the
               CPU oracle restatement when the reference is not installed
--impl reference times that CPU implementation alone (rank 0; other ranks exit 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

C4 = dict(vocab_size=32000, hidden_size=2048, num_heads=16, num_layers=12, intermediate_size=8192,
          max_seq_len=2048, seed=3)
BATCH, PROMPT, NEW_TOKENS = 32, 512, 128


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clocks", suffix=".csv")[1])

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # nvidia-smi takes a while to start (longer on an 8-GPU host): wait for
        # its first sample so that the timed region falls in its sampling
        self._lines_at_start = self._wait_lines(1, 3.0)
        return self

    def _lines(self) -> int:
        try:
            return sum(1 for line in self.path.read_text().splitlines() if line.strip())
        except OSError:
            return 0

    def _wait_lines(self, n: int, timeout: float) -> int:
        t0 = time.perf_counter()
        while self.proc is not None and self._lines() < n and time.perf_counter() - t0 < timeout:
            time.sleep(0.02)
        return self._lines()

    def __exit__(self, *exc):
        if self.proc is not None:
            # at least one sample taken after the timed region began
            self._wait_lines(self._lines_at_start + 1, 0.5)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in self.path.read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 7:
                    rows.append(parts)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][1]),
                "samples": len(rows), "reasons": reasons}


def cpu_oracle_decode(steps: int, warmup: int, threads: int, layers: int | None = None) -> dict:
    """Time the CPU oracle of the c4 decode step (fp32, torch CPU, all host cores).

    The sample: decode steps of the full batch at context 513+ over a KV cache
    prefilled with seeded random values (a real 512-token prefill would cost
    ~22 TFLOP on the CPU); weights ~ N(0,0.02) like the GPU arm.
    """
    from oracle import nebula as orc

    torch.set_num_threads(threads)
    cfg = dict(C4)
    nl = layers or cfg["num_layers"]
    h, f, v = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    g = torch.Generator().manual_seed(3)
    w = {"tok": torch.randn(v, h, generator=g) * 0.02, "pos": torch.randn(cfg["max_seq_len"], h, generator=g) * 0.02,
         "lnf_w": torch.ones(h), "lnf_b": torch.zeros(h), "head": torch.randn(v, h, generator=g) * 0.02}
    for i in range(nl):
        w[f"{i}.ln1_w"], w[f"{i}.ln1_b"] = torch.ones(h), torch.zeros(h)
        w[f"{i}.ln2_w"], w[f"{i}.ln2_b"] = torch.ones(h), torch.zeros(h)
        for name, shape in (("q", (h, h)), ("k", (h, h)), ("v", (h, h)), ("o", (h, h)), ("up", (f, h)), ("down", (h, f))):
            w[f"{i}.{name}"] = torch.randn(*shape, generator=g) * 0.02
    heads, hd = cfg["num_heads"], h // cfg["num_heads"]
    cap = PROMPT + warmup + steps + 1
    caches = [(torch.randn(BATCH, heads, cap, hd, generator=g), torch.randn(BATCH, heads, cap, hd, generator=g))
              for _ in range(nl)]
    tok = torch.randint(0, v, (BATCH, 1), generator=g)
    pos = PROMPT
    times = []
    for it in range(warmup + steps):
        t0 = time.perf_counter()
        logits = orc.forward(w, tok, heads, nl, caches=caches, start_pos=pos)
        tok = logits[:, -1].argmax(-1, keepdim=True)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
        pos += 1
    total = sum(times)
    scale = cfg["num_layers"] / nl
    return {"value": BATCH * len(times) / (total * scale), "unit": "tokens/s", "cores": threads,
            "seconds": total, "steps": len(times),
            "sample": f"{len(times)} decode steps, batch {BATCH}, context {PROMPT + warmup + 1}.."
                      f"{PROMPT + warmup + len(times)}, fp32 torch CPU oracle (oracle/nebula.py), "
                      f"{nl} of {cfg['num_layers']} layers timed and scaled, KV prefilled with random values"}


def reference_decode(steps: int, warmup: int, threads: int, layers: int | None = None) -> dict | None:
    """Time the reference's own CPU implementation of the c4 decode step.

    Runs the unmodified reference Engine (rayhankhilji/ForgeML's `nebula`,
    installed offline into baseline/_ref) on the host cores in fp32 (the
    reference refuses low precision on CPU, src/nebula/runtime.py:222-223).
    The sample: the full batch of 32 requests, KV cache filled to the prompt
    length through the reference's own KVCache.append with seeded random
    keys/values (a real 512-token prefill costs ~22 TFLOP on the CPU), then
    `steps` greedy decode steps through Engine.forward.  The context capacity
    (max_seq_len) is cut to what the sample needs: the reference preallocates
    it per request and layer, and per-step work does not depend on it.
    Returns None when the reference package is not importable.
    """
    ref_root = REPO / "baseline" / "_ref"
    if not (ref_root / "nebula").is_dir():
        return None
    saved_env = {k: os.environ.pop(k) for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK") if k in os.environ}
    sys.path.insert(0, str(ref_root))
    try:
        from nebula.model import DecoderConfig as RefConfig
        from nebula.parallel import ParallelContext as RefContext
        from nebula.runtime import Engine as RefEngine

        torch.set_num_threads(threads)
        nl = layers or C4["num_layers"]
        cfg = RefConfig(**{**C4, "num_layers": nl, "max_seq_len": PROMPT + warmup + steps + 8})
        torch.manual_seed(C4["seed"])
        engine = RefEngine(cfg, context=RefContext.from_env(device="cpu"), dtype=torch.float32, max_requests=BATCH)
        dec = engine.decoder
        ids = tuple(range(1, BATCH + 1))
        dec.cache.reserve(ids)
        g = torch.Generator().manual_seed(3)
        hl, hd = cfg.num_heads, cfg.hidden_size // cfg.num_heads
        for lid in dec.owned_layer_ids:
            dec.cache.append(lid, ids, torch.randn(BATCH, hl, PROMPT, hd, generator=g),
                             torch.randn(BATCH, hl, PROMPT, hd, generator=g), 0)
        tok = torch.randint(0, cfg.vocab_size, (BATCH, 1), generator=g)
        pos = PROMPT
        times = []
        with torch.inference_mode():
            for it in range(warmup + steps):
                t0 = time.perf_counter()
                logits = engine.forward(tok, ids, pos)
                tok = logits[:, -1].argmax(-1, keepdim=True)
                if it >= warmup:
                    times.append(time.perf_counter() - t0)
                pos += 1
        engine.close()
        total = sum(times)
        scale = C4["num_layers"] / nl
        return {"value": BATCH * len(times) / (total * scale), "unit": "tokens/s", "cores": threads,
                "seconds": total * scale, "steps": len(times), "kind": "reference",
                "sample": f"{len(times)} decode steps of the reference Engine (baseline/_ref, fp32 CPU), batch {BATCH}, "
                          f"context {PROMPT + warmup + 1}..{PROMPT + warmup + len(times)}, KV filled through the "
                          f"reference KVCache.append with random values"
                          + ("" if nl == C4["num_layers"] else f", {nl} of {C4['num_layers']} layers timed and scaled")}
    finally:
        sys.path.remove(str(ref_root))
        os.environ.update(saved_env)


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # a bounded sample of the workload: the reference's CPU step takes about a second
    steps = min(args.steps, 10)
    res = reference_decode(steps, min(args.warmup, 2), threads, layers=args.cpu_layers)
    if res is None:
        res = cpu_oracle_decode(steps, min(args.warmup, 2), threads, layers=args.cpu_layers) | {"kind": "port"}
    line = {
        "metric": "nebula_decode_tokens_per_s", "value": res["value"], "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": res["steps"], "warmup": args.warmup,
        "ms_per_step": 1000 * res["seconds"] / max(res["steps"], 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "nebula_c4_greedy_decode", "model": "12L d2048 h16x128 ffn8192 v32000",
                   "global_batch": BATCH, "prompt_len": PROMPT, "parallelism": f"cpu x{threads} threads"},
        "cpu_baseline": {"value": res["value"], "unit": "tokens/s", "cores": res["cores"], "kind": res["kind"],
                         "sample": res["sample"]},
        "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def gemm_headline(dev) -> dict:
    """Fused linear+GELU GEMM at 8192^3 bf16 (BASELINE config 3 headline shape)."""
    from forgeml_b200.forgeml import kernels
    from forgeml_b200.workloads import make_c3_operands

    m = n = k = 8192
    a, b, bias = make_c3_operands(m, n, k, torch.bfloat16, device=str(dev))
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        kernels.matmul(a, b, bias, activation="gelu", out=out)
    torch.cuda.synchronize()
    reps = 10
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        kernels.matmul(a, b, bias, activation="gelu", out=out)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    tf = 2 * m * n * k / (ms * 1e-3) / 1e12
    pk = _peaks()
    # the timed output, checked on 16 seeded rows against torch fp32 on the device
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(8))[:16].to(dev)
    want = torch.nn.functional.gelu((a[rows].float() @ b.float() + bias.float()).to(torch.bfloat16).float())
    got = out[rows].float()
    err = float(((got - want).abs() - 2e-2 * want.abs()).max())
    check = {"rows": 16, "vs": "torch fp32 matmul + bias + erf GELU on the device",
             "max_abs_err": float((got - want).abs().max()), "tol": "2e-2 rel + 2e-2 abs", "pass": err <= 2e-2}
    return {"shape": "8192x8192x8192 bf16 +bias +gelu(erf), B [K,N] N-major", "ms": ms, "tflops": tf,
            "peak_tflops": pk["bf16_tflops"], "frac": tf / pk["bf16_tflops"], "peak_source": pk["source"],
            "check": check}


def forgeml_cases(dev) -> dict:
    """ForgeML configs 1-3 on the native kernels (N=1, CUDA events, inputs
    resident on the device):
      c1  2-layer MLP, fp32 (3xTF32), compiled (fused_linear_gelu + linear)
      c2  pre-LN encoder block, fp32 and bf16, compiled (24-node graph)
      c3  GEMM + bias + GELU sweep: squares 256..8192 (bf16 and fp32) and
          skinny M in {1, 16, 128} with N = K = 4096 (bf16, HBM-bound)."""
    from forgeml_b200.forgeml import compile as fml_compile
    from forgeml_b200.forgeml import kernels
    from forgeml_b200.workloads import make_c1_mlp, make_c2_block, make_c3_operands

    pk = _peaks()

    def timed_ms(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    def graph_ms(fn, reps):
        """Device time of one call replayed from a CUDA graph (no host dispatch)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return timed_ms(g.replay, reps)

    out = {}
    with torch.inference_mode():
        m, x = make_c1_mlp()
        c = fml_compile(m.to(dev), (x.to(dev),), backend="triton")
        xd = x.to(dev)
        ms = timed_ms(lambda: c(xd), 50)
        gms = graph_ms(lambda: c(xd), 50)
        out["c1_mlp_fp32"] = {"us_per_call": ms * 1e3, "device_us_per_call": gms * 1e3, "gflop": 0.268,
                              "tflops": 0.268e9 / (ms * 1e-3) / 1e12, "device_tflops": 0.268e9 / (gms * 1e-3) / 1e12}
        for dt, name in ((torch.float32, "c2_block_fp32"), (torch.bfloat16, "c2_block_bf16")):
            m, x = make_c2_block(dtype=dt)
            m = m.to(dev, dt)
            c = fml_compile(m, (x.to(dev),), backend="triton")
            xd = x.to(dev)
            ms = timed_ms(lambda: c(xd), 10)
            gms = graph_ms(lambda: c(xd), 10)
            out[name] = {"ms_per_call": ms, "gflop": 64.42, "tflops": 64.42e9 / (ms * 1e-3) / 1e12,
                         "device_ms_per_call": gms, "device_tflops": 64.42e9 / (gms * 1e-3) / 1e12,
                         "node_ms": {k: round(v, 4) for k, v in c.node_times(xd).items()},
                         "native_fusions": c.fusions}
        sweep = {}
        for dt, dn in ((torch.bfloat16, "bf16"), (torch.float32, "fp32")):
            for sz in (256, 1024, 4096, 8192):
                a, b, bias = make_c3_operands(sz, sz, sz, dt, device=str(dev))
                o = torch.empty(sz, sz, dtype=dt, device=dev)
                ms = timed_ms(lambda: kernels.matmul(a, b, bias, activation="gelu", out=o), 5 if sz == 8192 else 20)
                tf = 2 * sz ** 3 / (ms * 1e-3) / 1e12
                sweep[f"{dn}_{sz}^3"] = {"ms": ms, "tflops": tf, "frac_of_bf16_peak": tf / pk["bf16_tflops"]}
        for mm in (1, 16, 128):
            a, b, bias = make_c3_operands(mm, 4096, 4096, torch.bfloat16, transposed_b=True, device=str(dev))
            o = torch.empty(mm, 4096, dtype=torch.bfloat16, device=dev)
            ms = timed_ms(lambda: kernels.matmul(a, b, bias, activation="gelu", out=o), 50)
            gms = graph_ms(lambda: kernels.matmul(a, b, bias, activation="gelu", out=o), 50)
            nbytes = (4096 * 4096 + mm * 4096 * 2 + 4096) * 2
            sweep[f"bf16_m{mm}_n4096_k4096"] = {"us": ms * 1e3, "GB/s": nbytes / (ms * 1e-3) / 1e9,
                                                "frac_of_hbm": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                                                "device_us": gms * 1e3,
                                                "device_frac_of_hbm": nbytes / (gms * 1e-3) / 1e9 / pk["hbm_gbs"]}
        out["c3_sweep"] = sweep
    out["reference_cpu"] = reference_forgeml_cpu()
    return out


def reference_forgeml_cpu() -> dict | None:
    """The reference's own compiled forward on the host cores (its
    `compile(..., backend="torch")` from baseline/_ref, fp32, all threads) for
    configs 1 and 2: the CPU baseline beside the native numbers."""
    ref_root = REPO / "baseline" / "_ref"
    if not (ref_root / "forgeml").is_dir():
        return None
    from forgeml_b200.workloads import make_c1_mlp, make_c2_block

    sys.path.insert(0, str(ref_root))
    try:
        import forgeml as ref_forgeml

        torch.set_num_threads(os.cpu_count() or 1)
        res = {"cores": os.cpu_count() or 1, "kind": "reference"}
        with torch.inference_mode():
            for name, (m, x), reps in (("c1_mlp_fp32", make_c1_mlp(), 20), ("c2_block_fp32", make_c2_block(), 3)):
                c = ref_forgeml.compile(m, (x,), backend="torch")
                c(x)
                t0 = time.perf_counter()
                for _ in range(reps):
                    c(x)
                res[name + "_ms"] = (time.perf_counter() - t0) / reps * 1e3
        return res
    finally:
        sys.path.remove(str(ref_root))


# DRAM traffic per launch over the algorithmic bytes, from the ncu captures
# summarised under profiles/ (dram__bytes_read.sum + dram__bytes_write.sum of
# each captured launch / its algorithmic bytes):
#   attention: neb_attn_bulk_kernel_b32_ctx1024.md
#              (ncu --set full --clock-control none -k regex:neb_attn ... bench.py --case attention)
#   gemm:      gemm_kernel_decode_fused_m32_tp1_tp8.md, the four TP1 launches
#              (ncu --set full --clock-control none -k regex:gemm_kernel ... bench.py --case gemm-fused --tp 1)
# Traffic in the JSON line is this ratio times the launch's algorithmic bytes.
TRAFFIC_RATIO = {"attention": (268.618240e6 + 4.372736e6) / 268697600,
                 "gemm": (33.801216 + 34.293248 + 25.405184 + 8.734208) / (34.209792 + 34.340864 + 25.690112 + 8.781824)}


def _graph_time_us(fns, reps: int = 5) -> float:
    """Device time per call of `fns` replayed from one CUDA graph (CUDA events
    on the replay stream, best of `reps` replays)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e3)
    del g
    return best


def _step_lanes(dec, b: int) -> list[int]:
    """Rows of each batch lane a decode step of ``b`` requests runs."""
    return dec._lanes(b, 1)


def all_reduce_family_us(dec, dev, world: int) -> dict | None:
    """Device time of one decode step's TP all-reduces (2 per layer and lane,
    [rows, d] each, + residual) replayed from a CUDA graph on every rank at
    once (max over ranks).  Collective: every rank calls it."""
    import torch.distributed as dist

    if world == 1 or dec._peer_ar is None:
        return None
    h = dec.config.hidden_size
    calls = []
    for rows in _step_lanes(dec, BATCH):
        part = torch.randn(rows, h, device=dev).to(dec.dtype)
        res = torch.randn(rows, h, device=dev).to(dec.dtype)
        out = torch.empty_like(part)
        calls += [lambda p=part, r=res, o=out: dec._peer_ar(p, r, o)] * (2 * len(dec.layers))
    dist.barrier()
    us = _graph_time_us(calls)
    t = torch.tensor([us], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())
    return {"kernel": "ar_ll_kernel / ar_ts_kernel (peer all-reduce + residual)", "us_per_step": us,
            "launches_per_step": len(calls), "us_per_launch": us / len(calls),
            "bytes_out_per_rank_per_launch": (world - 1) * (BATCH // len(_step_lanes(dec, BATCH))) * h * 2}


def kernel_rooflines(engine, dev, ctx_len: int, ms_per_step: float, ar_family: dict | None = None) -> dict:
    """HBM rooflines of the decode step's kernel families, each timed live
    with CUDA events as one step's launches of that family replayed from a
    CUDA graph on the engine's own weights and cache pools:
      gemm       gemm_kernel as the step runs it: per layer the LayerNorm-
                 folded QKV launch with the KV-append epilogue, o (+ residual
                 at TP1), the LayerNorm-folded up launch with tanh GELU, down
                 (+ residual at TP1); then lm_head.  Per batch lane when
                 the step is split.  Algorithmic bytes = weights + activations
                 in + outputs (K/V rows included) (+ residual)
      attention  neb_attn_bulk_kernel, one launch per layer and lane at the
                 step's context; algorithmic bytes = K + V rows + q + out
    The family with the larger share of the step is reported as `roofline`;
    `budget` splits the step's time among the families (they overlap when
    the step runs two lanes, so the remainder can be negative)."""
    from forgeml_b200.nebula import ops
    from forgeml_b200 import _native

    dec = engine.decoder
    es = torch.empty((), dtype=dec.dtype).element_size()
    h = dec.config.hidden_size
    hl_hd = dec.num_heads_local * dec.head_dim
    tp1 = dec.context.tp_size == 1
    g = torch.Generator(device=dev).manual_seed(11)
    lanes = _step_lanes(dec, BATCH)

    def rnd(*shape):
        return torch.randn(*shape, device=dev, generator=g).to(dec.dtype)

    # ---- GEMM family: one decode step's linears, as launched by the step
    fns, gbytes = [], 0
    scratch_pos = min(ctx_len, dec.config.max_seq_len - 1)  # KV rows written past the timed context
    for b in lanes:
        x, attn = rnd(b, h), rnd(b, hl_hd)
        slots = torch.arange(b, dtype=torch.int32, device=dev)
        starts = torch.full((b,), scratch_pos, dtype=torch.int32, device=dev)
        for L, lid in zip(dec.layers, dec.owned_layer_ids):
            f_l = L.wup.shape[0]
            q_out, o_out, up_out, dn_out = (torch.empty(b, n, device=dev, dtype=dec.dtype)
                                            for n in (hl_hd, h, f_l, h))
            mid = rnd(b, f_l)
            res = x if tp1 else None
            kp, vp = dec.cache.k_pool[lid], dec.cache.v_pool[lid]
            (qlin, qs, qb), (ulin, us_, ub) = L.qkv_ln, L.up_ln
            fns += [lambda q=qlin, o=q_out, ws=qs, wb=qb, kp=kp, vp=vp, sl=slots, st=starts:
                    q.fused(x, o, ln_fold=(ws, wb, 1e-5), kv=(kp, vp, sl, st, hl_hd, 1)),
                    lambda L=L, o=o_out, r=res: L.o(attn, o, residual=r),
                    lambda u=ulin, o=up_out, ws=us_, wb=ub: u.fused(x, o, act=_native.ACT_GELU_TANH,
                                                                     ln_fold=(ws, wb, 1e-5)),
                    lambda L=L, o=dn_out, m=mid, r=res: L.down(m, o, residual=r)]
            for w, n_in, n_out, r in ((L.wqkv, h, 3 * hl_hd, 0), (L.wo, hl_hd, h, res is not None),
                                      (L.wup, h, f_l, 0), (L.wdown, f_l, h, res is not None)):
                gbytes += (w.numel() + b * n_in + b * n_out * (2 if r else 1)) * es
    if dec.is_last:  # once per step for the whole batch
        xh = rnd(BATCH, h)
        head_out = torch.empty(BATCH, dec.config.vocab_size, device=dev, dtype=dec.dtype)
        fns.append(lambda: dec.head_gemm(xh, head_out))
        gbytes += (dec.head.numel() + BATCH * h + BATCH * dec.config.vocab_size) * es
    g_us = _graph_time_us(fns)
    n_g = len(fns)

    # ---- attention family: one launch per layer at the step's context
    hl, hd = dec.num_heads_local, dec.head_dim
    afns, abytes, row0 = [], 0, 0
    for b in lanes:
        q = rnd(b, 1, hl, hd)
        slots = torch.arange(row0, row0 + b, dtype=torch.int32, device=dev)
        starts = torch.full((b,), ctx_len - 1, dtype=torch.int32, device=dev)
        aout = torch.empty(b, 1, hl * hd, device=dev, dtype=dec.dtype)
        afns += [lambda lid=lid, q=q, sl=slots, st=starts, o=aout:
                 ops.attention(q, dec.cache.k_pool[lid], dec.cache.v_pool[lid], sl, st, o)
                 for lid in dec.owned_layer_ids]
        abytes += len(dec.owned_layer_ids) * b * hl * (2 * ctx_len * hd + 2 * hd) * es
        row0 += b
    a_us = _graph_time_us(afns)

    pk_ = _peaks()
    peak = pk_["hbm_gbs"]

    def entry(kernel, us, nbytes, launches, family, **more):
        ach = nbytes / (us * 1e-6) / 1e9
        per_launch = nbytes / launches
        ratio = TRAFFIC_RATIO.get(family)
        return {"kernel": kernel, "bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                "peak_source": pk_["source"], "traffic": (ratio * per_launch) if ratio else None,
                "algorithmic_bytes_per_launch": per_launch, "us_per_launch": us / launches,
                "launches_per_step": launches, "us_per_step": us, **more}

    gemm = entry("gemm_kernel (decode linears: qkv/o/up/down x layers + lm_head)", g_us, gbytes, n_g, "gemm")
    att = entry("neb_attn_bulk_kernel (decode attention over the KV pool)", a_us, abytes, len(afns), "attention",
                context=ctx_len)
    step_bytes = gbytes + abytes
    fam_us = g_us + a_us + (ar_family["us_per_step"] if ar_family else 0.0)
    budget = {"step_us": ms_per_step * 1e3, "gemm_us": g_us, "attention_us": a_us,
              "all_reduce_us": ar_family["us_per_step"] if ar_family else 0.0,
              "rest_us": ms_per_step * 1e3 - fam_us, "lanes": len(lanes),
              "note": "families replayed one after another; a two-lane step overlaps them" if len(lanes) > 1
              else "families replayed one after another"}
    step = {"bound": "hbm", "bytes_per_step": step_bytes, "achieved": step_bytes / (ms_per_step * 1e-3) / 1e9,
            "peak": peak, "unit": "GB/s", "frac": step_bytes / (ms_per_step * 1e-3) / 1e9 / peak}
    dominant, other = (gemm, att) if g_us >= a_us else (att, gemm)
    out = {"roofline": dominant, "roofline_other": other, "roofline_step": step, "budget": budget}
    if ar_family:
        out["roofline_all_reduce"] = ar_family
    return out


def full_normal_weights(cfg, dev, dtype) -> dict:
    """The whole model of the synthetic initialisation (every rank's shards
    together) rounded to ``dtype``, as fp32 CPU tensors keyed like the
    reference TinyDecoder's state dict."""
    from forgeml_b200.nebula.model import normal_weight

    h = cfg.hidden_size

    def full(key):
        return normal_weight(cfg, key, dev).to(dtype).float().cpu()

    sd = {"token_embedding.weight": full("tok"), "position_embedding.weight": full("pos"),
          "lm_head.weight": full("head"), "final_norm.weight": torch.ones(h), "final_norm.bias": torch.zeros(h)}
    for i in range(cfg.num_layers):
        for n in ("q", "k", "v", "o", "up", "down"):
            sd[f"blocks.{i}.{n}.weight"] = full(f"{i}.{n}")
        for n in ("ln1", "ln2"):
            sd[f"blocks.{i}.{n}.weight"], sd[f"blocks.{i}.{n}.bias"] = torch.ones(h), torch.zeros(h)
    return sd


def reference_logits(cfg, state_dict: dict, tokens: torch.Tensor) -> tuple[torch.Tensor, str]:
    """Logits [B, T, V] of the whole model over ``tokens`` on the host cores in
    fp32: the reference's own TinyDecoder (baseline/_ref) loaded with
    ``state_dict``, or the CPU oracle restatement when the reference is not
    installed.  Returns (logits, which)."""
    ref_root = REPO / "baseline" / "_ref"
    torch.set_num_threads(os.cpu_count() or 1)
    if (ref_root / "nebula").is_dir():
        sys.path.insert(0, str(ref_root))
        try:
            from nebula.model import DecoderConfig as RefConfig
            from nebula.model import TinyDecoder as RefDecoder

            rc = RefConfig(**{f: getattr(cfg, f) for f in ("vocab_size", "hidden_size", "num_heads", "num_layers",
                                                            "intermediate_size", "max_seq_len", "seed")})
            with torch.device("meta"):
                model = RefDecoder(rc)
            model.load_state_dict(state_dict, assign=True)
            with torch.inference_mode():
                return model.eval()(tokens), "reference TinyDecoder (baseline/_ref), fp32 CPU"
        finally:
            sys.path.remove(str(ref_root))
    from oracle import nebula as orc

    w = orc.weights_from_state_dict(state_dict, cfg.num_layers)
    return orc.forward(w, tokens, cfg.num_heads, cfg.num_layers), "CPU oracle (oracle/nebula.py), fp32"


def decode_parity(dec, dev, *, batch: int = BATCH, prompt_len: int = 16, steps: int = 16, tol: float = 2e-2,
                  min_agree: float = 0.9, ids_base: int = 900, checker: bool = True) -> dict | None:
    """Greedy decode on the native decoder checked against the reference's
    own CPU forward.

    Every rank runs the same steps (SPMD: a prefill of ``batch`` seeded
    prompts of ``prompt_len`` tokens, then ``steps - 1`` single-token greedy
    steps through the decoder's own path, CUDA graphs and TP collectives
    included).  On the checking rank the whole model then runs in fp32 on the
    host (reference_logits) with the bf16-rounded weights over the same token
    sequence (teacher-forced with the engine's own greedy tokens), and the
    logits of every step are compared:
      max_rel_err   max |got - want| / max |want| over the step's logits
      greedy_agree  fraction of (request, step) whose argmax agrees
    Returns the summary on the checking rank, None elsewhere."""
    from forgeml_b200.nebula import ops

    cfg = dec.config
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(0, cfg.vocab_size, (batch, prompt_len), generator=g)
    ids = tuple(range(ids_base, ids_base + batch))
    got, toks = [], []
    with torch.inference_mode():
        logits = dec.forward(prompts.to(dev), ids, 0, last_only=True)
        for s_ in range(steps):
            if s_:
                logits = dec.forward(toks[-1].view(-1, 1), ids, prompt_len + s_ - 1, last_only=True)
            got.append(logits[:, -1].float().cpu())
            toks.append(ops.argmax(logits[:, -1]))
        dec.cache.release(ids)
    torch.cuda.synchronize(dev)
    if not checker:
        return None
    t0 = time.perf_counter()
    sd = full_normal_weights(cfg, dev, dec.dtype)
    seq = torch.cat([prompts, torch.stack([t.cpu() for t in toks[:-1]], 1)], 1)
    want_all, which = reference_logits(cfg, sd, seq)
    del sd
    errs, agree = [], []
    for s_ in range(steps):
        want = want_all[:, prompt_len - 1 + s_].float()
        errs.append(float((got[s_] - want).abs().max() / want.abs().max()))
        agree.append((got[s_].argmax(-1) == want.argmax(-1)).float().mean().item())
    rel, ag = max(errs), sum(agree) / len(agree)
    return {"max_rel_err": rel, "greedy_agree": ag, "tol": f"{tol:g}", "min_agree": min_agree,
            "steps": steps, "batch": batch, "prompt_len": prompt_len, "layers": cfg.num_layers,
            "vs": which + " on the bf16-rounded weights, teacher-forced with the engine's greedy tokens",
            "check_s": time.perf_counter() - t0, "pass": bool(rel <= tol and ag >= min_agree)}


def run_native(args) -> None:
    import torch.distributed as dist

    from forgeml_b200 import _native
    from forgeml_b200.nebula import DecoderConfig, Engine, ParallelContext
    from forgeml_b200.nebula import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    ctx = ParallelContext.from_env(tp_size=world, pp_size=1, device="cuda", timeout_s=120.0)
    dev = ctx.device
    rank = ctx.rank
    cfg = DecoderConfig(**C4)
    engine = Engine(cfg, context=ctx, dtype=torch.bfloat16, max_requests=BATCH, init="normal")
    dec = engine.decoder
    g = torch.Generator().manual_seed(C4["seed"])
    prompts = torch.randint(0, cfg.vocab_size, (BATCH, PROMPT), generator=g)
    ids = tuple(range(100, 100 + BATCH))
    W, K = args.warmup, args.steps
    if PROMPT + W + K + 2 > cfg.max_seq_len:
        raise SystemExit("warmup + steps exceed the context capacity")

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    # ---- parity before the timed region: the full model at this N against the CPU oracle
    parity = None
    if not args.no_parity:
        parity = decode_parity(dec, dev, checker=rank == 0)
        sync_all()

    # ---- device-timed decode (SPMD: every rank runs the same steps) ----
    with torch.inference_mode():
        logits = dec.forward(prompts.to(dev), ids, 0, last_only=True)
        nxt = ops.argmax(logits[:, -1, :])
        pos = PROMPT
        launches0 = _native.launch_count()
        for _ in range(W):
            logits = dec.forward(nxt.view(-1, 1), ids, pos, last_only=True)
            nxt = ops.argmax(logits[:, -1, :])
            pos += 1
        per_step_launches = None
        sync_all()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(dev.index) as clk:
            sync_all()
            ev0.record()
            for _ in range(K):
                logits = dec.forward(nxt.view(-1, 1), ids, pos, last_only=True)
                nxt = ops.argmax(logits[:, -1, :])
                pos += 1
            ev1.record()
            sync_all()
        ms = ev0.elapsed_time(ev1)
        # native launches per step: a captured step replays the kernels counted at capture
        graphed = dec.use_cuda_graphs and ctx.pp_size == 1
        if graphed:
            n0 = _native.launch_count()
            dec._graphs.clear()
            logits = dec.forward(nxt.view(-1, 1), ids, pos, last_only=True)  # recapture counts its kernels
            per_step_launches = (_native.launch_count() - n0) // 2 + 1  # eager warm-up + capture, + argmax
            nxt = ops.argmax(logits[:, -1, :])
            pos += 1
        else:
            n0 = _native.launch_count()
            logits = dec.forward(nxt.view(-1, 1), ids, pos, last_only=True)
            nxt = ops.argmax(logits[:, -1, :])
            per_step_launches = _native.launch_count() - n0
            pos += 1
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        value = BATCH * K / (ms * 1e-3)
        dec.cache.release(ids)
        torch.cuda.synchronize(dev)

    # ---- TP all-reduce family, every rank at once (before the leader drives e2e)
    with torch.inference_mode():
        ar_family = all_reduce_family_us(dec, dev, world)

    # ---- end-to-end through the public Engine API (host tokens in, ids out) ----
    # Rank 0 drives the engine (it broadcasts the reference command protocol);
    # the other ranks serve until the leader's STOP at engine.close().
    e2e = None
    if rank == 0:
        with torch.inference_mode():
            host_tok = torch.empty(BATCH, 1, dtype=torch.long).pin_memory()
            host_out = torch.empty(BATCH, dtype=torch.long).pin_memory()
            logits = engine.forward(prompts, ids, 0, _internal=True, _last_only=True)
            host_out.copy_(ops.argmax(logits[:, -1, :]))
            pos = PROMPT
            for _ in range(W):
                host_tok.copy_(host_out.view(-1, 1))
                logits = engine.forward(host_tok, ids, pos, _internal=True, _last_only=True)
                host_out.copy_(ops.argmax(logits[:, -1, :]))
                pos += 1
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(K):
                host_tok.copy_(host_out.view(-1, 1))
                logits = engine.forward(host_tok, ids, pos, _internal=True, _last_only=True)
                host_out.copy_(ops.argmax(logits[:, -1, :]))  # device->host read of the step's result
                pos += 1
            torch.cuda.synchronize(dev)
            e2e_s = time.perf_counter() - t0
            engine.release(ids)
            # the workload's whole generation: prefill of every prompt, then
            # NEW_TOKENS greedy steps over contexts PROMPT+1 .. PROMPT+NEW_TOKENS
            host_prompts = prompts.tolist()
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            outs = engine.generate(host_prompts, NEW_TOKENS)
            gen_s = time.perf_counter() - t0
        e2e = {"value": BATCH * K / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": BATCH * 8,
               "d2h_bytes_per_step": BATCH * 8,
               "path": "Engine.forward(host int64 tokens) + native argmax + D2H ids, per step"
                       + ("" if world == 1 else "; leader drives workers through the command protocol")}
        generate = {"tokens_per_s": sum(len(o) for o in outs) / gen_s, "wall_s": gen_s, "new_tokens": NEW_TOKENS,
                    "batch": BATCH, "context": [PROMPT + 1, PROMPT + NEW_TOKENS],
                    "path": "Engine.generate(host prompts): prefill of every prompt + greedy decode, wall clock"}
    else:
        engine.serve()

    extra = {}
    if rank == 0:
        extra["generate"] = generate
    if rank == 0:
        with torch.inference_mode():
            extra.update(kernel_rooflines(engine, dev, PROMPT + W + K, ms / K, ar_family))
        if world == 1 and not args.no_gemm:
            extra["gemm"] = gemm_headline(dev)
            extra["forgeml"] = forgeml_cases(dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = reference_decode(args.cpu_steps, 1, os.cpu_count() or 1, layers=args.cpu_layers)
        if cpu is None:
            cpu = cpu_oracle_decode(args.cpu_steps, 1, os.cpu_count() or 1, layers=args.cpu_layers) | {"kind": "port"}
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "sample", "kind")}
    if rank == 0:
        line = {
            "metric": "nebula_decode_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "nebula_c4_greedy_decode", "model": "12L d2048 h16x128 ffn8192 v32000",
                       "global_batch": BATCH, "prompt_len": PROMPT, "context": [PROMPT + W + 1, PROMPT + W + K],
                       "parallelism": f"tp{world}", "cuda_graph": bool(dec.use_cuda_graphs and ctx.pp_size == 1),
                       "l2": "inputs larger than L2 (>3 GB streamed per step)"},
            "e2e": e2e, "gpu_launches": int(per_step_launches * K), "clocks": clk.summary(),
            "cpu_baseline": cpu, "parity": parity, **extra,
        }
        print(json.dumps(line), flush=True)
    if rank == 0:
        engine.close()  # sends STOP to the serving workers
    else:
        engine.close()
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier()
        ctx.close()
    if rank == 0 and parity is not None and not parity["pass"]:
        raise SystemExit(f"decode parity failed: {parity}")


C5 = dict(vocab_size=32000, hidden_size=4096, num_heads=32, num_layers=32, intermediate_size=16384,
          max_seq_len=4096, seed=4)


def run_c5(args) -> None:
    """Config 5: 32-layer d4096 decoder, TP x PP over the launched ranks (TP4 x
    PP2 on 8 GPUs), served through the AsyncBatcher (batch cap 64).  Requests
    arrive Poisson at 64 req/s with prompt lengths uniform in [128, 2048] and
    uniform token ids (seeded); the sample is --c5-requests requests of
    --c5-new tokens each (256 x 256 in the full workload).  Rank 0 drives the
    batcher; the other ranks serve.  Metric: generated tokens per second of
    wall time from the first arrival to the last completion."""
    import asyncio
    import random

    import torch.distributed as dist

    from forgeml_b200.nebula import AsyncBatcher, DecoderConfig, Engine, ParallelContext

    from forgeml_b200.nebula.runtime import ShardedDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    pp = 2 if world % 2 == 0 and world >= 2 else 1
    tp = world // pp
    ctx = ParallelContext.from_env(tp_size=tp, pp_size=pp, device="cuda", timeout_s=300.0)
    # parity first, on a 2-layer slice of the config-5 geometry over the same
    # TP x PP layout (the full 32-layer model is too large for the CPU check)
    parity = None
    if not args.no_parity:
        slice_cfg = DecoderConfig(**{**C5, "num_layers": 2 * pp})
        dec = ShardedDecoder(slice_cfg, ctx, dtype=torch.bfloat16, max_requests=8, init="normal")
        parity = decode_parity(dec, ctx.device, batch=8, prompt_len=16, steps=8, checker=ctx.rank == 0)
        dec.close()
        del dec
        torch.cuda.synchronize()
        dist.barrier()
    cfg = DecoderConfig(**C5)
    engine = Engine(cfg, context=ctx, dtype=torch.bfloat16, max_requests=64, init="normal")
    if ctx.rank != 0:
        engine.serve()
        engine.close()
        torch.cuda.synchronize()
        dist.barrier()
        ctx.close()
        return
    rng = random.Random(C5["seed"])
    n_req, n_new = args.c5_requests, args.c5_new
    prompts = [[rng.randrange(cfg.vocab_size) for _ in range(rng.randint(128, 2048))] for _ in range(n_req)]
    gaps = [rng.expovariate(64.0) for _ in range(n_req)]

    async def drive():
        # prompts of different lengths share decode batches (Engine.generate_mixed);
        # --c5-cohorts keeps the reference's equal-length cohorts instead
        b = AsyncBatcher(engine, max_batch_size=64, max_queue_size=n_req + 1, batch_window_ms=args.c5_window_ms,
                         mix_prompt_lengths=not args.c5_cohorts)
        lat = []

        async def one(i, delay):
            await asyncio.sleep(delay)
            t0 = time.perf_counter()
            toks = await b.submit(prompts[i], n_new)
            lat.append(time.perf_counter() - t0)
            return len(toks)

        t_start = time.perf_counter()
        delays, acc = [], 0.0
        for g_ in gaps:
            acc += g_
            delays.append(acc)
        counts = await asyncio.gather(*(one(i, d) for i, d in enumerate(delays)))
        wall = time.perf_counter() - t_start
        await b.close()  # closes the engine (STOP to the serving ranks)
        return sum(counts), wall, sorted(lat)

    # warm-up: one short request (captures nothing for PP, loads kernels)
    engine.generate([prompts[0][:128]], 4)
    total, wall, lat = asyncio.run(drive())
    line = {"metric": "nebula_c5_serving_tokens_per_s", "value": total / wall, "unit": "tokens/s", "n_gpus": world,
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "nebula_c5_async_batcher", "model": "32L d4096 h32x128 ffn16384 v32000",
                       "parallelism": f"tp{tp}xpp{pp}", "requests": n_req, "new_tokens": n_new,
                       "arrivals": "poisson 64 req/s (seeded)", "prompt_len": "uniform [128, 2048]",
                       "batch_cap": 64, "batching": "equal-length cohorts" if args.c5_cohorts
                       else "mixed prompt lengths (generate_mixed)", "window_ms": args.c5_window_ms},
            "wall_s": wall, "generated_tokens": total, "parity": parity,
            "latency_s": {"p50": lat[len(lat) // 2], "p90": lat[int(len(lat) * 0.9)], "max": lat[-1]}}
    print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    ctx.close()


def run_case(args) -> None:
    """Single-kernel micro-benchmarks on small device footprints (for ncu captures).

    attention    decode attention, batch 32 x 16 heads x 128, context 1024,
                 one layer's KV pool (268 MB, > L2)
    gemm-decode  the c4 decode GEMMs at batch 32 on pre-packed weights (the
                 engine's path): QKV 6144x2048, o 2048x2048 (+residual),
                 up 8192x2048 (+tanh GELU), down 2048x8192 (+residual),
                 lm_head 32000x2048; chains replayed from a CUDA graph
    gemm-fused   the decode step's fused launches at batch 32 for the TP
                 shard of --tp ranks: LayerNorm-folded QKV + KV append, o,
                 folded up + tanh GELU, down (residuals at TP1)
    gemm-l2      the c4 decode GEMMs at batch 32 as fused launches with the
                 residual epilogue, 20 launches replayed from a CUDA graph on
                 one L2-resident weight ("warm") and on 20 copies of it
                 ("cold", 20 x the bytes > L2): how much a launch depends on
                 where its weights come from
    gemm         8192^3 bf16 + bias + GELU
    c2           the compiled config-2 encoder block (bf16, then fp32): every
                 instruction's device time alone and the whole call
    """
    from forgeml_b200.forgeml import kernels
    from forgeml_b200.nebula import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    reps = args.steps
    res = {}

    g = torch.Generator(device=dev).manual_seed(0)
    if args.case == "attention":
        b, h, d, ctx = BATCH, 16, 128, 1024
        kp = torch.randn(b, h, ctx, d, device=dev, generator=g).to(torch.bfloat16)
        vp = torch.randn(b, h, ctx, d, device=dev, generator=g).to(torch.bfloat16)
        q = torch.randn(b, 1, h, d, device=dev, generator=g).to(torch.bfloat16)
        slots = torch.arange(b, dtype=torch.int32, device=dev)
        starts = torch.full((b,), ctx - 1, dtype=torch.int32, device=dev)
        out = torch.empty(b, 1, h * d, device=dev, dtype=torch.bfloat16)
        us = _graph_time_us([lambda: ops.attention(q, kp, vp, slots, starts, out)] * reps) / reps
        algo = b * h * (2 * ctx * d + 2 * d) * 2
        res["attention"] = {"us": us, "GB/s": algo / (us * 1e-6) / 1e9, "algo_bytes": algo}
    elif args.case == "gemm-decode":
        from forgeml_b200.linear import PackedLinear
        m = BATCH
        for name, n, k, act, resid in (("qkv", 6144, 2048, 0, False), ("o", 2048, 2048, 0, True),
                                       ("up", 8192, 2048, 2, False), ("down", 2048, 8192, 0, True),
                                       ("lm_head", 32000, 2048, 0, False)):
            # enough weight copies that the replayed chain streams > L2 from HBM
            copies = max(2, min(reps, int(400e6 // (n * k * 2)) + 1))
            ws = [PackedLinear((torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16))
                  for _ in range(copies)]
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            r = torch.randn(m, n, device=dev, generator=g).to(torch.bfloat16) if resid else None
            out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
            us = _graph_time_us([lambda w=ws[i % copies]: w(x, out, act, r) for i in range(reps)]) / reps
            algo = (n * k + m * k + m * n * (2 if resid else 1)) * 2
            res[name] = {"us": us, "GB/s": algo / (us * 1e-6) / 1e9, "algo_bytes": algo}
            del ws
    elif args.case == "gemm-fused":
        # the decode step's fused launches at batch 32 for one TP shard
        # (--tp): LayerNorm-folded QKV + KV append, o (+ residual), folded up
        # + tanh GELU, down (+ residual); enough layers' weights that the
        # replayed chain streams more than L2 from HBM
        from forgeml_b200.linear import PackedLinear, ln_fold_vectors

        tp = args.tp
        m, hdim, hd = BATCH, C4["hidden_size"], 128
        hl_hd, f_l = hdim // tp, C4["intermediate_size"] // tp
        heads = hl_hd // hd
        bf = torch.bfloat16
        layer_bytes = (3 * hl_hd * hdim + hdim * hl_hd + 2 * f_l * hdim) * 2
        n_layers = max(2, int(400e6 // layer_bytes) + 1)
        ones, zeros = torch.ones(hdim, device=dev, dtype=bf), torch.zeros(hdim, device=dev, dtype=bf)
        kp = torch.zeros(m, heads, 64, hd, device=dev, dtype=bf)
        vp = torch.zeros_like(kp)
        slots = torch.arange(m, dtype=torch.int32, device=dev)
        starts = torch.full((m,), 7, dtype=torch.int32, device=dev)
        x = torch.randn(m, hdim, device=dev, generator=g).to(bf)
        attn = torch.randn(m, hl_hd, device=dev, generator=g).to(bf)
        mid = torch.randn(m, f_l, device=dev, generator=g).to(bf)
        q_out, o_out = torch.empty(m, hl_hd, device=dev, dtype=bf), torch.empty(m, hdim, device=dev, dtype=bf)
        up_out, dn_out = torch.empty(m, f_l, device=dev, dtype=bf), torch.empty(m, hdim, device=dev, dtype=bf)
        fns = {"qkv_ln_kv": [], "o": [], "up_ln_gelu": [], "down": []}
        for _ in range(n_layers):
            wq = (torch.randn(3 * hl_hd, hdim, device=dev, generator=g) * 0.02).to(bf)
            wu = (torch.randn(f_l, hdim, device=dev, generator=g) * 0.02).to(bf)
            wo = PackedLinear((torch.randn(hdim, hl_hd, device=dev, generator=g) * 0.02).to(bf))
            wd = PackedLinear((torch.randn(hdim, f_l, device=dev, generator=g) * 0.02).to(bf))
            (wqp, qs, qb), (wup, us_, ub) = ln_fold_vectors(wq, ones, zeros), ln_fold_vectors(wu, ones, zeros)
            ql, ul = PackedLinear(wqp), PackedLinear(wup)
            r = x if tp == 1 else None
            fns["qkv_ln_kv"].append(lambda ql=ql, qs=qs, qb=qb: ql.fused(x, q_out, ln_fold=(qs, qb, 1e-5),
                                                                          kv=(kp, vp, slots, starts, hl_hd, 1)))
            fns["o"].append(lambda wo=wo, r=r: wo(attn, o_out, residual=r))
            fns["up_ln_gelu"].append(lambda ul=ul, us_=us_, ub=ub: ul.fused(x, up_out, act=2,
                                                                             ln_fold=(us_, ub, 1e-5)))
            fns["down"].append(lambda wd=wd, r=r: wd(mid, dn_out, residual=r))
        resid = 1 if tp == 1 else 0
        algo = {"qkv_ln_kv": (3 * hl_hd * hdim + m * hdim + m * 3 * hl_hd) * 2,
                "o": (hdim * hl_hd + m * hl_hd + m * hdim * (1 + resid)) * 2,
                "up_ln_gelu": (f_l * hdim + m * hdim + m * f_l) * 2,
                "down": (hdim * f_l + m * f_l + m * hdim * (1 + resid)) * 2}
        chain = [f for i in range(n_layers) for k in fns for f in (fns[k][i],)]
        us_chain = _graph_time_us(chain * max(1, reps // n_layers)) / (len(chain) * max(1, reps // n_layers))
        for k, lst in fns.items():
            us = _graph_time_us(lst * max(1, reps // n_layers)) / (len(lst) * max(1, reps // n_layers))
            res[k] = {"us": us, "GB/s": algo[k] / (us * 1e-6) / 1e9, "algo_bytes": algo[k], "tp_shard": tp}
        res["chain_avg_us"] = us_chain
    elif args.case == "gemm-l2":
        from forgeml_b200.linear import PackedLinear

        m, n_copies = BATCH, 20
        for name, n, k in (("up", 8192, 2048), ("down", 2048, 8192), ("qkv", 6144, 2048), ("o", 2048, 2048)):
            ws = [PackedLinear((torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16))
                  for _ in range(n_copies)]
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            r = torch.randn(m, n, device=dev, generator=g).to(torch.bfloat16)
            out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
            warm = _graph_time_us([lambda: ws[0].fused(x, out, residual=r)] * n_copies) / n_copies
            cold = _graph_time_us([lambda w=w: w.fused(x, out, residual=r) for w in ws]) / n_copies
            res[name] = {"warm_us": warm, "cold_us": cold, "weight_mb": n * k * 2 / 1e6}
            del ws
            torch.cuda.empty_cache()
    elif args.case == "gemm":
        res["gemm"] = gemm_headline(dev)
    elif args.case == "c2":
        # the compiled config-2 encoder block: each instruction's device time
        # alone (CompiledModel.node_times) and the whole call from a graph
        from forgeml_b200.forgeml import compile as fml_compile
        from forgeml_b200.workloads import make_c2_block

        for dt, name in ((torch.bfloat16, "c2_block_bf16"), (torch.float32, "c2_block_fp32")):
            m, x = make_c2_block(dtype=dt)
            c = fml_compile(m.to(dev, dt), (x.to(dev),), backend="triton")
            xd = x.to(dev)
            with torch.inference_mode():
                us = _graph_time_us([lambda: c(xd)] * max(1, reps)) / max(1, reps)
                nodes = {k: round(v * 1e3, 2) for k, v in c.node_times(xd, repeats=max(1, reps)).items()}
            res[name] = {"us": us, "tflops": 64.42e9 / (us * 1e-6) / 1e12, "node_us": nodes}
    print(json.dumps({"case": args.case, "results": res}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU oracle baseline")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the decode before timing")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--cpu-layers", type=int, default=None, help="time this many layers of the CPU oracle")
    ap.add_argument("--tp", type=int, default=1, help="--case gemm-fused: TP shard shapes of this degree")
    ap.add_argument("--case", choices=("attention", "gemm-decode", "gemm-fused", "gemm-l2", "gemm", "c2"), default=None,
                    help="run one kernel micro-benchmark instead of the decode bench")
    ap.add_argument("--workload", choices=("c4", "c5"), default="c4",
                    help="c5: serve config 5 through the AsyncBatcher over TP x PP (launch with torchrun)")
    ap.add_argument("--c5-requests", type=int, default=32)
    ap.add_argument("--c5-new", type=int, default=64)
    ap.add_argument("--c5-window-ms", type=float, default=50.0, help="batching window of the c5 batcher")
    ap.add_argument("--c5-cohorts", action="store_true", help="c5: equal-length cohorts (the reference's batching)")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.workload == "c5":
        run_c5(args)
        return
    if args.warmup < 3 and args.impl == "native":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
