"""Correctness-gated choice of GEMM tile configurations for one compiled model.

Contract of the reference autotuner (src/forgeml/autotune.py:16-103): for
every GEMM node planned on the native backend, each candidate configuration
(``kernels.CANDIDATES``: UMMA N tile and pipeline depth of the tcgen05 GEMM)
is launched on the node's real inputs and its result compared with the torch
evaluation of the node; a candidate that fails to launch or disagrees is
rejected with the reason, the survivors are timed and the fastest median
wins.  The choice is stored on that compiled model only.  A node with no
valid candidate is an error.

Agreement uses the tolerances of this package's parity bar: fp32 (3xTF32)
rtol 1e-5 / atol 1e-4, fp16 1e-2 / 1e-2, bf16 2e-2 / 2e-2.  Survivors are
timed on the device with CUDA events around each launch (``_time_candidates``).
"""

from __future__ import annotations

import statistics
from dataclasses import asdict
from typing import TYPE_CHECKING, Callable

import torch

from forgeml_b200.forgeml import kernels
from forgeml_b200.forgeml.ops import evaluate

if TYPE_CHECKING:
    from forgeml_b200.forgeml.compiler import CompiledModel

_TUNED_OPS = ("matmul", "linear", "fused_linear_gelu")
_TOLERANCE = {torch.float32: (1e-5, 1e-4), torch.float16: (1e-2, 1e-2), torch.bfloat16: (2e-2, 2e-2)}


def _agreement(got: torch.Tensor, want: torch.Tensor) -> dict:
    rtol, atol = _TOLERANCE.get(want.dtype, (1e-5, 1e-4))
    g, w = got.float(), want.float()
    excess = ((g - w).abs() - (atol + rtol * w.abs())).max().item() if w.numel() else 0.0
    return {"passed": bool(torch.isfinite(g).all().item()) and excess <= 0.0,
            "max_abs_err": (g - w).abs().max().item() if w.numel() else 0.0, "rtol": rtol, "atol": atol}


def _time_candidates(runs: dict[str, Callable[[], object]], *, device: torch.device, warmup: int,
                     repeats: int) -> dict[str, dict]:
    """Device time of each launch: CUDA events on the current stream around
    every repetition, after ``warmup`` untimed launches."""
    out = {}
    stream = torch.cuda.current_stream(device)
    for name, run in runs.items():
        for _ in range(warmup):
            run()
        samples = []
        for _ in range(repeats):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run()
            e1.record(stream)
            e1.synchronize()
            samples.append(e0.elapsed_time(e1))
        out[name] = {"median_ms": statistics.median(samples), "samples_ms": samples}
    return out


@torch.inference_mode()
def tune_graph(compiled: "CompiledModel", inputs: tuple[torch.Tensor, ...], *, warmup: int = 3,
               repeats: int = 10) -> dict:
    if warmup < 0 or repeats < 2:
        raise ValueError("autotuning requires warmup >= 0 and repeats >= 2")
    compiled(*inputs)
    env = dict(compiled.graph.constants)
    env.update(zip(compiled.graph.inputs, inputs))
    report, chosen = {}, {}
    for node in compiled.graph.nodes:
        args = tuple(env[i] for i in node.inputs)
        want = evaluate(node.op, args, node.attrs)
        env[node.name] = want
        if node.op not in _TUNED_OPS or compiled.kernel_plan.get(node.name) != "triton":
            continue
        act = "gelu" if node.op == "fused_linear_gelu" else "none"
        approx = node.attrs.get("approximate", "none") if act == "gelu" else "none"
        bias = args[2] if len(args) == 3 else None
        kept, rejected, checks = {}, {}, {}
        for idx, cfg in enumerate(kernels.CANDIDATES):
            name = f"candidate_{idx}"
            try:
                launch = kernels.PreparedGemm(want.dtype, act, approx, cfg)
                out = torch.empty_like(want)
                launch(args[0], args[1], bias, out)
                check = _agreement(out, want)
            except Exception as exc:  # noqa: BLE001 - a launch failure rejects the candidate
                rejected[name] = f"launch failed: {exc}"
                continue
            if not check["passed"]:
                rejected[name] = f"wrong result: max abs err {check['max_abs_err']:.3e}"
                continue
            checks[name] = check
            kept[name] = (cfg, lambda launch=launch, out=out: launch(args[0], args[1], bias, out))
        if not kept:
            raise RuntimeError(f"no numerically valid kernel candidate for {node.name!r}")
        timings = _time_candidates({n: run for n, (_, run) in kept.items()}, device=args[0].device,
                                   warmup=warmup, repeats=repeats)
        winner = min(timings, key=lambda n: timings[n]["median_ms"])
        chosen[node.name] = kept[winner][0]
        report[node.name] = {
            "winner": winner, "config": asdict(kept[winner][0]), "rejected": rejected,
            "candidates": {n: {"config": asdict(kept[n][0]), "timing": timings[n], "correctness": checks[n]}
                           for n in kept},
            "input_shapes": [list(a.shape) for a in args], "input_strides": [list(a.stride()) for a in args],
            "dtype": str(want.dtype), "device": str(args[0].device), "activation": act, "approximate": approx,
        }
    compiled.kernel_configs.update(chosen)
    return {"scope": "this_compiled_model_instance_only", "timing": "cuda_events_per_launch_median",
            "warmup": warmup, "repeats": repeats, "nodes": report}
