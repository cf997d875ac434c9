"""Correctness-gated tile selection for native GEMM nodes.

Contract of src/forgeml/autotune.py:16-103: for each node planned for the
native backend the expected value is evaluated with torch on the same inputs,
every candidate tile configuration (``kernels.CANDIDATES``: sm_100a UMMA N
tiles and pipeline depths) is launched and gated by ``check_output``; a
candidate that raises is recorded as rejected; the survivors are timed with
``measure_variants`` and the smallest median wins.  Selections live on the
CompiledModel instance only.
"""

from __future__ import annotations

from dataclasses import asdict
from typing import TYPE_CHECKING

import torch

from forgeml_b200.forgeml import kernels
from forgeml_b200.forgeml.measurement import check_output, measure_variants
from forgeml_b200.forgeml.ops import evaluate

if TYPE_CHECKING:
    from forgeml_b200.forgeml.compiler import CompiledModel

_TUNABLE = ("matmul", "linear", "fused_linear_gelu")


@torch.inference_mode()
def tune_graph(compiled: "CompiledModel", inputs: tuple[torch.Tensor, ...], *, warmup: int = 3,
               repeats: int = 10) -> dict:
    if warmup < 0 or repeats < 2:
        raise ValueError("autotuning requires warmup >= 0 and repeats >= 2")
    compiled(*inputs)
    values = dict(compiled.graph.constants)
    values.update(zip(compiled.graph.inputs, inputs))
    records, chosen = {}, {}
    for node in compiled.graph.nodes:
        args = tuple(values[n] for n in node.inputs)
        expected = evaluate(node.op, args, node.attrs)
        if compiled.kernel_plan.get(node.name) == "triton" and node.op in _TUNABLE:
            bias = args[2] if len(args) == 3 else None
            activation = "gelu" if node.op == "fused_linear_gelu" else "none"
            approximate = node.attrs.get("approximate", "none") if activation == "gelu" else "none"
            variants, configs, rejected, errors = {}, {}, {}, {}
            for idx, cfg in enumerate(kernels.CANDIDATES):
                name = f"candidate_{idx}"

                def launch(cfg=cfg, args=args, bias=bias, activation=activation, approximate=approximate):
                    return kernels.matmul(args[0], args[1], bias, activation=activation, approximate=approximate,
                                          config=cfg)

                try:
                    errors[name] = check_output(launch(), expected)
                except Exception as exc:  # noqa: BLE001 - any failure rejects the candidate
                    rejected[name] = str(exc)
                    continue
                variants[name] = launch
                configs[name] = cfg
            if not variants:
                raise RuntimeError(f"no numerically valid kernel candidate for {node.name!r}")
            timings = measure_variants(variants, device=args[0].device, warmup=warmup, repeats=repeats)
            winner = min(timings, key=lambda n: timings[n]["median_ms"])
            chosen[node.name] = configs[winner]
            records[node.name] = {
                "winner": winner, "config": asdict(configs[winner]),
                "candidates": {n: {"config": asdict(configs[n]), "timing": t, "correctness": errors[n]}
                               for n, t in timings.items()},
                "rejected": rejected,
                "input_shapes": [list(a.shape) for a in args], "input_strides": [list(a.stride()) for a in args],
                "dtype": str(args[0].dtype), "device": str(args[0].device),
                "activation": activation, "approximate": approximate,
            }
        values[node.name] = expected
    compiled.kernel_configs.update(chosen)
    return {"scope": "this_compiled_model_instance_only",
            "timing": "synchronized_host_wall_clock_including_output_allocation",
            "warmup": warmup, "repeats": repeats, "nodes": records}
