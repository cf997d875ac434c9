"""Generate the golden fixtures under tests/golden/ by running the REFERENCE.

Run in a container where the reference source tree is available:

    REFERENCE_SRC=/path/to/ForgeML/src python tests/golden/make_golden.py

It imports the reference packages (forgeml, nebula) and records, for small
seeded inputs:
  gemm.pt           the reference kernel contracts of tests/test_kernels.py
                    (shapes (1,17,9), (31,65,33), (64,64,64) x fp32/fp16/bf16,
                    bias+GELU erf/tanh 16x32x24, strided bias, .t() operands)
                    evaluated with the reference's own formulas, plus the
                    torch-backend result of forgeml.ops.evaluate
  memory_plans.json graph.to_dict() and plan_memory(graph).to_dict() for the
                    reference planner tests' graphs and the compiled c1/c2
                    graphs (forgeml.compile(..., backend="torch"))
  nebula_small.pt   TinyDecoder(DecoderConfig(32,16,4,2,32,16,seed=17))
                    state dict, prefill/decode logits and greedy tokens as
                    produced by nebula.Engine on CPU
The GPU box never runs this script; tests only read its outputs.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if "REFERENCE_SRC" not in os.environ:
    sys.exit("set REFERENCE_SRC to the reference project's src directory (the one holding forgeml/ and nebula/)")
sys.path.insert(0, os.environ["REFERENCE_SRC"])
sys.path.insert(0, str(REPO))

from forgeml import compile as ref_compile  # noqa: E402
from forgeml.ir import GraphBuilder, TensorSpec  # noqa: E402
from forgeml.memory import plan_memory  # noqa: E402
from forgeml.ops import evaluate  # noqa: E402
from nebula import DecoderConfig, Engine, ParallelContext, TinyDecoder  # noqa: E402

from forgeml_b200.workloads import make_c1_mlp, make_c2_block  # noqa: E402


def gemm_cases() -> dict:
    torch.manual_seed(1234)
    cases = []
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        for m, n, k in ((1, 17, 9), (31, 65, 33), (64, 64, 64)):
            a = torch.randn(m, k, dtype=torch.float32).to(dtype)
            b = torch.randn(k, n, dtype=torch.float32).to(dtype)
            # tests/test_kernels.py:110 contract: fp32 product rounded once to dtype
            want = torch.matmul(a.float(), b.float()).to(dtype)
            cases.append(dict(kind="matmul", a=a, b=b, bias=None, approximate="none", activation="none",
                              want=want, want_torch=evaluate("matmul", (a.float(), b.float()), {}).to(dtype)))
        for approx in ("none", "tanh"):
            a = torch.randn(16, 32).to(dtype)
            b = torch.randn(32, 24).to(dtype)
            bias = torch.randn(24).to(dtype)
            # tests/test_kernels.py:124-126 contract: gelu(round(a@b) + bias)
            want = torch.nn.functional.gelu((a.float() @ b.float()).to(dtype) + bias, approximate=approx)
            want_torch = evaluate("fused_linear_gelu", (a.float(), b.float(), bias.float()),
                                  {"approximate": approx}).to(dtype)
            cases.append(dict(kind="bias_gelu", a=a, b=b, bias=bias, approximate=approx, activation="gelu",
                              want=want, want_torch=want_torch))
    for approx in ("none", "tanh"):
        a = torch.randn(16, 32)
        b = torch.randn(32, 24)
        bias_base = torch.randn(48)
        bias = bias_base[::2]
        want = torch.nn.functional.gelu(a @ b + bias, approximate=approx)
        cases.append(dict(kind="strided_bias", a=a, b=b, bias=bias_base, bias_step=2, approximate=approx,
                          activation="gelu", want=want, want_torch=want))
    a_base = torch.randn(32, 16)
    b_base = torch.randn(24, 32)
    cases.append(dict(kind="transposed", a=a_base, b=b_base, bias=None, approximate="none", activation="none",
                      want=a_base.t() @ b_base.t(), want_torch=a_base.t() @ b_base.t()))
    return {"cases": cases}


def _spec(*shape):
    return TensorSpec(tuple(shape), torch.float32, "cpu")


def planner_graphs() -> list[tuple[str, object]]:
    out = []
    b = GraphBuilder({"x": _spec(4), "z": _spec(4)})
    b.add("a", "relu", ("x",)); b.add("b", "relu", ("a",)); b.add("c", "relu", ("z",))
    b.add("d", "relu", ("c",)); b.add("y", "add", ("b", "d"))
    out.append(("chain", b.finish(("y",))))
    b = GraphBuilder({"x": _spec(8), "z": _spec(2, 4)})
    b.add("a", "relu", ("x",)); b.add("r", "reshape", ("a",), shape=(2, 4)); b.add("c", "relu", ("z",))
    b.add("y", "add", ("r", "c"))
    out.append(("reshape_view", b.finish(("y",))))
    b = GraphBuilder({"x": _spec(2, 4), "z": _spec(4, 2)})
    b.add("a", "relu", ("x",)); b.add("t", "transpose", ("a",), dim0=0, dim1=1); b.add("c", "relu", ("z",))
    b.add("y", "add", ("t", "c"))
    out.append(("transpose_view", b.finish(("y",))))
    b = GraphBuilder({"x": _spec(8), "z": _spec(8)})
    b.add("a", "relu", ("x",)); b.add("b", "relu", ("a",)); b.add("c", "relu", ("z",)); b.add("y", "add", ("b", "c"))
    out.append(("naive_planned", b.finish(("y",))))
    b = GraphBuilder({"x": _spec(4), "z": _spec(4)})
    b.add("a", "relu", ("x",)); b.add("b", "relu", ("z",)); b.add("y", "add", ("a", "b"))
    out.append(("overlap", b.finish(("y",))))
    # best-fit among several free slots of different sizes, mixed dtypes
    b = GraphBuilder({"x": _spec(16), "h": TensorSpec((8,), torch.float16, "cpu")})
    b.add("big", "relu", ("x",)); b.add("bigger", "mul", ("big", "big"))
    b.add("small", "narrow", ("bigger",), dim=0, start=0, length=4)
    b.add("s2", "relu", ("small",)); b.add("hh", "relu", ("h",)); b.add("h2", "relu", ("hh",))
    b.add("s3", "relu", ("s2",)); b.add("s4", "add", ("s3", "s3")); b.add("y", "relu", ("s4",))
    out.append(("best_fit_mixed", b.finish(("y", "h2"))))
    return out


def compiled_graphs() -> list[tuple[str, object]]:
    out = []
    m, x = make_c1_mlp()
    c = ref_compile(m, (x,), backend="torch")
    out.append(("c1_mlp", c))
    m, x = make_c2_block()
    c = ref_compile(m, (x,), backend="torch")
    out.append(("c2_block", c))
    torch.manual_seed(0)
    mlp = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(16, 4)).eval()
    out.append(("test_mlp_tanh", ref_compile(mlp, (torch.randn(4, 8),), backend="torch")))

    class Mixed(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(16, 16)

        def forward(self, x):
            return torch.relu(self.lin(x)) + x

    torch.manual_seed(0)
    out.append(("mixed_relu_residual", ref_compile(Mixed().eval(), (torch.randn(4, 16),), backend="torch")))
    return out


def memory_plans() -> dict:
    recs = {}
    for name, g in planner_graphs():
        recs[name] = {"graph": g.to_dict(), "plan": plan_memory(g).to_dict()}
    for name, c in compiled_graphs():
        recs[name] = {
            "graph": c.graph.to_dict(),
            "plan": c.memory_plan.to_dict(),
            "original_nodes": len(c.original_graph.nodes),
            "passes": [[p.name, p.nodes_before, p.nodes_after] for p in c.passes],
        }
    return recs


def nebula_small() -> dict:
    cfg = DecoderConfig(vocab_size=32, hidden_size=16, num_heads=4, num_layers=2,
                        intermediate_size=32, max_seq_len=16, seed=17)
    ref = TinyDecoder(cfg).eval()
    eng = Engine(cfg, context=ParallelContext.from_env(), max_requests=4)
    toks = torch.tensor([[1, 2, 3], [4, 5, 6]])
    prefill = eng.forward(toks, (11, 12), 0)
    step = torch.tensor([[7], [8]])
    decode = eng.forward(step, (11, 12), 3)
    eng.release((11, 12))
    prompts = [[1, 2, 3], [4, 5], [9, 9, 9]]
    tokens = eng.generate(prompts, 3)
    long_tokens = eng.generate([[3, 1, 4, 1, 5]], 8)
    eng.close()
    with torch.no_grad():
        ref_logits = ref(torch.tensor([[1, 2, 3, 7], [4, 5, 6, 8]]))
    return {
        "config": dict(vocab_size=32, hidden_size=16, num_heads=4, num_layers=2, intermediate_size=32,
                       max_seq_len=16, seed=17),
        "state_dict": {k: v.clone() for k, v in ref.state_dict().items()},
        "prefill_tokens": toks, "prefill_ids": (11, 12), "prefill_logits": prefill,
        "decode_tokens": step, "decode_logits": decode,
        "monolithic_logits": ref_logits,
        "generate_prompts": prompts, "generate_tokens": tokens,
        "generate_long_prompt": [[3, 1, 4, 1, 5]], "generate_long_tokens": long_tokens,
    }


def main() -> None:
    torch.save(gemm_cases(), HERE / "gemm.pt")
    (HERE / "memory_plans.json").write_text(json.dumps(memory_plans(), indent=1, sort_keys=True))
    torch.save(nebula_small(), HERE / "nebula_small.pt")
    for p in sorted(HERE.iterdir()):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
