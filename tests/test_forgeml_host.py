"""ForgeML host logic on the CPU: graphs, passes and slot plans bit-exact
against the reference's own outputs (golden fixtures), kernel selection and
validation errors, and the native dispatch wiring (with the kernel calls
replaced by fakes, as the reference's tests/test_compiler.py:180-214 does)."""

import json
import random

import pytest
import torch
from torch import nn

from forgeml_b200.forgeml import compile, kernels
from forgeml_b200.forgeml.ir import Graph, GraphBuilder, GraphError, Node, TensorSpec
from forgeml_b200.forgeml.kernels import CANDIDATES, DEFAULT_CONFIG, KernelConfig
from forgeml_b200.forgeml.memory import plan_memory
from forgeml_b200.workloads import EncoderBlock, make_c1_mlp, make_c2_block
from oracle import memory as orc_memory
from tests.golden_io import load_memory_plans

_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "int64": torch.int64,
       "bool": torch.bool}


def graph_from_dict(d: dict) -> Graph:
    def spec(s):
        return TensorSpec(tuple(s["shape"]), _DT[s["dtype"]], s["device"])

    consts = {k: torch.zeros(tuple(v["shape"]), dtype=_DT[v["dtype"]]) for k, v in d["constants"].items()}
    nodes = []
    for n in d["nodes"]:
        attrs = {k: tuple(v) if isinstance(v, list) else v for k, v in n["attrs"].items()}
        nodes.append(Node(n["name"], n["op"], tuple(n["inputs"]), attrs, spec(n["spec"])))
    return Graph({k: spec(v) for k, v in d["inputs"].items()}, consts, nodes, tuple(d["outputs"]),
                 d["output_is_tuple"])


@pytest.mark.parametrize("name", sorted(load_memory_plans()))
def test_plan_memory_bit_exact_on_reference_graphs(name):
    rec = load_memory_plans()[name]
    g = graph_from_dict(rec["graph"])
    assert plan_memory(g).to_dict() == rec["plan"]


def _small_c2():
    torch.manual_seed(1)
    m = EncoderBlock(64, 4, 128).eval()
    return m, torch.randn(2, 16, 64)


@pytest.mark.parametrize("which", ["c1_mlp", "c2_block"])
def test_compile_reproduces_reference_graph_and_plan(which):
    gold = load_memory_plans()[which]
    m, x = make_c1_mlp() if which == "c1_mlp" else make_c2_block()
    c = compile(m, (x,))
    assert c.graph.to_dict() == gold["graph"]
    assert c.memory_plan.to_dict() == gold["plan"]
    assert len(c.original_graph.nodes) == gold["original_nodes"]
    assert [[p.name, p.nodes_before, p.nodes_after] for p in c.passes] == gold["passes"]
    ops = [n.op for n in c.graph.nodes]
    if which == "c2_block":
        assert ops.count("fused_linear_gelu") == 1 and ops.count("sdpa") == 1 and ops.count("narrow") == 3


def test_compile_reference_test_models():
    gold = load_memory_plans()
    torch.manual_seed(0)
    mlp = nn.Sequential(nn.Linear(8, 16), nn.GELU(approximate="tanh"), nn.Linear(16, 4)).eval()
    c = compile(mlp, (torch.randn(4, 8),))
    assert c.graph.to_dict() == gold["test_mlp_tanh"]["graph"]
    assert c.memory_plan.to_dict() == gold["test_mlp_tanh"]["plan"]

    class Mixed(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(16, 16)

        def forward(self, x):
            return torch.relu(self.lin(x)) + x

    torch.manual_seed(0)
    c = compile(Mixed().eval(), (torch.randn(4, 16),))
    assert c.graph.to_dict() == gold["mixed_relu_residual"]["graph"]


def test_planner_matches_oracle_on_random_graphs():
    rnd = random.Random(7)
    for trial in range(40):
        spec = lambda n: TensorSpec((n,), torch.float32, "cpu")  # noqa: E731
        b = GraphBuilder({"x": spec(8)})
        names = ["x"]
        for i in range(rnd.randint(3, 14)):
            op = rnd.choice(["relu", "add", "mul", "reshape_pair", "gelu"])
            src = rnd.choice(names)
            nm = f"n{i}"
            if op in ("add", "mul"):
                b.add(nm, op, (src, rnd.choice(names)))
            elif op == "reshape_pair":
                b.add(nm, "reshape", (src,), shape=(2, 4))
                b.add(nm + "f", "reshape", (nm,), shape=(8,))
                nm = nm + "f"
            else:
                b.add(nm, op, (src,))
            names.append(nm)
        outs = tuple(rnd.sample(names[1:], k=1))
        g = b.finish(outs)
        d = g.to_dict()
        assert plan_memory(g).to_dict() == orc_memory.plan(d["nodes"], d["outputs"]), trial


def test_torch_backend_parity_cpu():
    m, x = make_c1_mlp()
    c = compile(m, (x,))
    torch.testing.assert_close(c(x), m(x), rtol=1e-5, atol=1e-5)
    m2, x2 = _small_c2()
    c2 = compile(m2, (x2,))
    torch.testing.assert_close(c2(x2), m2(x2), rtol=1e-5, atol=1e-5)
    out1 = c2(x2)
    keep = out1.clone()
    out2 = c2(x2 + 1)
    torch.testing.assert_close(out1, keep)
    assert out1.data_ptr() != out2.data_ptr()


def test_kernel_front_door_cpu_errors():
    a = torch.randn(4, 4)
    with pytest.raises(GraphError, match="CUDA"):
        kernels.matmul(a, a)
    with pytest.raises(GraphError):
        kernels._check_config(KernelConfig(block_m=8))
    assert isinstance(DEFAULT_CONFIG, KernelConfig) and len(CANDIDATES) == 5
    assert kernels.available() is False
    assert "tcgen05.mma" in kernels.kernel_source()


def test_select_kernels_cpu():
    b = GraphBuilder({"x": TensorSpec((2, 4), torch.float32, "cpu")})
    b.constant("w", torch.randn(4, 8))
    b.add("mm", "matmul", ("x", "w"))
    g = b.finish(("mm",))
    assert kernels.select_kernels(g, "auto") == {"mm": "torch"}
    assert kernels.select_kernels(g, "torch") == {"mm": "torch"}
    with pytest.raises(GraphError, match="triton"):
        kernels.select_kernels(g, "triton")
    with pytest.raises(GraphError, match="backend"):
        kernels.select_kernels(g, "bogus")
    with pytest.raises(GraphError):
        compile(nn.Linear(8, 4).eval(), (torch.randn(2, 8),), backend="triton")
    with pytest.raises(GraphError, match="backend"):
        compile(nn.Linear(8, 4).eval(), (torch.randn(2, 8),), backend="tensorrt")


def test_native_dispatch_wiring_with_fakes(monkeypatch):
    """Force the native plan on CPU and replace the kernel launches with torch fakes:
    every GEMM/LN/SDPA node must reach its kernel with the right epilogue and write
    planned arena memory; the two residual adds ride in the o / fc2 GEMM epilogues
    and SDPA writes [B, S, H, D] through strides."""
    m, x = _small_c2()
    c = compile(m, (x,), backend="torch")
    calls = []
    arena = []

    def in_arena(t):
        return any(t.untyped_storage().data_ptr() == s.untyped_storage().data_ptr() for s in arena)

    def fake_gemm(self, a, b, bias, out, residual=None):
        calls.append(("matmul", self.act, in_arena(out), residual is not None))
        y = a @ b if bias is None else torch.addmm(bias, a, b)
        if self.act:
            y = torch.nn.functional.gelu(y, approximate="tanh" if self.act == 2 else "none")
        if residual is not None:
            y = y + residual
        return out.copy_(y)

    def fake_ln(xx, norm, w, b, eps, *, out=None):
        calls.append(("layer_norm", None, in_arena(out), False))
        return out.copy_(torch.nn.functional.layer_norm(xx, tuple(norm), w, b, eps))

    def fake_sdpa(q, k, v, mask=None, *, is_causal=False, scale=None, out=None):
        calls.append(("sdpa", out.stride(1) < out.stride(2), in_arena(out), False))
        return out.copy_(torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask,
                                                                          is_causal=is_causal, scale=scale))

    monkeypatch.setattr(kernels.PreparedGemm, "__call__", fake_gemm)
    monkeypatch.setattr(kernels, "layer_norm", fake_ln)
    monkeypatch.setattr(kernels, "sdpa", fake_sdpa)
    c.kernel_plan = {n.name: ("triton" if n.op in ("linear", "fused_linear_gelu", "layer_norm", "sdpa") else "torch")
                     for n in c.graph.nodes}
    arena.extend(c._arena.values())
    torch.testing.assert_close(c(x), m(x), rtol=1e-5, atol=1e-5)
    kinds = [k for k, *_ in calls]
    assert kinds.count("layer_norm") == 2 and kinds.count("sdpa") == 1 and kinds.count("matmul") == 4
    assert sum(1 for k, _, _, res in calls if k == "matmul" and res) == 2  # both residual adds fused
    assert ("matmul", 1, True, False) in calls  # fc1 + exact GELU into the arena
    assert ("sdpa", True, True, False) in calls  # [B, S, H, D] order, arena memory
    assert all(slot for k, _, slot, res in calls if not res)  # every other native node wrote the arena
    assert sorted(c.explain()["native_fusions"]["residual_add"]) == sorted(
        n.name for n in c.graph.nodes if n.op == "add")
    # the reference-compatible plan is untouched
    assert c.memory_plan.to_dict() == plan_memory(c.graph).to_dict()
    json.dumps(c.explain())
