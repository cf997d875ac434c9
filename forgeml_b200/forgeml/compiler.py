"""Compiled forward pass: per-node dispatch into the slot arena.

Drop-in for src/forgeml/compiler.py.  ``compile`` runs the frontend, the pass
pipeline, the slot planner and the kernel selection; ``CompiledModel`` keeps
the reference's contract (persistent slot arena allocated once, precompiled
per-node closures, refcount frees, output cloning rules, input guards,
non-reentrancy -- src/forgeml/compiler.py:19-237).

Nodes planned ``"triton"`` (the reference's label for its GPU kernel backend,
kept for API compatibility) run the sm_100a kernels: GEMM-family nodes write
their slot view through ``kernels.matmul(out=view)`` with the fused bias/GELU
epilogue, and LayerNorm / SDPA -- which the reference evaluated through torch
into fresh tensors -- write into an *extension* arena planned with the same
rules, so the reference-compatible ``memory_plan`` stays identical while the
native backend also keeps those outputs in planned memory.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field

import torch
import torch.nn.functional as F

from forgeml_b200.forgeml import kernels
from forgeml_b200.forgeml.analysis import graph_analysis
from forgeml_b200.forgeml.frontend import from_torch
from forgeml_b200.forgeml.ir import Graph, GraphError
from forgeml_b200.forgeml.kernels import DEFAULT_CONFIG, KernelConfig
from forgeml_b200.forgeml.memory import OUT_CAPABLE_OPS, VIEW_LIKE_OPS, MemoryPlan, plan_memory
from forgeml_b200.forgeml.ops import evaluate
from forgeml_b200.forgeml.passes import PassRecord
from forgeml_b200.forgeml.passes import optimize as optimize_graph

_EXT_OPS = frozenset({"layer_norm", "sdpa"})


def _slot_views(graph: Graph, plan: MemoryPlan) -> tuple[dict, dict]:
    slots = {s: torch.empty(spec.shape, dtype=spec.dtype, device=spec.device) for s, spec in plan.slot_specs.items()}
    views = {}
    for node in graph.nodes:
        a = plan.allocations.get(node.name)
        if a is not None:
            views[node.name] = slots[a.slot][: a.size_bytes // node.spec.dtype.itemsize].view(node.spec.shape)
    return slots, views


@dataclass
class CompiledModel:
    graph: Graph
    original_graph: Graph
    memory_plan: MemoryPlan
    passes: list[PassRecord]
    backend: str
    kernel_plan: dict[str, str] = field(default_factory=dict)
    kernel_configs: dict[str, KernelConfig] = field(default_factory=dict)

    def __post_init__(self) -> None:
        remaining: dict[str, int] = {}
        for node in self.graph.nodes:
            for i in node.inputs:
                remaining[i] = remaining.get(i, 0) + 1
        self._remaining_template = remaining
        self._outputs = frozenset(self.graph.outputs)
        self._produced = {n.name for n in self.graph.nodes}
        # The arena is allocated once and reused across calls, so __call__ is
        # not reentrant; concurrent callers must synchronise externally.
        self._slots, self._views = _slot_views(self.graph, self.memory_plan)
        self._build_ext_arena()
        self._steps = [(node, self._make_step(node)) for node in self.graph.nodes]

    def _build_ext_arena(self) -> None:
        """Slots for natively executed LayerNorm/SDPA nodes (same planning rules)."""
        ext = frozenset(OUT_CAPABLE_OPS | _EXT_OPS)
        plan = plan_memory(self.graph, out_capable=ext) if any(
            self.kernel_plan.get(n.name) == "triton" and n.op in _EXT_OPS for n in self.graph.nodes) else None
        self.ext_plan = plan
        self._ext_views = {}
        if plan is None:
            return
        only = {n.name for n in self.graph.nodes if n.op in _EXT_OPS and self.kernel_plan.get(n.name) == "triton"}
        sub = MemoryPlan({k: v for k, v in plan.allocations.items() if k in only}, {},
                         {}, plan.naive_bytes, 0)
        used = {a.slot for a in sub.allocations.values()}
        sub.slot_specs = {s: spec for s, spec in plan.slot_specs.items() if s in used}
        self._ext_slots, self._ext_views = _slot_views(self.graph, sub)

    def __setattr__(self, name, value):
        object.__setattr__(self, name, value)
        if name == "kernel_plan" and "_views" in self.__dict__:
            self._build_ext_arena()
            object.__setattr__(self, "_steps", [(n, self._make_step(n)) for n in self.graph.nodes])

    # ------------------------------------------------------------ dispatch
    def _make_step(self, node):
        native = self.kernel_plan.get(node.name) == "triton"
        is_output = node.name in self._outputs
        if node.op in VIEW_LIKE_OPS:
            if native:
                raise GraphError(f"no native kernel for op {node.op!r}")
            if is_output:
                return lambda args: self._evaluate(node, args).clone()
            return lambda args: self._evaluate(node, args)
        if native:
            view = None
            if not is_output:
                view = self._views.get(node.name)
                if view is None:
                    view = self._ext_views.get(node.name)
            return lambda args, node=node, view=view: self._run_native(node, args, view)
        if is_output:
            return lambda args: self._evaluate(node, args)
        if node.op not in OUT_CAPABLE_OPS:
            return lambda args: self._evaluate(node, args)
        view = self._views[node.name]
        op = node.op
        if op == "matmul":
            return lambda args: torch.matmul(args[0], args[1], out=view)
        if op == "linear":
            if len(node.inputs) == 3:
                return lambda args: torch.addmm(args[2], args[0], args[1], out=view)
            return lambda args: torch.mm(args[0], args[1], out=view)
        if op == "add":
            return lambda args: torch.add(args[0], args[1], out=view)
        if op == "mul":
            return lambda args: torch.mul(args[0], args[1], out=view)
        if op == "relu":
            return lambda args: torch.clamp_min(args[0], 0, out=view)
        if op == "softmax":
            dim = node.attrs["dim"]
            return lambda args: torch.softmax(args[0], dim=dim, out=view)
        if op == "gelu":
            approx = node.attrs.get("approximate", "none")
            return lambda args: F.gelu(args[0], approximate=approx, out=view)
        if op == "embedding":
            return lambda args: torch.ops.aten.embedding.out(args[1], args[0], -1, False, False, out=view)
        if op == "fused_linear_gelu":
            approx = node.attrs.get("approximate", "none")

            def run_fused(args, view=view, approx=approx):
                if len(args) == 3:
                    torch.addmm(args[2], args[0], args[1], out=view)
                else:
                    torch.mm(args[0], args[1], out=view)
                torch.ops.aten.gelu_.default(view, approximate=approx)
                return view

            return run_fused
        raise GraphError(f"no slot writer for op {node.op!r}")

    def _run_native(self, node, args, out):
        cfg = self.kernel_configs.get(node.name, DEFAULT_CONFIG)
        op = node.op
        if op == "matmul":
            return kernels.matmul(args[0], args[1], config=cfg, out=out)
        if op == "linear":
            return kernels.matmul(args[0], args[1], args[2] if len(args) == 3 else None, config=cfg, out=out)
        if op == "fused_linear_gelu":
            return kernels.matmul(args[0], args[1], args[2] if len(args) == 3 else None, activation="gelu",
                                  approximate=node.attrs.get("approximate", "none"), config=cfg, out=out)
        if op == "layer_norm":
            w, b = (args[1], args[2]) if len(args) == 3 else (None, None)
            return kernels.layer_norm(args[0], node.attrs["normalized_shape"], w, b, node.attrs["eps"], out=out)
        if op == "sdpa":
            return kernels.sdpa(args[0], args[1], args[2], args[3] if len(args) == 4 else None,
                                is_causal=node.attrs["is_causal"], scale=node.attrs.get("scale"), out=out)
        raise GraphError(f"no native kernel for op {op!r}")

    def autotune(self, *inputs: torch.Tensor, warmup: int = 3, repeats: int = 10) -> dict:
        from forgeml_b200.forgeml.autotune import tune_graph

        return tune_graph(self, inputs, warmup=warmup, repeats=repeats)

    def kernel_source(self) -> str:
        return kernels.kernel_source()

    def __call__(self, *inputs: torch.Tensor):
        names = list(self.graph.inputs)
        if len(inputs) != len(names):
            raise GraphError(f"expected {len(names)} inputs, got {len(inputs)}")
        values: dict[str, torch.Tensor] = {}
        for name, t in zip(names, inputs):
            if not isinstance(t, torch.Tensor):
                raise GraphError("inputs must be torch.Tensor")
            spec = self.graph.inputs[name]
            if tuple(t.shape) != spec.shape:
                raise GraphError(f"input {name!r} shape {tuple(t.shape)} != expected {spec.shape}")
            if t.dtype != spec.dtype:
                raise GraphError(f"input {name!r} dtype {t.dtype} != expected {spec.dtype}")
            if str(t.device) != spec.device:
                raise GraphError(f"input {name!r} device {t.device} != expected {spec.device}")
            values[name] = t
        values.update(self.graph.constants)
        remaining = dict(self._remaining_template)
        outputs = self._outputs
        with torch.inference_mode():
            for node, run in self._steps:
                values[node.name] = run(tuple(values[i] for i in node.inputs))
                for i in node.inputs:
                    if i in remaining:
                        remaining[i] -= 1
                        if remaining[i] == 0 and i not in outputs:
                            values.pop(i, None)
            result = []
            for name in self.graph.outputs:
                if name not in values:
                    raise GraphError(f"output {name!r} was not produced")
                result.append(values[name] if name in self._produced else values[name].clone())
        return tuple(result) if self.graph.output_is_tuple else result[0]

    @staticmethod
    def _evaluate(node, args):
        try:
            return evaluate(node.op, args, node.attrs)
        except GraphError:
            raise
        except Exception as e:  # noqa: BLE001
            raise GraphError(f"node {node.name!r} ({node.op}) execution failed: {e}") from e

    def explain(self) -> dict:
        a = graph_analysis(self.graph)
        oa = graph_analysis(self.original_graph)
        return {
            "backend": self.backend,
            "original_nodes": len(self.original_graph.nodes),
            "optimized_nodes": len(self.graph.nodes),
            "passes": [{"name": p.name, "nodes_before": p.nodes_before, "nodes_after": p.nodes_after}
                       for p in self.passes],
            "memory_plan": self.memory_plan.to_dict(),
            "extension_plan": self.ext_plan.to_dict() if self.ext_plan is not None else None,
            "graph": self.graph.to_dict(),
            "kernel_plan": dict(self.kernel_plan),
            "kernel_configs": {k: asdict(v) for k, v in self.kernel_configs.items()},
            "analysis": a,
            "original_analysis": oa,
            "optimization_delta": {
                "nodes": len(self.original_graph.nodes) - len(self.graph.nodes),
                "flops": oa["flops"] - a["flops"],
                "logical_bytes": oa["logical_bytes"] - a["logical_bytes"],
                "critical_path_ops": oa["critical_path_ops"] - a["critical_path_ops"],
                "planned_bytes": self.memory_plan.naive_bytes - self.memory_plan.planned_bytes,
            },
        }


def compile(model: torch.nn.Module | Graph, example_inputs: tuple[torch.Tensor, ...] = (), *,
            backend: str = "torch", optimize: bool = True) -> CompiledModel:
    if backend not in ("torch", "triton", "auto"):
        raise GraphError(f"unsupported backend {backend!r}; expected 'torch', 'triton', or 'auto'")
    if isinstance(model, Graph):
        model.validate()
        graph = model.clone()
    elif isinstance(model, torch.nn.Module):
        graph = from_torch(model, example_inputs)
    else:
        raise GraphError("compile expects an nn.Module or a Graph")
    original = graph.clone()
    if optimize:
        graph, records = optimize_graph(graph)
    else:
        graph.validate()
        records = []
    plan = plan_memory(graph)
    return CompiledModel(graph, original, plan, records, backend, kernel_plan=kernels.select_kernels(graph, backend))
