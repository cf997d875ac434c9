"""Compiled forward pass: a graph lowered to an instruction program over a
persistent slot arena, with the GEMM, LayerNorm and SDPA nodes on the sm_100a
kernels.

Public surface of the reference (src/forgeml/compiler.py:19-264):
``compile(model_or_graph, example_inputs, *, backend, optimize)`` and
``CompiledModel`` with graph, original_graph, memory_plan, passes, backend,
kernel_plan, kernel_configs, ``__call__``, ``autotune``, ``kernel_source``,
``explain``.  ``memory_plan`` is the reference's slot plan of the optimised
graph, bit for bit.  Input guards, output cloning (views and pass-through
values are returned as copies, never as arena memory) and non-reentrancy are
the reference's.

Execution.  ``compile`` lowers the graph once into a ``_Program``: every
value gets an integer id, every node one instruction (a precompiled closure,
its argument ids, its result id and the ids it is the last reader of).  The
program runs over its own arena, planned by the same slot rules over the
*execution* entries (``memory.plan_slots``).  With the torch backend those
entries are the graph's nodes and the arena is ``memory_plan`` itself.  With
the native backend ("triton", the reference's label, or "auto") two rewrites
keep more of the forward pass inside the kernels:

  * residual add into the GEMM epilogue: ``add(r, view(gemm(...)))`` (or
    the operands swapped), where the GEMM runs natively and feeds only that
    add through reshape views that keep its [M, N] rows, becomes one GEMM
    launch with ``residual=r`` writing the add's result;
  * SDPA in [B, S, H, D] order: a native SDPA whose only reader is
    ``transpose(., 1, 2)`` writes its output through strides into a
    [B, S, H, D] buffer, so that transpose and the following reshape are
    views (the reference materialised the transposed copy);

and LayerNorm / SDPA outputs get arena slots too (the reference returned
fresh tensors for them).  The rewrites only move where values are written;
each output element is computed by the same kernel arithmetic.
"""

from __future__ import annotations

import math
import warnings
from dataclasses import asdict
from typing import Callable

import torch
import torch.nn.functional as F

from forgeml_b200.forgeml import kernels
from forgeml_b200.forgeml.frontend import from_torch
from forgeml_b200.forgeml.ir import Graph, GraphError
from forgeml_b200.forgeml.kernels import DEFAULT_CONFIG, KernelConfig
from forgeml_b200.forgeml.memory import (OUT_CAPABLE_OPS, VIEW_LIKE_OPS, Entry, MemoryPlan, plan_memory,
                                         plan_slots)
from forgeml_b200.forgeml.ops import evaluate
from forgeml_b200.forgeml.passes import PassRecord
from forgeml_b200.forgeml.passes import optimize as optimize_graph

NATIVE = "triton"  # the reference's plan label for its GPU kernel backend
_GEMM_OPS = ("matmul", "linear", "fused_linear_gelu")
_NATIVE_ARENA_OPS = frozenset({"native:" + op for op in _GEMM_OPS + ("layer_norm", "sdpa", "gemm_residual")})


def _fail_wrap(node, fn: Callable) -> Callable:
    def run(*args):
        try:
            return fn(*args)
        except GraphError:
            raise
        except Exception as exc:  # noqa: BLE001 - every failure is reported as the node's
            raise GraphError(f"node {node.name!r} ({node.op}) execution failed: {exc}") from exc

    return run


class _Lowering:
    """Builds the execution entries and instructions of one compiled model."""

    def __init__(self, graph: Graph, kernel_plan: dict, kernel_configs: dict):
        self.g = graph
        self.plan = kernel_plan
        self.configs = kernel_configs
        self.nodes = {n.name: n for n in graph.nodes}
        self.readers: dict[str, list[str]] = {}
        for n in graph.nodes:
            for i in n.inputs:
                self.readers.setdefault(i, []).append(n.name)
        self.outputs = set(graph.outputs)
        self.native = {n.name for n in graph.nodes if kernel_plan.get(n.name) == NATIVE}

    # ---------------------------------------------------------- rewrites
    def _sole_reader(self, name: str) -> str | None:
        r = self.readers.get(name, [])
        return r[0] if len(r) == 1 and name not in self.outputs else None

    def _gemm_behind(self, name: str) -> tuple[str, list[str]] | None:
        """(gemm node, view chain) when ``name`` is a native GEMM's value seen
        through reshape views that are its only readers, one after another."""
        chain = []
        cur = self.nodes.get(name)
        while cur is not None and cur.op == "reshape":
            chain.append(cur.name)
            cur = self.nodes.get(cur.inputs[0])
        if cur is None or cur.op not in _GEMM_OPS or cur.name not in self.native:
            return None
        path = [cur.name] + chain[::-1]
        for a, b in zip(path, path[1:] + [None]):
            if b is not None and self._sole_reader(a) != b:
                return None
        if cur.name in self.outputs or any(v in self.outputs for v in chain):
            return None
        return cur.name, chain

    def residual_fusions(self) -> dict[str, tuple[str, list[str], str]]:
        """add node -> (gemm node, view chain, residual operand)."""
        found = {}
        for n in self.g.nodes:
            if n.op != "add" or len(n.inputs) != 2 or n.inputs[0] == n.inputs[1]:
                continue
            for side in (1, 0):
                hit = self._gemm_behind(n.inputs[side])
                if hit is None:
                    continue
                gemm, chain = hit
                last = chain[-1] if chain else gemm
                if self._sole_reader(last) != n.name:
                    continue
                other = n.inputs[1 - side]
                ospec, gspec = self.g.specs()[other], self.nodes[gemm].spec
                if (tuple(ospec.shape) != tuple(n.spec.shape) or ospec.dtype != n.spec.dtype
                        or n.spec.shape[-1] != gspec.shape[-1] or gspec.dtype != n.spec.dtype
                        or math.prod(n.spec.shape) != math.prod(gspec.shape)):
                    continue
                found[n.name] = (gemm, chain, other)
                break
        return found

    def bshd_sdpa(self) -> set[str]:
        out = set()
        for n in self.g.nodes:
            if n.op != "sdpa" or n.name not in self.native:
                continue
            r = self._sole_reader(n.name)
            t = self.nodes.get(r) if r else None
            if t is not None and t.op == "transpose" and {t.attrs["dim0"] % 4, t.attrs["dim1"] % 4} == {1, 2}:
                out.add(n.name)
        return out


class _Program:
    """Straight-line instruction list over integer value ids."""

    def __init__(self, n_values: int, inputs: list[int], constants: list[tuple[int, torch.Tensor]],
                 instrs: list[tuple], outputs: list[tuple[int, bool]]):
        self.n_values = n_values
        self.inputs = inputs
        self.constants = constants
        self.instrs = instrs
        self.outputs = outputs

    def run(self, args: tuple) -> list[torch.Tensor]:
        vals: list = [None] * self.n_values
        for vid, t in zip(self.inputs, args):
            vals[vid] = t
        for vid, t in self.constants:
            vals[vid] = t
        for fn, arg_ids, out_id, drops in self.instrs:
            vals[out_id] = fn(*[vals[i] for i in arg_ids])
            for d in drops:
                vals[d] = None
        return [vals[i].clone() if copy else vals[i] for i, copy in self.outputs]


class CompiledModel:
    """A graph compiled for one device; not reentrant (one arena per model)."""

    def __init__(self, graph: Graph, original_graph: Graph, memory_plan: MemoryPlan, passes: list[PassRecord],
                 backend: str, kernel_plan: dict[str, str] | None = None,
                 kernel_configs: dict[str, KernelConfig] | None = None):
        self.graph = graph
        self.original_graph = original_graph
        self.memory_plan = memory_plan
        self.passes = passes
        self.backend = backend
        self.kernel_configs = dict(kernel_configs or {})
        self.kernel_plan = dict(kernel_plan or {})  # lowers the program

    # A changed plan (tests force nodes native) or tile config re-lowers.
    @property
    def kernel_plan(self) -> dict[str, str]:
        return self._kernel_plan

    @kernel_plan.setter
    def kernel_plan(self, plan: dict[str, str]) -> None:
        self._kernel_plan = dict(plan)
        self._lower()

    # ------------------------------------------------------------ lowering
    def _lower(self) -> None:
        g = self.graph
        low = _Lowering(g, self._kernel_plan, self.kernel_configs)
        fused = low.residual_fusions()
        skipped = {gm for gm, _, _ in fused.values()} | {v for _, ch, _ in fused.values() for v in ch}
        bshd = low.bshd_sdpa()
        self.fusions = {"residual_add": {z: gm for z, (gm, _, _) in fused.items()}, "sdpa_bshd": sorted(bshd)}

        # execution entries (what the arena is planned over)
        entries = []
        for n in g.nodes:
            if n.name in skipped:
                continue
            if n.name in fused:
                gm, _, other = fused[n.name]
                entries.append(Entry(n.name, "native:gemm_residual", tuple(low.nodes[gm].inputs) + (other,), n.spec))
            elif n.name in low.native:
                entries.append(Entry(n.name, "native:" + n.op, tuple(n.inputs), n.spec))
            else:
                entries.append(Entry(n.name, n.op, tuple(n.inputs), n.spec))
        self.execution_plan = plan_slots(entries, g.outputs, OUT_CAPABLE_OPS | _NATIVE_ARENA_OPS)
        plan = self.execution_plan
        slots = {s: torch.empty(spec.shape, dtype=spec.dtype, device=spec.device)
                 for s, spec in plan.slot_specs.items()}
        self._arena = slots  # keeps the slot storage alive

        def arena_view(name: str, shape) -> torch.Tensor:
            a = plan.allocations[name]
            spec = next(e.spec for e in entries if e.name == name)
            return slots[a.slot][: a.size_bytes // spec.dtype.itemsize].view(tuple(shape))

        # value ids: inputs, constants, then entries
        ids: dict[str, int] = {}
        for name in g.inputs:
            ids[name] = len(ids)
        for name in g.constants:
            ids[name] = len(ids)
        for e in entries:
            ids[e.name] = len(ids)
        last_reader: dict[str, int] = {}
        for k, e in enumerate(entries):
            for i in e.inputs:
                last_reader[i] = k
        keep = set(g.outputs) | set(g.inputs) | set(g.constants)
        instrs = []
        for k, e in enumerate(entries):
            node = low.nodes[e.name]
            is_out = e.name in low.outputs
            has_slot = e.name in plan.allocations
            if e.op == "native:gemm_residual":
                gm, _, _ = fused[e.name]
                fn = self._gemm_residual_step(low.nodes[gm], node, arena_view if has_slot else None)
            elif e.op.startswith("native:"):
                fn = self._native_step(node, arena_view if has_slot else None, e.name in bshd)
            else:
                fn = self._torch_step(node, is_out, arena_view(e.name, [plan.allocations[e.name].size_bytes
                                                                         // node.spec.dtype.itemsize])
                                      if has_slot else None)
            drops = tuple(ids[i] for i in set(e.inputs) if last_reader.get(i) == k and i not in keep)
            instrs.append((_fail_wrap(node, fn), tuple(ids[i] for i in e.inputs), ids[e.name], drops))
        self._instr_names = [f"{e.name} ({e.op})" for e in entries]
        produced = {e.name for e in entries}
        outputs = [(ids[o], o not in produced) for o in g.outputs]
        self._program = _Program(len(ids), [ids[n] for n in g.inputs],
                                 [(ids[n], t) for n, t in g.constants.items()], instrs, outputs)

    def _torch_step(self, node, is_out: bool, flat: torch.Tensor | None) -> Callable:
        op, attrs = node.op, node.attrs
        if op in VIEW_LIKE_OPS:
            if is_out:
                return lambda *a: evaluate(op, a, attrs).clone()
            return lambda *a: evaluate(op, a, attrs)
        if flat is None:  # outputs and ops without an out= writer allocate
            return lambda *a: evaluate(op, a, attrs)
        view = flat.view(node.spec.shape)
        approx = attrs.get("approximate", "none")
        writers = {
            "matmul": lambda x, y: torch.matmul(x, y, out=view),
            "linear": lambda x, w, b=None: torch.mm(x, w, out=view) if b is None else torch.addmm(b, x, w, out=view),
            "add": lambda x, y: torch.add(x, y, out=view),
            "mul": lambda x, y: torch.mul(x, y, out=view),
            "relu": lambda x: torch.clamp_min(x, 0, out=view),
            "softmax": lambda x: torch.softmax(x, dim=attrs.get("dim"), out=view),
            "gelu": lambda x: F.gelu(x, approximate=approx, out=view),
            "embedding": lambda i, w: torch.ops.aten.embedding.out(w, i, -1, False, False, out=view),
        }
        if op == "fused_linear_gelu":
            def linear_gelu(x, w, b=None):
                torch.mm(x, w, out=view) if b is None else torch.addmm(b, x, w, out=view)
                return torch.ops.aten.gelu_.default(view, approximate=approx)

            return linear_gelu
        if op not in writers:
            raise GraphError(f"no slot writer for op {op!r}")
        return writers[op]

    def _gemm_launch(self, node) -> kernels.PreparedGemm:
        act = "gelu" if node.op == "fused_linear_gelu" else "none"
        approx = node.attrs.get("approximate", "none") if act == "gelu" else "none"
        launch = kernels.PreparedGemm(node.spec.dtype, act, approx,
                                      self.kernel_configs.get(node.name, DEFAULT_CONFIG))
        w = self.graph.constants.get(node.inputs[1])
        if w is not None and w.dtype == torch.float32 and w.is_cuda:
            launch.pack_constant_b(w)  # a compiled fp32 weight is split into its 3xTF32 image once
            torch.cuda.current_stream(w.device).synchronize()  # ready for calls on any stream
        return launch

    def _native_step(self, node, arena_view, bshd: bool) -> Callable:
        op, attrs, spec = node.op, node.attrs, node.spec
        fresh = arena_view is None

        def target(shape=spec.shape):
            return (torch.empty(shape, dtype=spec.dtype, device=spec.device) if fresh
                    else arena_view(node.name, shape))

        if op in _GEMM_OPS:
            if spec.dtype not in (torch.float32, torch.float16, torch.bfloat16):
                raise GraphError(f"no native kernel for {spec.dtype}")
            launch = self._gemm_launch(node)
            out_view = None if fresh else arena_view(node.name, spec.shape)

            def gemm(a, b, bias=None):
                return launch(a, b, bias, out_view if out_view is not None else target())

            return gemm
        if op == "layer_norm":
            out_view = None if fresh else arena_view(node.name, spec.shape)
            norm, eps = attrs["normalized_shape"], attrs["eps"]

            def ln(x, w=None, b=None):
                return kernels.layer_norm(x, norm, w, b, eps, out=out_view if out_view is not None else target())

            return ln
        if op == "sdpa":
            b_, h_, s_, d_ = spec.shape
            if bshd and not fresh:
                out_view = arena_view(node.name, (b_, s_, h_, d_)).transpose(1, 2)
            else:
                out_view = None if fresh else arena_view(node.name, spec.shape)
            causal, scale = attrs["is_causal"], attrs.get("scale")

            def attention(q, k, v, mask=None):
                return kernels.sdpa(q, k, v, mask, is_causal=causal, scale=scale,
                                    out=out_view if out_view is not None else target())

            return attention
        raise GraphError(f"no native kernel for op {op!r}")

    def _gemm_residual_step(self, gemm_node, add_node, arena_view) -> Callable:
        launch = self._gemm_launch(gemm_node)
        m, n = gemm_node.spec.shape
        spec = add_node.spec
        out2d = arena_view(add_node.name, (m, n)) if arena_view is not None else None

        def gemm_add(a, b, *rest):
            bias, resid = (rest[0], rest[1]) if len(rest) == 2 else (None, rest[0])
            out = out2d if out2d is not None else torch.empty((m, n), dtype=spec.dtype, device=spec.device)
            launch(a, b, bias, out, residual=resid.reshape(m, n))
            return out.view(spec.shape)

        return gemm_add

    # ------------------------------------------------------------ calls
    def __call__(self, *inputs: torch.Tensor):
        specs = self.graph.inputs
        if len(inputs) != len(specs):
            raise GraphError(f"expected {len(specs)} inputs, got {len(inputs)}")
        for (name, spec), t in zip(specs.items(), inputs):
            if not isinstance(t, torch.Tensor):
                raise GraphError("inputs must be torch.Tensor")
            if tuple(t.shape) != spec.shape:
                raise GraphError(f"input {name!r} shape {tuple(t.shape)} != expected {spec.shape}")
            if t.dtype != spec.dtype:
                raise GraphError(f"input {name!r} dtype {t.dtype} != expected {spec.dtype}")
            if str(t.device) != spec.device:
                raise GraphError(f"input {name!r} device {t.device} != expected {spec.device}")
        with torch.inference_mode():
            result = self._program.run(inputs)
        return tuple(result) if self.graph.output_is_tuple else result[0]

    def autotune(self, *inputs: torch.Tensor, warmup: int = 3, repeats: int = 10) -> dict:
        from forgeml_b200.forgeml.autotune import tune_graph

        report = tune_graph(self, inputs, warmup=warmup, repeats=repeats)
        self._lower()  # the chosen tiles take effect
        return report

    def kernel_source(self) -> str:
        return kernels.kernel_source()

    def node_times(self, *inputs: torch.Tensor, repeats: int = 20) -> dict[str, float]:
        """Device milliseconds of each instruction of the program: the
        instruction alone, ``repeats`` times back to back from one CUDA graph
        (operands from a preceding full run), best of three replays -- no
        host gaps, no overlap with other instructions.  View-only
        instructions launch nothing and report ~0.  A fused residual add
        reports under the add's name."""
        prog = self._program
        dev = next(t.device for t in inputs)
        vals: list = [None] * prog.n_values
        with torch.inference_mode():
            for vid, t in zip(prog.inputs, inputs):
                vals[vid] = t
            for vid, t in prog.constants:
                vals[vid] = t
            for fn, arg_ids, out_id, _ in prog.instrs:  # keep every value: each instruction is replayed alone
                vals[out_id] = fn(*[vals[i] for i in arg_ids])
            torch.cuda.synchronize(dev)
            times: dict[str, float] = {}
            for name, (fn, arg_ids, _, _) in zip(self._instr_names, prog.instrs):
                args = [vals[i] for i in arg_ids]
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    fn(*args)
                torch.cuda.current_stream(dev).wait_stream(side)
                torch.cuda.synchronize(dev)
                graph = torch.cuda.CUDAGraph()
                with warnings.catch_warnings():  # view-only instructions capture an empty graph
                    warnings.simplefilter("ignore", UserWarning)
                    with torch.cuda.graph(graph):
                        for _ in range(repeats):
                            fn(*args)
                graph.replay()
                torch.cuda.synchronize(dev)
                best = float("inf")
                for _ in range(3):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    graph.replay()
                    e1.record()
                    e1.synchronize()
                    best = min(best, e0.elapsed_time(e1) / repeats)
                times[name] = best
                del graph
        return times

    def explain(self) -> dict:
        return {
            "backend": self.backend,
            "original_nodes": len(self.original_graph.nodes),
            "optimized_nodes": len(self.graph.nodes),
            "passes": [{"name": p.name, "nodes_before": p.nodes_before, "nodes_after": p.nodes_after}
                       for p in self.passes],
            "memory_plan": self.memory_plan.to_dict(),
            "execution_plan": self.execution_plan.to_dict(),
            "native_fusions": self.fusions,
            "graph": self.graph.to_dict(),
            "kernel_plan": dict(self.kernel_plan),
            "kernel_configs": {k: asdict(v) for k, v in self.kernel_configs.items()},
        }

    @property
    def ext_plan(self) -> MemoryPlan:
        """The arena the program runs over (kept under the former name)."""
        return self.execution_plan


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
    records: list[PassRecord] = []
    if optimize:
        graph, records = optimize_graph(graph)
    else:
        graph.validate()
    return CompiledModel(graph, original, plan_memory(graph), records, backend,
                         kernel_plan=kernels.select_kernels(graph, backend))
