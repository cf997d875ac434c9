"""Graph IR consumed by the compiled-forward dispatch.

Same data model as the reference IR (src/forgeml/ir.py:29-75 TensorSpec/Node,
:390-510 Graph, :513-571 GraphBuilder) so that graphs, memory plans and
``to_dict()`` outputs compare one to one.  Spec inference evaluates each op on
meta tensors (no device work), after structural checks that mirror the
reference's rules in src/forgeml/ir.py:148-383.
"""

from __future__ import annotations

import copy
import math
from dataclasses import dataclass
from typing import Any

import torch


class GraphError(ValueError):
    pass


SUPPORTED_DTYPES = frozenset(
    {
        torch.float16,
        torch.bfloat16,
        torch.float32,
        torch.float64,
        torch.int8,
        torch.int16,
        torch.int32,
        torch.int64,
        torch.uint8,
        torch.bool,
    }
)


def _is_int(v: Any) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


@dataclass(frozen=True)
class TensorSpec:
    shape: tuple[int, ...]
    dtype: torch.dtype
    device: str

    def __post_init__(self) -> None:
        if not isinstance(self.shape, tuple) or not all(_is_int(d) for d in self.shape):
            raise GraphError(f"shape must be a tuple of ints, got {self.shape!r}")
        if any(d <= 0 for d in self.shape):
            raise GraphError(f"shape dims must be positive integers, got {self.shape!r}")
        if not isinstance(self.dtype, torch.dtype):
            raise GraphError(f"dtype must be a torch.dtype, got {self.dtype!r}")
        if self.dtype not in SUPPORTED_DTYPES:
            raise GraphError(f"unsupported dtype {self.dtype}")
        if not isinstance(self.device, str) or not self.device:
            raise GraphError(f"device must be a non-empty string, got {self.device!r}")
        try:
            dev = torch.device(self.device)
        except (RuntimeError, TypeError) as e:
            raise GraphError(f"invalid device {self.device!r}") from e
        if dev.type == "cuda" and dev.index is None:
            object.__setattr__(self, "device", "cuda:0")

    @property
    def nbytes(self) -> int:
        return math.prod(self.shape) * self.dtype.itemsize

    def to_dict(self) -> dict:
        return {
            "shape": list(self.shape),
            "dtype": str(self.dtype).replace("torch.", ""),
            "device": self.device,
        }


@dataclass(frozen=True)
class Node:
    name: str
    op: str
    inputs: tuple[str, ...]
    attrs: dict[str, Any]
    spec: TensorSpec


def spec_of(t: torch.Tensor, device: str | None = None) -> TensorSpec:
    return TensorSpec(tuple(t.shape), t.dtype, device or str(t.device))


# op -> (allowed attrs, required attrs, accepted arities)
_OP_TABLE: dict[str, tuple[frozenset, frozenset, tuple[int, ...]]] = {
    "matmul": (frozenset(), frozenset(), (2,)),
    "linear": (frozenset(), frozenset(), (2, 3)),
    "add": (frozenset(), frozenset(), (2,)),
    "mul": (frozenset(), frozenset(), (2,)),
    "relu": (frozenset(), frozenset(), (1,)),
    "gelu": (frozenset({"approximate"}), frozenset(), (1,)),
    "reshape": (frozenset({"shape"}), frozenset({"shape"}), (1,)),
    "transpose": (frozenset({"dim0", "dim1"}), frozenset({"dim0", "dim1"}), (1,)),
    "softmax": (frozenset({"dim"}), frozenset({"dim"}), (1,)),
    "narrow": (frozenset({"dim", "start", "length"}), frozenset({"dim", "start", "length"}), (1,)),
    "fused_linear_gelu": (frozenset({"approximate"}), frozenset(), (2, 3)),
    "layer_norm": (frozenset({"normalized_shape", "eps"}), frozenset({"normalized_shape", "eps"}), (1, 3)),
    "sdpa": (frozenset({"is_causal", "scale"}), frozenset({"is_causal"}), (3, 4)),
    "conv2d": (
        frozenset({"stride", "padding", "dilation", "groups"}),
        frozenset({"stride", "padding", "dilation", "groups"}),
        (2, 3),
    ),
    "embedding": (frozenset(), frozenset(), (2,)),
}
_FLOAT_ONLY = {"gelu", "softmax", "fused_linear_gelu", "layer_norm", "sdpa", "conv2d"}


def _check_rank2_product(op: str, a: TensorSpec, b: TensorSpec) -> None:
    if len(a.shape) != 2 or len(b.shape) != 2:
        kind = "matmul inputs" if op != "linear" else "input and weight tensors"
        raise GraphError(f"{op} requires rank-2 {kind}")
    if a.dtype != b.dtype:
        raise GraphError(f"{op} dtype mismatch {a.dtype} vs {b.dtype}")
    if a.dtype == torch.bool:
        raise GraphError(f"{op} does not support bool inputs")
    if a.shape[1] != b.shape[0]:
        raise GraphError(f"{op} shape mismatch {a.shape} x {b.shape}")


def _check_bias(op: str, bias: TensorSpec, width: int, dtype: torch.dtype) -> None:
    if len(bias.shape) != 1 or bias.shape[0] != width:
        raise GraphError(f"{op} bias must be a 1-D tensor of output width")
    if bias.dtype != dtype:
        raise GraphError(f"{op} bias dtype mismatch")


def _check_dim(name: str, v: Any, rank: int) -> None:
    if not _is_int(v) or not -rank <= v < rank:
        raise GraphError(f"{name}={v!r} out of range for rank {rank}")


def _pair(value: Any, name: str, positive: bool) -> tuple[int, int]:
    if _is_int(value):
        pair = (value, value)
    elif isinstance(value, (tuple, list)) and len(value) == 2 and all(_is_int(v) for v in value):
        pair = tuple(value)
    else:
        raise GraphError(f"conv2d {name} must be an int or pair of ints, got {value!r}")
    lo = 1 if positive else 0
    if any(v < lo for v in pair):
        raise GraphError(f"conv2d {name} values must be {'positive' if positive else 'non-negative'}")
    return pair


def _structural_checks(op: str, specs: list[TensorSpec], attrs: dict) -> None:
    if op in ("matmul", "linear", "fused_linear_gelu"):
        _check_rank2_product(op, specs[0], specs[1])
        if len(specs) == 3:
            _check_bias(op, specs[2], specs[1].shape[1], specs[0].dtype)
    if op in ("add", "mul"):
        a, b = specs
        if a.dtype != b.dtype and a.shape != () and b.shape != ():
            raise GraphError(f"{op} dtype mismatch")
    if op in ("gelu", "fused_linear_gelu") and attrs.get("approximate", "none") not in ("none", "tanh"):
        raise GraphError(f"{op} approximate must be 'none' or 'tanh'")
    if op == "reshape":
        shape = attrs["shape"]
        if not isinstance(shape, (tuple, list)) or not all(_is_int(d) and d > 0 for d in shape):
            raise GraphError(f"reshape shape must be positive ints, got {shape!r}")
        if math.prod(shape) != math.prod(specs[0].shape):
            raise GraphError(f"reshape numel mismatch {specs[0].shape} -> {tuple(shape)}")
    if op == "transpose":
        for key in ("dim0", "dim1"):
            _check_dim(f"transpose {key}", attrs[key], len(specs[0].shape))
    if op == "softmax":
        _check_dim("softmax dim", attrs["dim"], len(specs[0].shape))
    if op == "narrow":
        x = specs[0]
        rank = len(x.shape)
        for key in ("dim", "start", "length"):
            if not _is_int(attrs[key]):
                raise GraphError(f"narrow {key} must be an int, got {attrs[key]!r}")
        if rank == 0 or not -rank <= attrs["dim"] < rank:
            raise GraphError(f"narrow dim={attrs['dim']!r} out of range for rank {rank}")
        d = attrs["dim"] % rank
        if attrs["length"] <= 0 or attrs["start"] < 0 or attrs["start"] + attrs["length"] > x.shape[d]:
            raise GraphError("narrow range exceeds the dimension")
    if op == "layer_norm":
        norm = attrs["normalized_shape"]
        if _is_int(norm):
            norm = (norm,)
        if not isinstance(norm, (tuple, list)) or not norm or not all(_is_int(d) and d > 0 for d in norm):
            raise GraphError(f"layer_norm normalized_shape must be positive ints, got {norm!r}")
        norm = tuple(norm)
        x = specs[0]
        if len(x.shape) < len(norm) or x.shape[-len(norm):] != norm:
            raise GraphError(f"layer_norm shape {x.shape} does not end with {norm!r}")
        if len(specs) == 3:
            w, b = specs[1:]
            if w.shape != norm or b.shape != norm:
                raise GraphError("layer_norm weight/bias must match normalized_shape")
            if not (x.dtype == w.dtype == b.dtype):
                raise GraphError("layer_norm dtype mismatch")
        eps = attrs["eps"]
        if not isinstance(eps, (int, float)) or isinstance(eps, bool) or not math.isfinite(float(eps)) or eps <= 0:
            raise GraphError("layer_norm eps must be a finite positive number")
    if op == "sdpa":
        q, k, v = specs[:3]
        if not (len(q.shape) == len(k.shape) == len(v.shape) == 4):
            raise GraphError("sdpa requires rank-4 [batch, heads, sequence, dim] tensors")
        if q.shape[:2] != k.shape[:2] or k.shape != v.shape or q.shape[3] != k.shape[3]:
            raise GraphError("sdpa batch/head/key-value shapes are incompatible")
        if not (q.dtype == k.dtype == v.dtype):
            raise GraphError("sdpa dtype mismatch")
        if not isinstance(attrs["is_causal"], bool):
            raise GraphError("sdpa is_causal must be a bool")
        if len(specs) == 4:
            mask = specs[3]
            if attrs["is_causal"]:
                raise GraphError("sdpa attn_mask cannot be combined with is_causal")
            if mask.dtype != torch.bool and mask.dtype != q.dtype:
                raise GraphError("sdpa attn_mask must be bool or match the query dtype")
            target = (q.shape[0], q.shape[1], q.shape[2], k.shape[2])
            try:
                merged = torch.broadcast_shapes(mask.shape, target)
            except RuntimeError as e:
                raise GraphError(f"sdpa attn_mask shape {mask.shape} cannot broadcast to {target}") from e
            if merged != target:
                raise GraphError(f"sdpa attn_mask shape {mask.shape} cannot broadcast to {target}")
        scale = attrs.get("scale")
        if scale is not None and (
            not isinstance(scale, (int, float)) or isinstance(scale, bool)
            or not math.isfinite(float(scale)) or scale <= 0
        ):
            raise GraphError("sdpa scale must be a finite positive number or None")
    if op == "conv2d":
        x, w = specs[:2]
        if len(x.shape) != 4 or len(w.shape) != 4:
            raise GraphError("conv2d requires NCHW input and OIHW weight tensors")
        g = attrs["groups"]
        if not _is_int(g) or g <= 0:
            raise GraphError("conv2d groups must be a positive integer")
        if x.shape[1] % g or w.shape[0] % g or x.shape[1] != w.shape[1] * g:
            raise GraphError("conv2d channels/groups are incompatible")
        if len(specs) == 3 and (len(specs[2].shape) != 1 or specs[2].shape[0] != w.shape[0]):
            raise GraphError("conv2d bias must be a 1-D tensor of output channels")
        if x.dtype != w.dtype:
            raise GraphError("conv2d dtype mismatch")
        _pair(attrs["stride"], "stride", True)
        _pair(attrs["padding"], "padding", False)
        _pair(attrs["dilation"], "dilation", True)
    if op == "embedding":
        idx, w = specs
        if idx.dtype != torch.int64:
            raise GraphError("embedding indices must be int64")
        if len(w.shape) != 2:
            raise GraphError("embedding weight must be rank-2 [vocab, dim]")


def _result_device(op: str, specs: list[TensorSpec]) -> str:
    if op in ("add", "mul") and all(len(s.shape) == 0 for s in specs):
        return next((s.device for s in specs if torch.device(s.device).type != "cpu"), specs[0].device)
    return next((s.device for s in specs if len(s.shape) > 0), specs[0].device)


def infer_spec(op: str, input_specs: list[TensorSpec], attrs: dict[str, Any]) -> TensorSpec:
    from forgeml_b200.forgeml.ops import evaluate

    if op not in _OP_TABLE:
        raise GraphError(f"unsupported op {op!r}")
    if not isinstance(attrs, dict):
        raise GraphError(f"op {op!r} attrs must be a dict, got {type(attrs).__name__}")
    allowed, required, arity = _OP_TABLE[op]
    extra = set(attrs) - allowed
    if extra:
        raise GraphError(f"op {op!r} got unsupported attrs {sorted(extra)}")
    missing = required - set(attrs)
    if missing:
        raise GraphError(f"op {op!r} requires attrs {sorted(missing)}")
    if len(input_specs) not in arity:
        raise GraphError(
            f"op {op!r} expects {'/'.join(map(str, arity))} inputs, got {len(input_specs)}"
        )
    if op in _FLOAT_ONLY:
        gated = input_specs[:3] if op == "sdpa" else input_specs
        if any(not s.dtype.is_floating_point for s in gated):
            raise GraphError(f"op {op!r} requires floating-point inputs")
    _structural_checks(op, input_specs, attrs)
    devices = {s.device for s in input_specs}
    if len(devices) > 1:
        scalar_ok = op in ("add", "mul") and any(
            s.shape == () and torch.device(s.device).type == "cpu" for s in input_specs
        )
        if not scalar_ok:
            raise GraphError(f"{op} device mismatch {sorted(devices)}")
    try:
        metas = tuple(torch.empty(s.shape, dtype=s.dtype, device="meta") for s in input_specs)
        out = evaluate(op, metas, dict(attrs))
    except GraphError:
        raise
    except Exception as e:  # noqa: BLE001 - surface any torch shape error as a graph error
        raise GraphError(f"op {op!r} failed spec inference: {e}") from e
    return TensorSpec(tuple(out.shape), out.dtype, _result_device(op, input_specs))


@dataclass
class Graph:
    inputs: dict[str, TensorSpec]
    constants: dict[str, torch.Tensor]
    nodes: list[Node]
    outputs: tuple[str, ...]
    output_is_tuple: bool = False

    def specs(self) -> dict[str, TensorSpec]:
        out = dict(self.inputs)
        out.update({k: spec_of(v) for k, v in self.constants.items()})
        out.update({n.name: n.spec for n in self.nodes})
        return out

    def validate(self) -> None:
        seen: set[str] = set()
        for name in list(self.inputs) + list(self.constants):
            if not isinstance(name, str) or not name:
                raise GraphError("value names must be non-empty strings")
            if name in seen:
                raise GraphError(f"duplicate name {name!r}")
            seen.add(name)
        for name, spec in self.inputs.items():
            if not isinstance(spec, TensorSpec):
                raise GraphError(f"input {name!r} spec must be a TensorSpec")
        env = dict(self.inputs)
        for name, t in self.constants.items():
            if not isinstance(t, torch.Tensor):
                raise GraphError(f"constant {name!r} is not a torch.Tensor")
            env[name] = spec_of(t)
        for node in self.nodes:
            if not isinstance(node.name, str) or not node.name:
                raise GraphError("node names must be non-empty strings")
            if not isinstance(node.spec, TensorSpec):
                raise GraphError(f"node {node.name!r} spec must be a TensorSpec")
            if node.name in seen:
                raise GraphError(f"duplicate name {node.name!r}")
            seen.add(node.name)
            for i in node.inputs:
                if i not in env:
                    raise GraphError(f"node {node.name!r} input {i!r} is not defined before use")
            if not isinstance(node.attrs, dict):
                raise GraphError(f"node {node.name!r} attrs must be a dict, got {type(node.attrs).__name__}")
            try:
                spec = infer_spec(node.op, [env[i] for i in node.inputs], dict(node.attrs))
            except GraphError as e:
                raise GraphError(f"node {node.name!r}: {e}") from e
            if spec != node.spec:
                raise GraphError(f"node {node.name!r} spec mismatch: declared {node.spec}, inferred {spec}")
            env[node.name] = node.spec
        if not self.outputs:
            raise GraphError("graph outputs must be non-empty")
        if not isinstance(self.output_is_tuple, bool):
            raise GraphError("output_is_tuple must be a bool")
        if len(self.outputs) > 1 and not self.output_is_tuple:
            raise GraphError("multiple graph outputs require output_is_tuple=True")
        for name in self.outputs:
            if name not in env:
                raise GraphError(f"graph output {name!r} is not defined")

    def clone(self) -> Graph:
        return Graph(
            inputs=dict(self.inputs),
            constants={k: v.detach().clone() for k, v in self.constants.items()},
            nodes=[Node(n.name, n.op, tuple(n.inputs), copy.deepcopy(n.attrs), n.spec) for n in self.nodes],
            outputs=tuple(self.outputs),
            output_is_tuple=self.output_is_tuple,
        )

    def to_dict(self) -> dict:
        def attr(v):
            return list(v) if isinstance(v, tuple) else v

        return {
            "inputs": {k: v.to_dict() for k, v in self.inputs.items()},
            "constants": {k: spec_of(v).to_dict() for k, v in self.constants.items()},
            "nodes": [
                {
                    "name": n.name,
                    "op": n.op,
                    "inputs": list(n.inputs),
                    "attrs": {k: attr(v) for k, v in n.attrs.items()},
                    "spec": n.spec.to_dict(),
                }
                for n in self.nodes
            ],
            "outputs": list(self.outputs),
            "output_is_tuple": self.output_is_tuple,
        }


class GraphBuilder:
    def __init__(self, inputs: dict[str, TensorSpec]):
        self._inputs = dict(inputs)
        for name, spec in self._inputs.items():
            if not isinstance(name, str) or not name:
                raise GraphError("input names must be non-empty strings")
            if not isinstance(spec, TensorSpec):
                raise GraphError(f"input {name!r} spec must be a TensorSpec")
        self._constants: dict[str, torch.Tensor] = {}
        self._nodes: list[Node] = []
        self._names = set(self._inputs)
        self._env: dict[str, TensorSpec] = dict(self._inputs)

    def _claim(self, name: str) -> None:
        if not isinstance(name, str) or not name:
            raise GraphError("names must be non-empty strings")
        if name in self._names:
            raise GraphError(f"duplicate name {name!r}")
        self._names.add(name)

    def spec(self, name: str) -> TensorSpec:
        return self._env[name]

    def constant(self, name: str, value: torch.Tensor) -> str:
        self._claim(name)
        if not isinstance(value, torch.Tensor):
            raise GraphError(f"constant {name!r} must be a torch.Tensor")
        spec = spec_of(value)
        self._constants[name] = value.detach().clone()
        self._env[name] = spec
        return name

    def add(self, name: str, op: str, inputs: tuple[str, ...], **attrs) -> str:
        self._claim(name)
        for i in inputs:
            if i not in self._env:
                self._names.discard(name)
                raise GraphError(f"node {name!r} input {i!r} is not defined")
        try:
            spec = infer_spec(op, [self._env[i] for i in inputs], attrs)
        except GraphError as e:
            self._names.discard(name)
            raise GraphError(f"node {name!r}: {e}") from e
        self._nodes.append(Node(name, op, tuple(inputs), dict(attrs), spec))
        self._env[name] = spec
        return name

    def finish(self, outputs: tuple[str, ...], output_is_tuple: bool = False) -> Graph:
        g = Graph(
            inputs=dict(self._inputs),
            constants=dict(self._constants),
            nodes=list(self._nodes),
            outputs=tuple(outputs),
            output_is_tuple=output_is_tuple or len(outputs) > 1,
        )
        g.validate()
        return g
