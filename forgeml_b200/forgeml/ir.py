"""Graph IR of the compiled forward pass.

The data model is the reference IR's public one (src/forgeml/ir.py:29-75,
390-571): ``TensorSpec(shape, dtype, device)``, ``Node(name, op, inputs,
attrs, spec)``, ``Graph(inputs, constants, nodes, outputs, output_is_tuple)``
with ``specs``, ``validate``, ``clone``, ``to_dict`` and ``GraphBuilder``;
graphs and their dictionaries compare one to one with the reference's, so
memory plans can be checked bit for bit.

Each op is described once in ``_SCHEMAS``: its arity, attributes, whether its
operands must be floating point, and a structural check that raises
GraphError with the reference's conditions.  A node's result spec is then
obtained by running the op's torch semantics (ops.evaluate) on meta tensors:
no device work, and torch's own shape rules decide the rest.
"""

from __future__ import annotations

import copy
import math
from dataclasses import dataclass, field
from typing import Any, Callable

import torch


class GraphError(ValueError):
    pass


SUPPORTED_DTYPES = frozenset({torch.float16, torch.bfloat16, torch.float32, torch.float64, torch.int8, torch.int16,
                              torch.int32, torch.int64, torch.uint8, torch.bool})


def _int(v: Any) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _positive_real(v: Any) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(float(v)) and v > 0


@dataclass(frozen=True)
class TensorSpec:
    shape: tuple[int, ...]
    dtype: torch.dtype
    device: str

    def __post_init__(self) -> None:
        if not isinstance(self.shape, tuple) or not all(_int(d) for d in self.shape):
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
        if dev.type == "cuda" and dev.index is None:  # "cuda" names the first GPU
            object.__setattr__(self, "device", "cuda:0")

    @property
    def nbytes(self) -> int:
        return math.prod(self.shape) * self.dtype.itemsize

    def to_dict(self) -> dict:
        return {"shape": list(self.shape), "dtype": str(self.dtype).replace("torch.", ""), "device": self.device}


@dataclass(frozen=True)
class Node:
    name: str
    op: str
    inputs: tuple[str, ...]
    attrs: dict[str, Any]
    spec: TensorSpec


def spec_of(t: torch.Tensor, device: str | None = None) -> TensorSpec:
    return TensorSpec(tuple(t.shape), t.dtype, device or str(t.device))


# ----------------------------------------------------------------- op schemas
@dataclass(frozen=True)
class _Schema:
    arity: tuple[int, ...]
    attrs: frozenset = frozenset()
    required: frozenset = frozenset()
    float_operands: int = 0  # leading operands that must be floating point (0: none checked)
    check: Callable[[list[TensorSpec], dict], None] | None = field(default=None, compare=False)


def _dim_ok(label: str, v: Any, rank: int) -> None:
    if not _int(v) or not -rank <= v < rank:
        raise GraphError(f"{label}={v!r} out of range for rank {rank}")


def _check_product(op: str) -> Callable:
    def check(s: list[TensorSpec], attrs: dict) -> None:
        a, b = s[0], s[1]
        if len(a.shape) != 2 or len(b.shape) != 2:
            what = "input and weight tensors" if op == "linear" else "matmul inputs"
            raise GraphError(f"{op} requires rank-2 {what}")
        if a.dtype != b.dtype:
            raise GraphError(f"{op} dtype mismatch {a.dtype} vs {b.dtype}")
        if a.dtype == torch.bool:
            raise GraphError(f"{op} does not support bool inputs")
        if a.shape[1] != b.shape[0]:
            raise GraphError(f"{op} shape mismatch {a.shape} x {b.shape}")
        if len(s) == 3:
            if len(s[2].shape) != 1 or s[2].shape[0] != b.shape[1]:
                raise GraphError(f"{op} bias must be a 1-D tensor of output width")
            if s[2].dtype != a.dtype:
                raise GraphError(f"{op} bias dtype mismatch")
        if attrs.get("approximate", "none") not in ("none", "tanh"):
            raise GraphError(f"{op} approximate must be 'none' or 'tanh'")

    return check


def _check_binary(op: str) -> Callable:
    def check(s, _):
        if s[0].dtype != s[1].dtype and s[0].shape != () and s[1].shape != ():
            raise GraphError(f"{op} dtype mismatch")

    return check


def _check_gelu(_, attrs):
    if attrs.get("approximate", "none") not in ("none", "tanh"):
        raise GraphError("gelu approximate must be 'none' or 'tanh'")


def _check_reshape(s, attrs):
    shape = attrs["shape"]
    if not isinstance(shape, (tuple, list)) or not all(_int(d) and d > 0 for d in shape):
        raise GraphError(f"reshape shape must be positive ints, got {shape!r}")
    if math.prod(shape) != math.prod(s[0].shape):
        raise GraphError(f"reshape numel mismatch {s[0].shape} -> {tuple(shape)}")


def _check_transpose(s, attrs):
    for key in ("dim0", "dim1"):
        _dim_ok(f"transpose {key}", attrs[key], len(s[0].shape))


def _check_softmax(s, attrs):
    _dim_ok("softmax dim", attrs["dim"], len(s[0].shape))


def _check_narrow(s, attrs):
    rank = len(s[0].shape)
    for key in ("dim", "start", "length"):
        if not _int(attrs[key]):
            raise GraphError(f"narrow {key} must be an int, got {attrs[key]!r}")
    if rank == 0 or not -rank <= attrs["dim"] < rank:
        raise GraphError(f"narrow dim={attrs['dim']!r} out of range for rank {rank}")
    extent = s[0].shape[attrs["dim"] % rank]
    if attrs["length"] <= 0 or attrs["start"] < 0 or attrs["start"] + attrs["length"] > extent:
        raise GraphError("narrow range exceeds the dimension")


def _check_layer_norm(s, attrs):
    norm = attrs["normalized_shape"]
    norm = (norm,) if _int(norm) else norm
    if not isinstance(norm, (tuple, list)) or not norm or not all(_int(d) and d > 0 for d in norm):
        raise GraphError(f"layer_norm normalized_shape must be positive ints, got {norm!r}")
    norm = tuple(norm)
    x = s[0]
    if len(x.shape) < len(norm) or x.shape[-len(norm):] != norm:
        raise GraphError(f"layer_norm shape {x.shape} does not end with {norm!r}")
    if len(s) == 3:
        if s[1].shape != norm or s[2].shape != norm:
            raise GraphError("layer_norm weight/bias must match normalized_shape")
        if not (x.dtype == s[1].dtype == s[2].dtype):
            raise GraphError("layer_norm dtype mismatch")
    if not _positive_real(attrs["eps"]):
        raise GraphError("layer_norm eps must be a finite positive number")


def _check_sdpa(s, attrs):
    q, k, v = s[:3]
    if not all(len(t.shape) == 4 for t in (q, k, v)):
        raise GraphError("sdpa requires rank-4 [batch, heads, sequence, dim] tensors")
    if q.shape[:2] != k.shape[:2] or k.shape != v.shape or q.shape[3] != k.shape[3]:
        raise GraphError("sdpa batch/head/key-value shapes are incompatible")
    if not (q.dtype == k.dtype == v.dtype):
        raise GraphError("sdpa dtype mismatch")
    if not isinstance(attrs["is_causal"], bool):
        raise GraphError("sdpa is_causal must be a bool")
    if len(s) == 4:
        mask = s[3]
        if attrs["is_causal"]:
            raise GraphError("sdpa attn_mask cannot be combined with is_causal")
        if mask.dtype not in (torch.bool, q.dtype):
            raise GraphError("sdpa attn_mask must be bool or match the query dtype")
        full = (q.shape[0], q.shape[1], q.shape[2], k.shape[2])
        try:
            ok = torch.broadcast_shapes(mask.shape, full) == full
        except RuntimeError:
            ok = False
        if not ok:
            raise GraphError(f"sdpa attn_mask shape {mask.shape} cannot broadcast to {full}")
    scale = attrs.get("scale")
    if scale is not None and not _positive_real(scale):
        raise GraphError("sdpa scale must be a finite positive number or None")


def _pair_ok(value: Any, name: str, least: int) -> None:
    pair = (value, value) if _int(value) else value
    if not (isinstance(pair, (tuple, list)) and len(pair) == 2 and all(_int(v) for v in pair)):
        raise GraphError(f"conv2d {name} must be an int or pair of ints, got {value!r}")
    if any(v < least for v in pair):
        raise GraphError(f"conv2d {name} values must be {'positive' if least else 'non-negative'}")


def _check_conv2d(s, attrs):
    x, w = s[:2]
    if len(x.shape) != 4 or len(w.shape) != 4:
        raise GraphError("conv2d requires NCHW input and OIHW weight tensors")
    g = attrs["groups"]
    if not _int(g) or g <= 0:
        raise GraphError("conv2d groups must be a positive integer")
    if x.shape[1] % g or w.shape[0] % g or x.shape[1] != w.shape[1] * g:
        raise GraphError("conv2d channels/groups are incompatible")
    if len(s) == 3 and (len(s[2].shape) != 1 or s[2].shape[0] != w.shape[0]):
        raise GraphError("conv2d bias must be a 1-D tensor of output channels")
    if x.dtype != w.dtype:
        raise GraphError("conv2d dtype mismatch")
    _pair_ok(attrs["stride"], "stride", 1)
    _pair_ok(attrs["padding"], "padding", 0)
    _pair_ok(attrs["dilation"], "dilation", 1)


def _check_embedding(s, _):
    if s[0].dtype != torch.int64:
        raise GraphError("embedding indices must be int64")
    if len(s[1].shape) != 2:
        raise GraphError("embedding weight must be rank-2 [vocab, dim]")


def _fs(*names) -> frozenset:
    return frozenset(names)


_CONV = _fs("stride", "padding", "dilation", "groups")
_SCHEMAS: dict[str, _Schema] = {
    "matmul": _Schema((2,), check=_check_product("matmul")),
    "linear": _Schema((2, 3), check=_check_product("linear")),
    "fused_linear_gelu": _Schema((2, 3), _fs("approximate"), float_operands=3, check=_check_product("fused_linear_gelu")),
    "add": _Schema((2,), check=_check_binary("add")),
    "mul": _Schema((2,), check=_check_binary("mul")),
    "relu": _Schema((1,)),
    "gelu": _Schema((1,), _fs("approximate"), float_operands=1, check=_check_gelu),
    "reshape": _Schema((1,), _fs("shape"), _fs("shape"), check=_check_reshape),
    "transpose": _Schema((1,), _fs("dim0", "dim1"), _fs("dim0", "dim1"), check=_check_transpose),
    "softmax": _Schema((1,), _fs("dim"), _fs("dim"), float_operands=1, check=_check_softmax),
    "narrow": _Schema((1,), _fs("dim", "start", "length"), _fs("dim", "start", "length"), check=_check_narrow),
    "layer_norm": _Schema((1, 3), _fs("normalized_shape", "eps"), _fs("normalized_shape", "eps"), float_operands=3,
                          check=_check_layer_norm),
    "sdpa": _Schema((3, 4), _fs("is_causal", "scale"), _fs("is_causal"), float_operands=3, check=_check_sdpa),
    "conv2d": _Schema((2, 3), _CONV, _CONV, float_operands=3, check=_check_conv2d),
    "embedding": _Schema((2,), check=_check_embedding),
}


def _result_device(op: str, specs: list[TensorSpec]) -> str:
    # a 0-d CPU scalar operand never decides where the result lives
    if op in ("add", "mul") and all(not s.shape for s in specs):
        return next((s.device for s in specs if torch.device(s.device).type != "cpu"), specs[0].device)
    return next((s.device for s in specs if s.shape), specs[0].device)


def infer_spec(op: str, input_specs: list[TensorSpec], attrs: dict[str, Any]) -> TensorSpec:
    from forgeml_b200.forgeml.ops import evaluate

    schema = _SCHEMAS.get(op)
    if schema is None:
        raise GraphError(f"unsupported op {op!r}")
    if not isinstance(attrs, dict):
        raise GraphError(f"op {op!r} attrs must be a dict, got {type(attrs).__name__}")
    if set(attrs) - schema.attrs:
        raise GraphError(f"op {op!r} got unsupported attrs {sorted(set(attrs) - schema.attrs)}")
    if schema.required - set(attrs):
        raise GraphError(f"op {op!r} requires attrs {sorted(schema.required - set(attrs))}")
    if len(input_specs) not in schema.arity:
        raise GraphError(f"op {op!r} expects {'/'.join(map(str, schema.arity))} inputs, got {len(input_specs)}")
    if schema.float_operands and not all(s.dtype.is_floating_point for s in input_specs[:schema.float_operands]):
        raise GraphError(f"op {op!r} requires floating-point inputs")
    if schema.check is not None:
        schema.check(input_specs, attrs)
    devices = {s.device for s in input_specs}
    if len(devices) > 1 and not (op in ("add", "mul") and any(
            not s.shape and torch.device(s.device).type == "cpu" for s in input_specs)):
        raise GraphError(f"{op} device mismatch {sorted(devices)}")
    try:
        metas = tuple(torch.empty(s.shape, dtype=s.dtype, device="meta") for s in input_specs)
        out = evaluate(op, metas, dict(attrs))
    except GraphError:
        raise
    except Exception as e:  # noqa: BLE001 - torch's shape errors become graph errors
        raise GraphError(f"op {op!r} failed spec inference: {e}") from e
    return TensorSpec(tuple(out.shape), out.dtype, _result_device(op, input_specs))


# ----------------------------------------------------------------- graphs
def _value_name_ok(name: Any) -> bool:
    return isinstance(name, str) and bool(name)


@dataclass
class Graph:
    inputs: dict[str, TensorSpec]
    constants: dict[str, torch.Tensor]
    nodes: list[Node]
    outputs: tuple[str, ...]
    output_is_tuple: bool = False

    def specs(self) -> dict[str, TensorSpec]:
        env = dict(self.inputs)
        env.update((k, spec_of(v)) for k, v in self.constants.items())
        env.update((n.name, n.spec) for n in self.nodes)
        return env

    def validate(self) -> None:
        names: set[str] = set()

        def claim(name, what="value"):
            if not _value_name_ok(name):
                raise GraphError(f"{what} names must be non-empty strings")
            if name in names:
                raise GraphError(f"duplicate name {name!r}")
            names.add(name)

        env: dict[str, TensorSpec] = {}
        for name, spec in self.inputs.items():
            claim(name)
            if not isinstance(spec, TensorSpec):
                raise GraphError(f"input {name!r} spec must be a TensorSpec")
            env[name] = spec
        for name, t in self.constants.items():
            claim(name)
            if not isinstance(t, torch.Tensor):
                raise GraphError(f"constant {name!r} is not a torch.Tensor")
            env[name] = spec_of(t)
        for node in self.nodes:
            claim(node.name, "node")
            if not isinstance(node.spec, TensorSpec):
                raise GraphError(f"node {node.name!r} spec must be a TensorSpec")
            undefined = next((i for i in node.inputs if i not in env), None)
            if undefined is not None:
                raise GraphError(f"node {node.name!r} input {undefined!r} is not defined before use")
            if not isinstance(node.attrs, dict):
                raise GraphError(f"node {node.name!r} attrs must be a dict, got {type(node.attrs).__name__}")
            try:
                spec = infer_spec(node.op, [env[i] for i in node.inputs], dict(node.attrs))
            except GraphError as e:
                raise GraphError(f"node {node.name!r}: {e}") from e
            if spec != node.spec:
                raise GraphError(f"node {node.name!r} spec mismatch: declared {node.spec}, inferred {spec}")
            env[node.name] = spec
        if not self.outputs:
            raise GraphError("graph outputs must be non-empty")
        if not isinstance(self.output_is_tuple, bool):
            raise GraphError("output_is_tuple must be a bool")
        if len(self.outputs) > 1 and not self.output_is_tuple:
            raise GraphError("multiple graph outputs require output_is_tuple=True")
        missing = next((o for o in self.outputs if o not in env), None)
        if missing is not None:
            raise GraphError(f"graph output {missing!r} is not defined")

    def clone(self) -> Graph:
        return Graph(dict(self.inputs), {k: v.detach().clone() for k, v in self.constants.items()},
                     [Node(n.name, n.op, tuple(n.inputs), copy.deepcopy(n.attrs), n.spec) for n in self.nodes],
                     tuple(self.outputs), self.output_is_tuple)

    def to_dict(self) -> dict:
        def plain(v):
            return list(v) if isinstance(v, tuple) else v

        return {
            "inputs": {k: v.to_dict() for k, v in self.inputs.items()},
            "constants": {k: spec_of(v).to_dict() for k, v in self.constants.items()},
            "nodes": [{"name": n.name, "op": n.op, "inputs": list(n.inputs),
                       "attrs": {k: plain(v) for k, v in n.attrs.items()}, "spec": n.spec.to_dict()}
                      for n in self.nodes],
            "outputs": list(self.outputs),
            "output_is_tuple": self.output_is_tuple,
        }


class GraphBuilder:
    """Appends nodes with inferred specs; ``finish`` returns a validated Graph."""

    def __init__(self, inputs: dict[str, TensorSpec]):
        for name, spec in inputs.items():
            if not _value_name_ok(name):
                raise GraphError("input names must be non-empty strings")
            if not isinstance(spec, TensorSpec):
                raise GraphError(f"input {name!r} spec must be a TensorSpec")
        self._inputs = dict(inputs)
        self._constants: dict[str, torch.Tensor] = {}
        self._nodes: list[Node] = []
        self._env: dict[str, TensorSpec] = dict(inputs)

    def _new_name(self, name: str) -> None:
        if not _value_name_ok(name):
            raise GraphError("names must be non-empty strings")
        if name in self._env:
            raise GraphError(f"duplicate name {name!r}")

    def spec(self, name: str) -> TensorSpec:
        return self._env[name]

    def constant(self, name: str, value: torch.Tensor) -> str:
        self._new_name(name)
        if not isinstance(value, torch.Tensor):
            raise GraphError(f"constant {name!r} must be a torch.Tensor")
        self._constants[name] = value.detach().clone()
        self._env[name] = spec_of(value)
        return name

    def add(self, name: str, op: str, inputs: tuple[str, ...], **attrs) -> str:
        self._new_name(name)
        undefined = next((i for i in inputs if i not in self._env), None)
        if undefined is not None:
            raise GraphError(f"node {name!r} input {undefined!r} is not defined")
        try:
            spec = infer_spec(op, [self._env[i] for i in inputs], attrs)
        except GraphError as e:
            raise GraphError(f"node {name!r}: {e}") from e
        self._nodes.append(Node(name, op, tuple(inputs), dict(attrs), spec))
        self._env[name] = spec
        return name

    def finish(self, outputs: tuple[str, ...], output_is_tuple: bool = False) -> Graph:
        g = Graph(dict(self._inputs), dict(self._constants), list(self._nodes), tuple(outputs),
                  output_is_tuple or len(outputs) > 1)
        g.validate()
        return g
