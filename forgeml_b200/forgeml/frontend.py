"""torch.fx frontend: ``from_torch(model, example_inputs) -> Graph``.

Lowers the module types, functions and tensor methods the compiled-forward
workloads use (the configs' MLP and pre-LN encoder block, the reference's test
models) into the IR.  Value names are part of the drop-in contract -- graphs
and memory plans are compared with the reference's dictionary for
dictionary -- so they follow the reference frontend's scheme
(src/forgeml/frontend.py): placeholders ``input_<i>``, fx node names for
nodes, and generated constants / helper nodes ``<node>_<role>_<n>`` from one
counter shared by the whole trace (roles weight_t, flatten, bias, linear,
weight; ``scalar_<n>`` for Python scalars).  A Linear stores its weight
transposed and contiguous, [K, N]; a Linear on a rank != 2 input is wrapped in
reshape views to and from [rows, K].  Shape arithmetic (``x.shape``,
``size()``, integer operators) is evaluated at trace time.

Each supported module, function and method has one handler, registered in the
tables below; anything else raises UnsupportedOperator.
"""

from __future__ import annotations

import math
import operator
from typing import Any, Callable

import torch
import torch.fx
import torch.nn.functional as F
from torch import nn

from forgeml_b200.forgeml.ir import Graph, GraphBuilder, GraphError, TensorSpec


class UnsupportedOperator(GraphError):
    pass


class _Known:
    """A trace-time constant (a shape, an int, a dtype ...)."""

    def __init__(self, value: Any):
        self.value = value


def _int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _static_shape(raw, src: tuple[int, ...], where: str) -> tuple[int, ...]:
    if not isinstance(raw, (tuple, list)):
        raise UnsupportedOperator(f"{where} requires a static shape tuple/list")
    dims = list(raw)
    if not all(_int(d) for d in dims):
        raise UnsupportedOperator(f"{where} shape dims must be ints, got {dims!r}")
    if dims.count(-1) > 1:
        raise UnsupportedOperator(f"{where} allows at most one -1 dim, got {dims!r}")
    if any(d == 0 or d < -1 for d in dims):
        raise UnsupportedOperator(f"{where} dims must be positive or -1, got {dims!r}")
    if -1 in dims:
        rest = math.prod(d for d in dims if d != -1)
        if rest == 0 or math.prod(src) % rest:
            raise GraphError(f"{where} cannot infer -1 dim for input {src}")
        dims[dims.index(-1)] = math.prod(src) // rest
    return tuple(dims)


def _flattened(shape: tuple[int, ...], start, end, where: str) -> tuple[int, ...]:
    rank = len(shape)
    if rank == 0:
        raise UnsupportedOperator(f"{where} requires a tensor of rank >= 1")
    for label, v in (("start_dim", start), ("end_dim", end)):
        if not _int(v) or not -rank <= v < rank:
            raise UnsupportedOperator(f"{where} {label}={v!r} out of range for rank {rank}")
    s, e = start % rank, end % rank
    if s > e:
        raise UnsupportedOperator(f"{where} has start_dim > end_dim")
    return shape[:s] + (math.prod(shape[s:e + 1]),) + shape[e + 1:]


_MODULES: list[tuple[type, Callable]] = []
_FUNCTIONS: dict[Any, Callable] = {}
_METHODS: dict[str, Callable] = {}


def _on_module(*types):
    def reg(fn):
        _MODULES.extend((t, fn) for t in types)
        return fn

    return reg


def _on_function(*targets):
    def reg(fn):
        _FUNCTIONS.update(dict.fromkeys(targets, fn))
        return fn

    return reg


def _on_method(*names):
    def reg(fn):
        _METHODS.update(dict.fromkeys(names, fn))
        return fn

    return reg


class _Tracer:
    def __init__(self, model: nn.Module, example_inputs: tuple[torch.Tensor, ...]):
        self.model = model
        self.examples = example_inputs
        self.g: GraphBuilder | None = None
        self.values: dict[str, str] = {}  # fx node -> graph value
        self.known: dict[str, Any] = {}   # fx node -> trace-time constant
        self.consts: dict[str, torch.Tensor] = {}
        self.count = 0

    # ------------------------------------------------------------ naming
    def fresh(self, stem: str) -> str:
        self.count += 1
        return f"{stem}_{self.count}"

    def const(self, name: str, t: torch.Tensor) -> str:
        t = t.detach().clone().contiguous()
        self.g.constant(name, t)
        self.consts[name] = t
        return name

    def spec(self, value: str) -> TensorSpec:
        return self.g.spec(value)

    # ------------------------------------------------------------ arguments
    def args(self, node, *names: str, **defaults) -> dict:
        """fx call arguments bound to ``names`` (positional then keyword)."""
        if len(node.args) > len(names):
            raise UnsupportedOperator(f"too many arguments at {node.name!r}")
        got = dict(zip(names, node.args))
        for k, v in node.kwargs.items():
            if k not in names or k in got:
                raise UnsupportedOperator(f"unsupported or repeated argument {k!r} at {node.name!r}")
            got[k] = v
        for k, v in defaults.items():
            got.setdefault(k, v)
        if set(names) - set(got):
            raise UnsupportedOperator(f"missing argument at {node.name!r}")
        return got

    def try_known(self, v) -> tuple[bool, Any]:
        if isinstance(v, torch.fx.Node):
            return (True, self.known[v.name]) if v.name in self.known else (False, None)
        if isinstance(v, torch.Size):
            return True, tuple(int(d) for d in v)
        if isinstance(v, (tuple, list)):
            items = [self.try_known(x) for x in v]
            return (True, tuple(x for _, x in items)) if all(ok for ok, _ in items) else (False, None)
        return True, v

    def known_value(self, v):
        ok, val = self.try_known(v)
        if ok:
            return val
        if isinstance(v, torch.fx.Node):
            raise UnsupportedOperator(f"fx value {v.name!r} must resolve statically at compile time")
        raise UnsupportedOperator(f"unsupported static value {v!r}")

    def tensor(self, a) -> str:
        """The graph value of an fx argument (Python scalars become constants)."""
        if isinstance(a, torch.fx.Node):
            if a.name in self.values:
                return self.values[a.name]
            if a.name not in self.known:
                raise GraphError(f"fx node {a.name!r} has no produced value")
            a = self.known[a.name]
        if isinstance(a, (int, float, bool)):
            return self.const(self.fresh("scalar"), torch.tensor(a))
        raise UnsupportedOperator(f"unsupported argument {a!r} of type {type(a).__name__}")

    # ------------------------------------------------------------ linear
    def linear(self, name: str, x: str, weight: torch.Tensor, bias: torch.Tensor | None) -> str:
        if weight.dim() != 2:
            raise UnsupportedOperator(f"linear weight at {name!r} must be rank-2, got rank {weight.dim()}")
        if bias is not None and bias.dim() != 1:
            raise UnsupportedOperator(f"linear bias at {name!r} must be rank-1, got rank {bias.dim()}")
        w = self.const(self.fresh(f"{name}_weight_t"), weight.t())
        shape = self.spec(x).shape
        rows_in = x
        wrapped = len(shape) != 2
        if wrapped:
            if not shape:
                raise UnsupportedOperator(f"linear input at {name!r} must have rank >= 1")
            rows_in = self.g.add(self.fresh(f"{name}_flatten"), "reshape", (x,),
                                 shape=(math.prod(shape[:-1]), shape[-1]))
        ins = (rows_in, w)
        if bias is not None:
            ins += (self.const(self.fresh(f"{name}_bias"), bias),)
        y = self.g.add(self.fresh(f"{name}_linear") if wrapped else name, "linear", ins)
        if not wrapped:
            return y
        return self.g.add(name, "reshape", (y,), shape=shape[:-1] + (weight.shape[0],))

    # ------------------------------------------------------------ driver
    def run(self) -> Graph:
        try:
            traced = torch.fx.symbolic_trace(self.model)
        except Exception as e:  # noqa: BLE001 - tracing errors become frontend errors
            raise UnsupportedOperator(f"symbolic trace failed: {e}") from e
        places = [n for n in traced.graph.nodes if n.op == "placeholder"]
        if len(places) != len(self.examples):
            raise GraphError(f"model expects {len(places)} inputs, got {len(self.examples)} example inputs")
        self.g = GraphBuilder({f"input_{i}": TensorSpec(tuple(t.shape), t.dtype, str(t.device))
                               for i, t in enumerate(self.examples)})
        for i, p in enumerate(places):
            self.values[p.name] = f"input_{i}"
        for node in traced.graph.nodes:
            if node.op == "placeholder":
                continue
            if node.op == "output":
                return self.finish(node.args[0])
            out = self.visit(traced, node)
            if isinstance(out, _Known):
                self.known[node.name] = out.value
            else:
                self.values[node.name] = out
        raise GraphError("traced graph has no output node")

    def visit(self, traced, node):
        if node.op == "get_attr":
            obj: Any = traced
            for part in node.target.split("."):
                if not isinstance(obj, (nn.Module, torch.Tensor)) or not hasattr(obj, part):
                    raise GraphError(f"cannot resolve attribute {node.target!r}")
                obj = getattr(obj, part)
            if not isinstance(obj, torch.Tensor):
                raise GraphError(f"attribute {node.target!r} is not a tensor")
            return self.const(node.name, obj)
        if node.op == "call_module":
            mod = traced.get_submodule(node.target)
            handler = next((fn for t, fn in _MODULES if isinstance(mod, t)), None)
            if handler is None:
                raise UnsupportedOperator(f"unsupported module {type(mod).__name__} at {node.name!r}")
            x = self.tensor(self.args(node, "input")["input"])
            return handler(self, node.name, x, mod)
        if node.op == "call_function":
            handler = _FUNCTIONS.get(node.target)
            if handler is None:
                raise UnsupportedOperator(f"unsupported function {getattr(node.target, '__name__', node.target)!r} "
                                          f"at {node.name!r}")
            return handler(self, node.name, node)
        if node.op == "call_method":
            handler = _METHODS.get(node.target)
            if handler is None:
                raise UnsupportedOperator(f"unsupported method {node.target!r} at {node.name!r}")
            return handler(self, node.name, node)
        raise UnsupportedOperator(f"unsupported fx node op {node.op!r} at {node.name!r}")

    def finish(self, res) -> Graph:
        if isinstance(res, torch.fx.Node):
            if res.name not in self.values:
                raise UnsupportedOperator("model outputs must be produced tensors; static values are not supported")
            return self.g.finish((self.values[res.name],), output_is_tuple=False)
        if isinstance(res, tuple):
            if not all(isinstance(r, torch.fx.Node) and r.name in self.values for r in res):
                raise UnsupportedOperator("only flat tuples of produced tensors are supported as outputs")
            return self.g.finish(tuple(self.values[r.name] for r in res), output_is_tuple=True)
        raise UnsupportedOperator(
            f"unsupported output type {type(res).__name__}; only a tensor or flat tuple of tensors is supported")


# ================================================================ modules
@_on_module(nn.Identity)
def _identity(tr, name, x, mod):
    return x


@_on_module(nn.Linear)
def _linear_module(tr, name, x, mod):
    return tr.linear(name, x, mod.weight.detach().clone(), None if mod.bias is None else mod.bias.detach().clone())


@_on_module(nn.LayerNorm)
def _layer_norm_module(tr, name, x, mod):
    norm = tuple(mod.normalized_shape)
    if not mod.elementwise_affine:
        return tr.g.add(name, "layer_norm", (x,), normalized_shape=norm, eps=float(mod.eps))
    if mod.weight is None or mod.bias is None:
        raise UnsupportedOperator(f"partially affine LayerNorm at {name!r}")
    w = tr.const(tr.fresh(f"{name}_weight"), mod.weight)
    b = tr.const(tr.fresh(f"{name}_bias"), mod.bias)
    return tr.g.add(name, "layer_norm", (x, w, b), normalized_shape=norm, eps=float(mod.eps))


@_on_module(nn.GELU)
def _gelu_module(tr, name, x, mod):
    return tr.g.add(name, "gelu", (x,), approximate=mod.approximate)


@_on_module(nn.ReLU)
def _relu_module(tr, name, x, mod):
    if mod.inplace:
        raise UnsupportedOperator(f"in-place ReLU at {name!r} is not supported")
    return tr.g.add(name, "relu", (x,))


@_on_module(nn.Softmax)
def _softmax_module(tr, name, x, mod):
    if mod.dim is None:
        raise UnsupportedOperator(f"Softmax at {name!r} has no static dim")
    return tr.g.add(name, "softmax", (x,), dim=mod.dim)


@_on_module(nn.Flatten)
def _flatten_module(tr, name, x, mod):
    return tr.g.add(name, "reshape", (x,),
                    shape=_flattened(tr.spec(x).shape, mod.start_dim, mod.end_dim, f"Flatten at {name!r}"))


@_on_module(nn.Embedding)
def _embedding_module(tr, name, x, mod):
    if (mod.padding_idx is not None or mod.max_norm is not None or mod.norm_type != 2.0 or mod.scale_grad_by_freq
            or mod.sparse):
        raise UnsupportedOperator(f"Embedding options at {name!r} are not supported in inference lowering")
    return tr.g.add(name, "embedding", (x, tr.const(tr.fresh(f"{name}_weight"), mod.weight)))


@_on_module(nn.Conv2d)
def _conv2d_module(tr, name, x, mod):
    if mod.padding_mode != "zeros":
        raise UnsupportedOperator(f"Conv2d padding_mode={mod.padding_mode!r} at {name!r} is not supported")
    ins = (x, tr.const(tr.fresh(f"{name}_weight"), mod.weight))
    if mod.bias is not None:
        ins += (tr.const(tr.fresh(f"{name}_bias"), mod.bias),)
    return tr.g.add(name, "conv2d", ins, stride=mod.stride, padding=mod.padding, dilation=mod.dilation,
                    groups=mod.groups)


# ================================================================ functions
@_on_function(getattr)
def _getattr(tr, name, node):
    a = tr.args(node, "input", "name")
    src = a["input"]
    if not isinstance(src, torch.fx.Node) or src.name not in tr.values:
        raise UnsupportedOperator(f"getattr source at {name!r} must be a tensor value")
    spec = tr.spec(tr.values[src.name])
    table = {"shape": spec.shape, "ndim": len(spec.shape), "device": torch.device(spec.device), "dtype": spec.dtype}
    if a["name"] not in table:
        raise UnsupportedOperator(f"getattr {a['name']!r} at {name!r} is not supported")
    return _Known(table[a["name"]])


@_on_function(operator.getitem)
def _getitem(tr, name, node):
    a = tr.args(node, "input", "index")
    try:
        return _Known(tr.known_value(a["input"])[tr.known_value(a["index"])])
    except (IndexError, KeyError, TypeError) as e:
        raise UnsupportedOperator(f"invalid static index at {name!r}") from e


def _known_operands(tr, node):
    pairs = [tr.try_known(v) for v in node.args]
    return [v for _, v in pairs] if pairs and all(ok for ok, _ in pairs) else None


def _arith(op):
    def handler(tr, name, node):
        vals = _known_operands(tr, node)
        if vals is not None and len(vals) == 2:
            return _Known(op(*vals))
        if op is operator.add:
            return _add(tr, name, node)
        if op is operator.mul:
            return _mul(tr, name, node)
        raise UnsupportedOperator(f"unsupported function {op.__name__!r} at {name!r}")

    return handler


for _op in (operator.sub, operator.floordiv, operator.truediv, operator.mod):
    _FUNCTIONS[_op] = _arith(_op)


@_on_function(operator.neg, operator.pos)
def _unary_known(tr, name, node):
    vals = _known_operands(tr, node)
    if vals is None:
        raise UnsupportedOperator(f"unsupported function {node.target.__name__!r} at {name!r}")
    return _Known(node.target(vals[0]))


def _second_operand(name, a) -> Any:
    if (a["other"] is None) == (a["mat2"] is None):
        raise UnsupportedOperator(f"matmul at {name!r} needs exactly one second operand")
    return a["other"] if a["other"] is not None else a["mat2"]


@_on_function(torch.matmul, torch.mm, operator.matmul)
def _matmul(tr, name, node):
    a = tr.args(node, "input", "other", "mat2", other=None, mat2=None)
    return tr.g.add(name, "matmul", (tr.tensor(a["input"]), tr.tensor(_second_operand(name, a))))


@_on_function(torch.add)
def _add(tr, name, node):
    vals = _known_operands(tr, node) if node.target is operator.add else None
    if vals is not None and len(vals) == 2:
        return _Known(vals[0] + vals[1])
    a = tr.args(node, "input", "other", "alpha", "out", alpha=1, out=None)
    if a["out"] is not None or a["alpha"] != 1:
        raise UnsupportedOperator(f"add out=/alpha at {name!r} is not supported")
    return tr.g.add(name, "add", (tr.tensor(a["input"]), tr.tensor(a["other"])))


@_on_function(torch.mul)
def _mul(tr, name, node):
    vals = _known_operands(tr, node) if node.target is operator.mul else None
    if vals is not None and len(vals) == 2:
        return _Known(vals[0] * vals[1])
    a = tr.args(node, "input", "other", "out", out=None)
    if a["out"] is not None:
        raise UnsupportedOperator(f"mul out= at {name!r} is not supported")
    return tr.g.add(name, "mul", (tr.tensor(a["input"]), tr.tensor(a["other"])))


_FUNCTIONS[operator.add] = _add
_FUNCTIONS[operator.mul] = _mul


@_on_function(F.relu, torch.relu)
def _relu(tr, name, node):
    if node.target is F.relu:
        a = tr.args(node, "input", "inplace", inplace=False)
        if a["inplace"] is not False:
            raise UnsupportedOperator(f"in-place relu at {name!r} is not supported")
    else:
        a = tr.args(node, "input")
    return tr.g.add(name, "relu", (tr.tensor(a["input"]),))


@_on_function(F.gelu)
def _gelu(tr, name, node):
    a = tr.args(node, "input", "approximate", approximate="none")
    if a["approximate"] not in ("none", "tanh"):
        raise UnsupportedOperator(f"gelu approximate {a['approximate']!r} at {name!r}")
    return tr.g.add(name, "gelu", (tr.tensor(a["input"]),), approximate=a["approximate"])


@_on_function(F.linear)
def _linear_fn(tr, name, node):
    a = tr.args(node, "input", "weight", "bias", bias=None)
    x, w = tr.tensor(a["input"]), tr.tensor(a["weight"])
    if w not in tr.consts:
        raise UnsupportedOperator(f"linear weight at {name!r} must be constant")
    bias = None
    if a["bias"] is not None:
        b = tr.tensor(a["bias"])
        if b not in tr.consts:
            raise UnsupportedOperator(f"linear bias at {name!r} must be constant")
        bias = tr.consts[b]
    return tr.linear(name, x, tr.consts[w], bias)


@_on_function(torch.reshape, torch.Tensor.reshape, torch.Tensor.view)
def _reshape_fn(tr, name, node):
    a = tr.args(node, "input", "shape")
    x = tr.tensor(a["input"])
    return tr.g.add(name, "reshape", (x,), shape=_static_shape(tr.known_value(a["shape"]), tr.spec(x).shape, "reshape"))


@_on_function(torch.transpose)
def _transpose_fn(tr, name, node):
    a = tr.args(node, "input", "dim0", "dim1")
    return tr.g.add(name, "transpose", (tr.tensor(a["input"]),), dim0=tr.known_value(a["dim0"]),
                    dim1=tr.known_value(a["dim1"]))


def _softmax_node(tr, name, x_arg, dim_arg, dtype):
    if dtype is not None:
        raise UnsupportedOperator(f"softmax dtype= at {name!r} is not supported")
    dim = tr.known_value(dim_arg)
    if not _int(dim):
        raise UnsupportedOperator(f"softmax at {name!r} needs a static int dim")
    return tr.g.add(name, "softmax", (tr.tensor(x_arg),), dim=dim)


@_on_function(F.softmax, torch.softmax)
def _softmax_fn(tr, name, node):
    a = tr.args(node, "input", "dim", "_stacklevel", "dtype", dim=None, _stacklevel=3, dtype=None)
    return _softmax_node(tr, name, a["input"], a["dim"], a["dtype"])


@_on_function(F.layer_norm)
def _layer_norm_fn(tr, name, node):
    a = tr.args(node, "input", "normalized_shape", "weight", "bias", "eps", weight=None, bias=None, eps=1e-5)
    x = tr.tensor(a["input"])
    norm = tr.known_value(a["normalized_shape"])
    norm = (norm,) if _int(norm) else norm
    if (a["weight"] is None) != (a["bias"] is None):
        raise UnsupportedOperator(f"layer_norm at {name!r} needs weight and bias together")
    ins = (x,) if a["weight"] is None else (x, tr.tensor(a["weight"]), tr.tensor(a["bias"]))
    return tr.g.add(name, "layer_norm", ins, normalized_shape=tuple(norm), eps=float(tr.known_value(a["eps"])))


@_on_function(F.scaled_dot_product_attention)
def _sdpa_fn(tr, name, node):
    a = tr.args(node, "query", "key", "value", "attn_mask", "dropout_p", "is_causal", "scale", "enable_gqa",
                attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False)
    if tr.known_value(a["dropout_p"]) != 0:
        raise UnsupportedOperator(f"sdpa dropout_p at {name!r} must be zero")
    if tr.known_value(a["enable_gqa"]) is not False:
        raise UnsupportedOperator(f"sdpa enable_gqa at {name!r} is not supported")
    causal = tr.known_value(a["is_causal"])
    if not isinstance(causal, bool):
        raise UnsupportedOperator(f"sdpa is_causal at {name!r} must be a bool")
    ins = tuple(tr.tensor(a[k]) for k in ("query", "key", "value"))
    if a["attn_mask"] is not None:
        ins += (tr.tensor(a["attn_mask"]),)
    return tr.g.add(name, "sdpa", ins, is_causal=causal, scale=tr.known_value(a["scale"]))


@_on_function(F.embedding, torch.embedding)
def _embedding_fn(tr, name, node):
    a = tr.args(node, "input", "weight")
    return tr.g.add(name, "embedding", (tr.tensor(a["input"]), tr.tensor(a["weight"])))


def _flatten_call(tr, name, node):
    a = tr.args(node, "input", "start_dim", "end_dim", start_dim=0, end_dim=-1)
    x = tr.tensor(a["input"])
    return tr.g.add(name, "reshape", (x,), shape=_flattened(tr.spec(x).shape, tr.known_value(a["start_dim"]),
                                                             tr.known_value(a["end_dim"]), f"flatten at {name!r}"))


_FUNCTIONS[torch.flatten] = _flatten_call


# ================================================================ methods
@_on_method("size", "dim", "ndim")
def _size_method(tr, name, node):
    a = tr.args(node, "input", "dim", dim=None)
    shape = tr.spec(tr.tensor(a["input"])).shape
    if a["dim"] is None:
        return _Known(shape if node.target == "size" else len(shape))
    i = tr.known_value(a["dim"])
    if not _int(i) or not -len(shape) <= i < len(shape):
        raise UnsupportedOperator(f"{node.target} index at {name!r} out of range")
    return _Known(shape[i])


@_on_method("matmul", "mm")
def _matmul_method(tr, name, node):
    a = tr.args(node, "input", "other", "mat2", other=None, mat2=None)
    other = a["other"] if a["other"] is not None else a["mat2"]
    if other is None:
        raise UnsupportedOperator(f"{node.target} at {name!r} needs a second operand")
    return tr.g.add(name, "matmul", (tr.tensor(a["input"]), tr.tensor(other)))


@_on_method("view", "reshape")
def _reshape_method(tr, name, node):
    if node.kwargs or len(node.args) < 2:
        raise UnsupportedOperator(f"{node.target} at {name!r} needs a positional shape")
    x = tr.tensor(node.args[0])
    dims = tuple(tr.known_value(v) for v in node.args[1:])
    if len(dims) == 1 and isinstance(dims[0], (tuple, list)):
        dims = tuple(dims[0])
    return tr.g.add(name, "reshape", (x,), shape=_static_shape(dims, tr.spec(x).shape, node.target))


_METHODS["flatten"] = _flatten_call


@_on_method("transpose")
def _transpose_method(tr, name, node):
    return _transpose_fn(tr, name, node)


@_on_method("t")
def _t_method(tr, name, node):
    x = tr.tensor(tr.args(node, "input")["input"])
    if len(tr.spec(x).shape) != 2:
        raise UnsupportedOperator(f"t() at {name!r} requires a rank-2 tensor")
    return tr.g.add(name, "transpose", (x,), dim0=0, dim1=1)


@_on_method("softmax")
def _softmax_method(tr, name, node):
    a = tr.args(node, "input", "dim", "dtype", dtype=None)
    return _softmax_node(tr, name, a["input"], a["dim"], a["dtype"])


# ================================================================ entry point
def from_torch(model: nn.Module, example_inputs: tuple[torch.Tensor, ...]) -> Graph:
    if not isinstance(model, nn.Module):
        raise GraphError("from_torch expects an nn.Module")
    bad = next((i for i, t in enumerate(example_inputs) if not isinstance(t, torch.Tensor)), None)
    if bad is not None:
        raise GraphError(f"example input {bad} is not a tensor")
    for m in model.modules():
        if m.training and isinstance(m, (nn.modules.dropout._DropoutNd, nn.modules.batchnorm._BatchNorm)):
            raise GraphError(f"module {type(m).__name__} is in training mode; call model.eval() before compiling")
    with torch.no_grad():
        return _Tracer(model, tuple(example_inputs)).run()
