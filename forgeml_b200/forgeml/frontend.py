"""torch.fx frontend: nn.Module -> Graph.

Lowers the module types and functions the compiled-forward workloads use into
the IR with the reference frontend's value naming (src/forgeml/frontend.py:
``input_<i>`` placeholders, fx node names for nodes, ``<node>_weight_t_<n>``,
``<node>_flatten_<n>``, ``<node>_bias_<n>``, ``<node>_linear_<n>``,
``<node>_weight_<n>``, ``scalar_<n>`` with one shared counter), because node
and constant names appear in graph and memory-plan dictionaries that compare
one to one with the reference.  Linear weights are stored transposed and
contiguous as [K, N] (src/forgeml/frontend.py:198-200); rank != 2 linear
inputs are wrapped in reshape views (:204-233).  Shape arithmetic
(``x.shape``, ``size()``, integer ops) is resolved statically.
"""

from __future__ import annotations

import math
import operator
from typing import Any

import torch
import torch.fx
import torch.nn.functional as F
from torch import nn

from forgeml_b200.forgeml.ir import Graph, GraphBuilder, GraphError, TensorSpec


class UnsupportedOperator(GraphError):
    pass


class _Static:
    """A value known at compile time (shapes, ints, dtypes)."""

    def __init__(self, value: Any):
        self.value = value


def _spec(t: torch.Tensor) -> TensorSpec:
    return TensorSpec(tuple(t.shape), t.dtype, str(t.device))


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _resolve_shape(raw, in_shape: tuple[int, ...], where: str) -> tuple[int, ...]:
    if not isinstance(raw, (tuple, list)):
        raise UnsupportedOperator(f"{where} requires a static shape tuple/list")
    dims = list(raw)
    if not all(_is_int(d) for d in dims):
        raise UnsupportedOperator(f"{where} shape dims must be ints, got {dims!r}")
    if sum(d == -1 for d in dims) > 1:
        raise UnsupportedOperator(f"{where} allows at most one -1 dim, got {dims!r}")
    if any(d == 0 or d < -1 for d in dims):
        raise UnsupportedOperator(f"{where} dims must be positive or -1, got {dims!r}")
    if -1 in dims:
        known = math.prod(d for d in dims if d != -1)
        total = math.prod(in_shape)
        if known == 0 or total % known:
            raise GraphError(f"{where} cannot infer -1 dim for input {in_shape}")
        dims[dims.index(-1)] = total // known
    return tuple(dims)


def _flatten(shape: tuple[int, ...], start, end, where: str) -> tuple[int, ...]:
    rank = len(shape)
    if rank == 0:
        raise UnsupportedOperator(f"{where} requires a tensor of rank >= 1")
    idx = []
    for name, v in (("start_dim", start), ("end_dim", end)):
        if not _is_int(v) or not -rank <= v < rank:
            raise UnsupportedOperator(f"{where} {name}={v!r} out of range for rank {rank}")
        idx.append(v % rank)
    s, e = idx
    if s > e:
        raise UnsupportedOperator(f"{where} has start_dim > end_dim")
    return shape[:s] + (math.prod(shape[s:e + 1]),) + shape[e + 1:]


_STATIC_BINARY = {operator.add, operator.sub, operator.mul, operator.floordiv, operator.truediv, operator.mod}


class _Lowering:
    def __init__(self, model: nn.Module, example_inputs: tuple[torch.Tensor, ...]):
        self.model = model
        self.example_inputs = example_inputs
        self.b: GraphBuilder | None = None
        self.env: dict[str, str] = {}          # fx node name -> graph value name
        self.consts: dict[str, torch.Tensor] = {}
        self.statics: dict[str, Any] = {}
        self.counter = 0

    # ----------------------------------------------------------- helpers
    def fresh(self, hint: str) -> str:
        self.counter += 1
        return f"{hint}_{self.counter}"

    def spec(self, value: str) -> TensorSpec:
        return self.b.spec(value)

    def add_const(self, name: str, t: torch.Tensor) -> str:
        t = t.detach().clone().contiguous()
        self.b.constant(name, t)
        self.consts[name] = t
        return name

    def literal(self, v):
        ok, val = self.maybe_literal(v)
        if not ok:
            if isinstance(v, torch.fx.Node):
                raise UnsupportedOperator(f"fx value {v.name!r} must resolve statically at compile time")
            raise UnsupportedOperator(f"unsupported static value {v!r}")
        return val

    def maybe_literal(self, v):
        if isinstance(v, torch.fx.Node):
            return (True, self.statics[v.name]) if v.name in self.statics else (False, None)
        if isinstance(v, torch.Size):
            return True, tuple(int(d) for d in v)
        if isinstance(v, (tuple, list)):
            out = []
            for item in v:
                ok, val = self.maybe_literal(item)
                if not ok:
                    return False, None
                out.append(val)
            return True, tuple(out)
        return True, v

    def value(self, a) -> str:
        if isinstance(a, torch.fx.Node):
            if a.name in self.env:
                return self.env[a.name]
            if a.name not in self.statics:
                raise GraphError(f"fx node {a.name!r} has no produced value")
            a = self.statics[a.name]
        if isinstance(a, (int, float, bool)):
            t = torch.tensor(a)
            name = self.fresh("scalar")
            self.b.constant(name, t)
            self.consts[name] = t
            return name
        raise UnsupportedOperator(f"unsupported argument {a!r} of type {type(a).__name__}")

    @staticmethod
    def bind(node, names: tuple[str, ...], defaults: dict | None = None) -> dict:
        if len(node.args) > len(names):
            raise UnsupportedOperator(f"too many arguments at {node.name!r}")
        bound = dict(zip(names, node.args))
        for k, v in node.kwargs.items():
            if k not in names or k in bound:
                raise UnsupportedOperator(f"unsupported or repeated argument {k!r} at {node.name!r}")
            bound[k] = v
        for k, v in (defaults or {}).items():
            bound.setdefault(k, v)
        if set(names) - set(bound):
            raise UnsupportedOperator(f"missing argument at {node.name!r}")
        return bound

    # ----------------------------------------------------------- linear
    def linear(self, out_name: str, x: str, weight: torch.Tensor, bias: torch.Tensor | None) -> str:
        if weight.dim() != 2:
            raise UnsupportedOperator(f"linear weight at {out_name!r} must be rank-2, got rank {weight.dim()}")
        if bias is not None and bias.dim() != 1:
            raise UnsupportedOperator(f"linear bias at {out_name!r} must be rank-1, got rank {bias.dim()}")
        w_name = self.fresh(f"{out_name}_weight_t")
        w_t = weight.t().contiguous()
        self.b.constant(w_name, w_t)
        self.consts[w_name] = w_t
        xs = self.spec(x)
        flat = len(xs.shape) != 2
        src = x
        if flat:
            if not xs.shape:
                raise UnsupportedOperator(f"linear input at {out_name!r} must have rank >= 1")
            src = self.b.add(self.fresh(f"{out_name}_flatten"), "reshape", (x,),
                             shape=(math.prod(xs.shape[:-1]), xs.shape[-1]))
        inputs = (src, w_name)
        if bias is not None:
            b_name = self.fresh(f"{out_name}_bias")
            bc = bias.contiguous()
            self.b.constant(b_name, bc)
            self.consts[b_name] = bc
            inputs += (b_name,)
        result = self.b.add(self.fresh(f"{out_name}_linear") if flat else out_name, "linear", inputs)
        if not flat:
            return result
        return self.b.add(out_name, "reshape", (result,), shape=xs.shape[:-1] + (w_t.shape[1],))

    # ----------------------------------------------------------- driver
    def lower(self) -> Graph:
        inputs = {f"input_{i}": _spec(t) for i, t in enumerate(self.example_inputs)}
        try:
            traced = torch.fx.symbolic_trace(self.model)
        except Exception as e:  # noqa: BLE001 - tracing errors become frontend errors
            raise UnsupportedOperator(f"symbolic trace failed: {e}") from e
        self.b = GraphBuilder(inputs)
        placeholders = [n for n in traced.graph.nodes if n.op == "placeholder"]
        if len(placeholders) != len(self.example_inputs):
            raise GraphError(f"model expects {len(placeholders)} inputs, got {len(self.example_inputs)} example inputs")
        for i, ph in enumerate(placeholders):
            self.env[ph.name] = f"input_{i}"
        for node in traced.graph.nodes:
            if node.op == "placeholder":
                continue
            if node.op == "output":
                return self.finish(node)
            out = self.lower_node(traced, node)
            if isinstance(out, _Static):
                self.statics[node.name] = out.value
            else:
                self.env[node.name] = out
        raise GraphError("traced graph has no output node")

    def lower_node(self, traced, node):
        if node.op == "get_attr":
            obj: Any = traced
            for part in node.target.split("."):
                if not isinstance(obj, (nn.Module, torch.Tensor)) or not hasattr(obj, part):
                    raise GraphError(f"cannot resolve attribute {node.target!r}")
                obj = getattr(obj, part)
            if not isinstance(obj, torch.Tensor):
                raise GraphError(f"attribute {node.target!r} is not a tensor")
            return self.add_const(node.name, obj)
        if node.op == "call_module":
            mod = traced
            for part in node.target.split("."):
                mod = getattr(mod, part)
            return self.lower_module(node.name, mod, node)
        if node.op == "call_function":
            return self.lower_function(node.name, node)
        if node.op == "call_method":
            return self.lower_method(node.name, node)
        raise UnsupportedOperator(f"unsupported fx node op {node.op!r} at {node.name!r}")

    def finish(self, out_node) -> Graph:
        res = out_node.args[0]
        if isinstance(res, torch.fx.Node):
            if res.name not in self.env:
                raise UnsupportedOperator("model outputs must be produced tensors; static values are not supported")
            return self.b.finish((self.env[res.name],), output_is_tuple=False)
        if isinstance(res, tuple):
            names = []
            for r in res:
                if not isinstance(r, torch.fx.Node) or r.name not in self.env:
                    raise UnsupportedOperator("only flat tuples of produced tensors are supported as outputs")
                names.append(self.env[r.name])
            return self.b.finish(tuple(names), output_is_tuple=True)
        raise UnsupportedOperator(
            f"unsupported output type {type(res).__name__}; only a tensor or flat tuple of tensors is supported"
        )

    # ----------------------------------------------------------- modules
    def lower_module(self, name: str, mod: nn.Module, node):
        x = self.value(self.bind(node, ("input",))["input"])
        if isinstance(mod, nn.Identity):
            return x
        if isinstance(mod, nn.Linear):
            return self.linear(name, x, mod.weight.detach().clone(),
                               None if mod.bias is None else mod.bias.detach().clone())
        if isinstance(mod, nn.LayerNorm):
            norm = tuple(mod.normalized_shape)
            if mod.elementwise_affine:
                if mod.weight is None or mod.bias is None:
                    raise UnsupportedOperator(f"partially affine LayerNorm at {name!r}")
                w = self.add_const(self.fresh(f"{name}_weight"), mod.weight)
                bb = self.add_const(self.fresh(f"{name}_bias"), mod.bias)
                return self.b.add(name, "layer_norm", (x, w, bb), normalized_shape=norm, eps=float(mod.eps))
            return self.b.add(name, "layer_norm", (x,), normalized_shape=norm, eps=float(mod.eps))
        if isinstance(mod, nn.GELU):
            return self.b.add(name, "gelu", (x,), approximate=mod.approximate)
        if isinstance(mod, nn.ReLU):
            if mod.inplace:
                raise UnsupportedOperator(f"in-place ReLU at {name!r} is not supported")
            return self.b.add(name, "relu", (x,))
        if isinstance(mod, nn.Softmax):
            if mod.dim is None:
                raise UnsupportedOperator(f"Softmax at {name!r} has no static dim")
            return self.b.add(name, "softmax", (x,), dim=mod.dim)
        if isinstance(mod, nn.Flatten):
            return self.b.add(name, "reshape", (x,),
                              shape=_flatten(self.spec(x).shape, mod.start_dim, mod.end_dim, f"Flatten at {name!r}"))
        if isinstance(mod, nn.Embedding):
            if (mod.padding_idx is not None or mod.max_norm is not None or mod.norm_type != 2.0
                    or mod.scale_grad_by_freq or mod.sparse):
                raise UnsupportedOperator(f"Embedding options at {name!r} are not supported in inference lowering")
            w = self.add_const(self.fresh(f"{name}_weight"), mod.weight)
            return self.b.add(name, "embedding", (x, w))
        if isinstance(mod, nn.Conv2d):
            if mod.padding_mode != "zeros":
                raise UnsupportedOperator(f"Conv2d padding_mode={mod.padding_mode!r} at {name!r} is not supported")
            w = self.add_const(self.fresh(f"{name}_weight"), mod.weight)
            ins = (x, w)
            if mod.bias is not None:
                ins += (self.add_const(self.fresh(f"{name}_bias"), mod.bias),)
            return self.b.add(name, "conv2d", ins, stride=mod.stride, padding=mod.padding,
                              dilation=mod.dilation, groups=mod.groups)
        raise UnsupportedOperator(f"unsupported module {type(mod).__name__} at {name!r}")

    # ----------------------------------------------------------- functions
    def lower_function(self, name: str, node):
        t = node.target
        if t is getattr:
            bound = self.bind(node, ("input", "name"))
            src = bound["input"]
            if not hasattr(src, "name") or src.name not in self.env:
                raise UnsupportedOperator(f"getattr source at {name!r} must be a tensor value")
            spec = self.spec(self.env[src.name])
            attr = bound["name"]
            table = {"shape": spec.shape, "ndim": len(spec.shape), "device": torch.device(spec.device),
                     "dtype": spec.dtype}
            if attr not in table:
                raise UnsupportedOperator(f"getattr {attr!r} at {name!r} is not supported")
            return _Static(table[attr])
        if t is operator.getitem:
            bound = self.bind(node, ("input", "index"))
            val, idx = self.literal(bound["input"]), self.literal(bound["index"])
            try:
                return _Static(val[idx])
            except (IndexError, KeyError, TypeError) as e:
                raise UnsupportedOperator(f"invalid static index at {name!r}") from e
        if t in _STATIC_BINARY:
            ok_a, a = self.maybe_literal(node.args[0])
            ok_b, b = self.maybe_literal(node.args[1])
            if ok_a and ok_b:
                return _Static(t(a, b))
        if t in (operator.neg, operator.pos):
            ok, v = self.maybe_literal(node.args[0])
            if ok:
                return _Static(t(v))
        if t in (torch.matmul, torch.mm, operator.matmul):
            bound = self.bind(node, ("input", "other", "mat2"), {"other": None, "mat2": None})
            other = bound["other"] if bound["other"] is not None else bound["mat2"]
            if other is None or (bound["other"] is not None and bound["mat2"] is not None):
                raise UnsupportedOperator(f"matmul at {name!r} needs exactly one second operand")
            return self.b.add(name, "matmul", (self.value(bound["input"]), self.value(other)))
        if t in (operator.add, torch.add):
            bound = self.bind(node, ("input", "other", "alpha", "out"), {"alpha": 1, "out": None})
            if bound["out"] is not None or bound["alpha"] != 1:
                raise UnsupportedOperator(f"add out=/alpha at {name!r} is not supported")
            return self.b.add(name, "add", (self.value(bound["input"]), self.value(bound["other"])))
        if t in (operator.mul, torch.mul):
            bound = self.bind(node, ("input", "other", "out"), {"out": None})
            if bound["out"] is not None:
                raise UnsupportedOperator(f"mul out= at {name!r} is not supported")
            return self.b.add(name, "mul", (self.value(bound["input"]), self.value(bound["other"])))
        if t is F.relu or t is torch.relu:
            if t is F.relu:
                bound = self.bind(node, ("input", "inplace"), {"inplace": False})
                if bound["inplace"] is not False:
                    raise UnsupportedOperator(f"in-place relu at {name!r} is not supported")
            else:
                bound = self.bind(node, ("input",))
            return self.b.add(name, "relu", (self.value(bound["input"]),))
        if t is F.gelu:
            bound = self.bind(node, ("input", "approximate"), {"approximate": "none"})
            if bound["approximate"] not in ("none", "tanh"):
                raise UnsupportedOperator(f"gelu approximate {bound['approximate']!r} at {name!r}")
            return self.b.add(name, "gelu", (self.value(bound["input"]),), approximate=bound["approximate"])
        if t is F.linear:
            bound = self.bind(node, ("input", "weight", "bias"), {"bias": None})
            x = self.value(bound["input"])
            w = self.value(bound["weight"])
            if w not in self.consts:
                raise UnsupportedOperator(f"linear weight at {name!r} must be constant")
            bias = None
            if bound["bias"] is not None:
                bn = self.value(bound["bias"])
                if bn not in self.consts:
                    raise UnsupportedOperator(f"linear bias at {name!r} must be constant")
                bias = self.consts[bn]
            return self.linear(name, x, self.consts[w], bias)
        if t in (torch.reshape, torch.Tensor.reshape, torch.Tensor.view):
            bound = self.bind(node, ("input", "shape"))
            x = self.value(bound["input"])
            return self.b.add(name, "reshape", (x,),
                              shape=_resolve_shape(self.literal(bound["shape"]), self.spec(x).shape, "reshape"))
        if t is torch.transpose:
            bound = self.bind(node, ("input", "dim0", "dim1"))
            return self.b.add(name, "transpose", (self.value(bound["input"]),),
                              dim0=self.literal(bound["dim0"]), dim1=self.literal(bound["dim1"]))
        if t in (F.softmax, torch.softmax):
            bound = self.bind(node, ("input", "dim", "_stacklevel", "dtype"),
                              {"dim": None, "_stacklevel": 3, "dtype": None})
            if bound["dtype"] is not None:
                raise UnsupportedOperator(f"softmax dtype= at {name!r} is not supported")
            dim = self.literal(bound["dim"])
            if not _is_int(dim):
                raise UnsupportedOperator(f"softmax at {name!r} needs a static int dim")
            return self.b.add(name, "softmax", (self.value(bound["input"]),), dim=dim)
        if t is F.layer_norm:
            bound = self.bind(node, ("input", "normalized_shape", "weight", "bias", "eps"),
                              {"weight": None, "bias": None, "eps": 1e-5})
            x = self.value(bound["input"])
            norm = self.literal(bound["normalized_shape"])
            norm = (norm,) if _is_int(norm) else norm
            if (bound["weight"] is None) != (bound["bias"] is None):
                raise UnsupportedOperator(f"layer_norm at {name!r} needs weight and bias together")
            ins = (x,)
            if bound["weight"] is not None:
                ins += (self.value(bound["weight"]), self.value(bound["bias"]))
            return self.b.add(name, "layer_norm", ins, normalized_shape=tuple(norm),
                              eps=float(self.literal(bound["eps"])))
        if t is F.scaled_dot_product_attention:
            bound = self.bind(node, ("query", "key", "value", "attn_mask", "dropout_p", "is_causal", "scale",
                                     "enable_gqa"),
                              {"attn_mask": None, "dropout_p": 0.0, "is_causal": False, "scale": None,
                               "enable_gqa": False})
            if self.literal(bound["dropout_p"]) != 0:
                raise UnsupportedOperator(f"sdpa dropout_p at {name!r} must be zero")
            if self.literal(bound["enable_gqa"]) is not False:
                raise UnsupportedOperator(f"sdpa enable_gqa at {name!r} is not supported")
            causal = self.literal(bound["is_causal"])
            if not isinstance(causal, bool):
                raise UnsupportedOperator(f"sdpa is_causal at {name!r} must be a bool")
            ins = (self.value(bound["query"]), self.value(bound["key"]), self.value(bound["value"]))
            if bound["attn_mask"] is not None:
                ins += (self.value(bound["attn_mask"]),)
            return self.b.add(name, "sdpa", ins, is_causal=causal, scale=self.literal(bound["scale"]))
        if t in (F.embedding, torch.embedding):
            bound = self.bind(node, ("input", "weight"))
            return self.b.add(name, "embedding", (self.value(bound["input"]), self.value(bound["weight"])))
        if t is torch.flatten:
            bound = self.bind(node, ("input", "start_dim", "end_dim"), {"start_dim": 0, "end_dim": -1})
            x = self.value(bound["input"])
            return self.b.add(name, "reshape", (x,), shape=_flatten(
                self.spec(x).shape, self.literal(bound["start_dim"]), self.literal(bound["end_dim"]),
                f"flatten at {name!r}"))
        raise UnsupportedOperator(f"unsupported function {getattr(t, '__name__', t)!r} at {name!r}")

    # ----------------------------------------------------------- methods
    def lower_method(self, name: str, node):
        m = node.target
        if m in ("size", "dim", "ndim"):
            bound = self.bind(node, ("input", "dim"), {"dim": None})
            shape = self.spec(self.value(bound["input"])).shape
            if m in ("dim", "ndim") and bound["dim"] is None:
                return _Static(len(shape))
            if bound["dim"] is None:
                return _Static(shape)
            i = self.literal(bound["dim"])
            if not _is_int(i) or not -len(shape) <= i < len(shape):
                raise UnsupportedOperator(f"{m} index at {name!r} out of range")
            return _Static(shape[i])
        if m in ("matmul", "mm"):
            bound = self.bind(node, ("input", "other", "mat2"), {"other": None, "mat2": None})
            other = bound["other"] if bound["other"] is not None else bound["mat2"]
            if other is None:
                raise UnsupportedOperator(f"{m} at {name!r} needs a second operand")
            return self.b.add(name, "matmul", (self.value(bound["input"]), self.value(other)))
        if m in ("view", "reshape"):
            if node.kwargs or len(node.args) < 2:
                raise UnsupportedOperator(f"{m} at {name!r} needs a positional shape")
            x = self.value(node.args[0])
            raw = tuple(self.literal(v) for v in node.args[1:])
            dims = raw[0] if len(raw) == 1 and isinstance(raw[0], (tuple, list)) else raw
            return self.b.add(name, "reshape", (x,), shape=_resolve_shape(tuple(dims), self.spec(x).shape, m))
        if m == "flatten":
            bound = self.bind(node, ("input", "start_dim", "end_dim"), {"start_dim": 0, "end_dim": -1})
            x = self.value(bound["input"])
            return self.b.add(name, "reshape", (x,), shape=_flatten(
                self.spec(x).shape, self.literal(bound["start_dim"]), self.literal(bound["end_dim"]),
                f"flatten at {name!r}"))
        if m == "transpose":
            bound = self.bind(node, ("input", "dim0", "dim1"))
            return self.b.add(name, "transpose", (self.value(bound["input"]),),
                              dim0=self.literal(bound["dim0"]), dim1=self.literal(bound["dim1"]))
        if m == "t":
            x = self.value(self.bind(node, ("input",))["input"])
            if len(self.spec(x).shape) != 2:
                raise UnsupportedOperator(f"t() at {name!r} requires a rank-2 tensor")
            return self.b.add(name, "transpose", (x,), dim0=0, dim1=1)
        if m == "softmax":
            bound = self.bind(node, ("input", "dim", "dtype"), {"dtype": None})
            if bound["dtype"] is not None:
                raise UnsupportedOperator(f"softmax dtype= at {name!r} is not supported")
            dim = self.literal(bound["dim"])
            if not _is_int(dim):
                raise UnsupportedOperator(f"softmax at {name!r} needs a static int dim")
            return self.b.add(name, "softmax", (self.value(bound["input"]),), dim=dim)
        raise UnsupportedOperator(f"unsupported method {m!r} at {name!r}")


def _check_modules(model: nn.Module) -> None:
    for m in model.modules():
        if m.training and isinstance(m, (nn.modules.dropout._DropoutNd, nn.modules.batchnorm._BatchNorm)):
            raise GraphError(f"module {type(m).__name__} is in training mode; call model.eval() before compiling")


def from_torch(model: nn.Module, example_inputs: tuple[torch.Tensor, ...]) -> Graph:
    if not isinstance(model, nn.Module):
        raise GraphError("from_torch expects an nn.Module")
    for i, t in enumerate(example_inputs):
        if not isinstance(t, torch.Tensor):
            raise GraphError(f"example input {i} is not a tensor")
    _check_modules(model)
    with torch.no_grad():
        return _Lowering(model, tuple(example_inputs)).lower()
