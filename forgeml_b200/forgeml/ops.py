"""Torch semantics of the graph ops.

The compiled model's torch-planned nodes, the frontend's spec inference and
the autotuner's expected values all evaluate an op through ``evaluate``.  The
meaning of each op is the reference's (src/forgeml/ops.py:25-83: "linear" is
addmm with a [K, N] weight, "fused_linear_gelu" that plus GELU, "narrow"
takes a possibly negative dim, ...); the native backend computes the GEMM,
LayerNorm and SDPA ops on the sm_100a kernels instead.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.nn.functional as F


def _gemm(args) -> torch.Tensor:
    a, b = args[0], args[1]
    return torch.addmm(args[2], a, b) if len(args) == 3 else torch.mm(a, b)


def _layer_norm(args, attrs) -> torch.Tensor:
    shape = attrs["normalized_shape"]
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    weight, bias = (args[1], args[2]) if len(args) == 3 else (None, None)
    return F.layer_norm(args[0], shape, weight, bias, attrs["eps"])


def _sdpa(args, attrs) -> torch.Tensor:
    return F.scaled_dot_product_attention(args[0], args[1], args[2], attn_mask=args[3] if len(args) == 4 else None,
                                          dropout_p=0.0, is_causal=attrs["is_causal"], scale=attrs.get("scale"))


def _conv2d(args, attrs) -> torch.Tensor:
    return F.conv2d(args[0], args[1], args[2] if len(args) == 3 else None, stride=attrs["stride"],
                    padding=attrs["padding"], dilation=attrs["dilation"], groups=attrs["groups"])


_EVAL: dict[str, Callable] = {
    "matmul": lambda a, _: torch.matmul(a[0], a[1]),
    "linear": lambda a, _: _gemm(a),
    "fused_linear_gelu": lambda a, at: F.gelu(_gemm(a), approximate=at.get("approximate", "none")),
    "add": lambda a, _: torch.add(a[0], a[1]),
    "mul": lambda a, _: torch.mul(a[0], a[1]),
    "relu": lambda a, _: F.relu(a[0]),
    "gelu": lambda a, at: F.gelu(a[0], approximate=at.get("approximate", "none")),
    "reshape": lambda a, at: torch.reshape(a[0], tuple(at["shape"])),
    "transpose": lambda a, at: torch.transpose(a[0], at["dim0"], at["dim1"]),
    "softmax": lambda a, at: torch.softmax(a[0], dim=at["dim"]),
    "narrow": lambda a, at: torch.narrow(a[0], at["dim"] % a[0].dim(), at["start"], at["length"]),
    "layer_norm": lambda a, at: _layer_norm(a, at),
    "sdpa": lambda a, at: _sdpa(a, at),
    "conv2d": lambda a, at: _conv2d(a, at),
    "embedding": lambda a, _: F.embedding(a[0], a[1]),
}

SUPPORTED_OPS = frozenset(_EVAL)


def evaluate(op: str, args: tuple[torch.Tensor, ...], attrs: dict) -> torch.Tensor:
    fn = _EVAL.get(op)
    if fn is None:
        raise ValueError(f"unsupported op {op!r}")
    return fn(args, attrs)
