"""Torch evaluation of graph ops.

Used for meta-tensor spec inference and by the explicit ``backend="torch"``
executor, exactly as the reference uses src/forgeml/ops.py:25-83.  The
``"triton"``/``"auto"`` backends route GEMM, LayerNorm and SDPA nodes to the
sm_100a kernels instead (forgeml_b200.forgeml.kernels).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

SUPPORTED_OPS = frozenset(
    {
        "matmul",
        "linear",
        "add",
        "mul",
        "relu",
        "gelu",
        "reshape",
        "transpose",
        "softmax",
        "narrow",
        "fused_linear_gelu",
        "layer_norm",
        "sdpa",
        "conv2d",
        "embedding",
    }
)


def _mm_bias(args):
    return torch.addmm(args[2], args[0], args[1]) if len(args) == 3 else torch.mm(args[0], args[1])


def evaluate(op: str, args: tuple[torch.Tensor, ...], attrs: dict) -> torch.Tensor:
    if op == "matmul":
        return torch.matmul(args[0], args[1])
    if op == "linear":
        return _mm_bias(args)
    if op == "fused_linear_gelu":
        return F.gelu(_mm_bias(args), approximate=attrs.get("approximate", "none"))
    if op == "add":
        return torch.add(args[0], args[1])
    if op == "mul":
        return torch.mul(args[0], args[1])
    if op == "relu":
        return F.relu(args[0])
    if op == "gelu":
        return F.gelu(args[0], approximate=attrs.get("approximate", "none"))
    if op == "reshape":
        return torch.reshape(args[0], tuple(attrs["shape"]))
    if op == "transpose":
        return torch.transpose(args[0], attrs["dim0"], attrs["dim1"])
    if op == "softmax":
        return torch.softmax(args[0], dim=attrs["dim"])
    if op == "narrow":
        x = args[0]
        return torch.narrow(x, attrs["dim"] % x.dim(), attrs["start"], attrs["length"])
    if op == "layer_norm":
        norm = attrs["normalized_shape"]
        norm = (norm,) if isinstance(norm, int) else tuple(norm)
        w, b = (args[1], args[2]) if len(args) == 3 else (None, None)
        return F.layer_norm(args[0], norm, w, b, attrs["eps"])
    if op == "sdpa":
        return F.scaled_dot_product_attention(
            args[0],
            args[1],
            args[2],
            attn_mask=args[3] if len(args) == 4 else None,
            dropout_p=0.0,
            is_causal=attrs["is_causal"],
            scale=attrs.get("scale"),
        )
    if op == "conv2d":
        return F.conv2d(
            args[0],
            args[1],
            args[2] if len(args) == 3 else None,
            stride=attrs["stride"],
            padding=attrs["padding"],
            dilation=attrs["dilation"],
            groups=attrs["groups"],
        )
    if op == "embedding":
        return F.embedding(args[0], args[1])
    raise ValueError(f"unsupported op {op!r}")
