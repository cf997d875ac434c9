"""LayerNorm oracle: F.layer_norm semantics of src/forgeml/ops.py:54-60 and
src/nebula/runtime.py:130,151,185, evaluated in float64 and rounded once."""

from __future__ import annotations

import torch


def layer_norm(x, normalized_shape, weight=None, bias=None, eps=1e-5):
    norm = (normalized_shape,) if isinstance(normalized_shape, int) else tuple(normalized_shape)
    xd = x.detach().cpu().double()
    dims = tuple(range(-len(norm), 0))
    mean = xd.mean(dim=dims, keepdim=True)
    var = ((xd - mean) ** 2).mean(dim=dims, keepdim=True)
    y = (xd - mean) / torch.sqrt(var + eps)
    if weight is not None:
        y = y * weight.detach().cpu().double() + bias.detach().cpu().double()
    return y.to(x.dtype)
