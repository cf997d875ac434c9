"""GEMM + fused epilogue oracle.

Restates the reference Triton template's arithmetic contract
(src/forgeml/_triton.py:43-57):
    value = round_out(acc)                       (:43)
    value = round_out(value + bias)              (:46, when a bias is given)
    value = gelu_erf(value) | gelu_tanh(value)   (:47-57, computed in fp32)
    store round_out(value)                       (:58-62)
The accumulator is formed in float64 so the oracle is at least as exact as
the fp32 tensor-core accumulation it checks.
"""

from __future__ import annotations

import torch


def gelu_f32(x: torch.Tensor, approximate: str) -> torch.Tensor:
    x = x.to(torch.float32)
    if approximate == "tanh":
        return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))
    return 0.5 * x * (1.0 + torch.erf(x * 0.7071067811865476))


def matmul_epilogue(
    a: torch.Tensor,
    b: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    activation: str = "none",
    approximate: str = "none",
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    dtype = a.dtype
    acc = a.detach().cpu().double() @ b.detach().cpu().double()
    value = acc.to(torch.float32).to(dtype).to(torch.float32)
    if bias is not None:
        value = (value + bias.detach().cpu().to(torch.float32)).to(dtype).to(torch.float32)
    if activation == "gelu":
        value = gelu_f32(value, approximate)
    if residual is not None:
        value = value.to(dtype).to(torch.float32) + residual.detach().cpu().to(torch.float32)
    return value.to(dtype)
