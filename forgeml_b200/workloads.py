"""Synthetic workloads of the headline configurations (seeded, no datasets).

c1  ForgeML-compiled 2-layer MLP: [64,512] -> Linear(512,2048) -> exact GELU
    -> Linear(2048,512); default nn.Linear init under seed 0, x ~ N(0,1).
c2  ForgeML-compiled pre-LN encoder block: [8,512,768], 12 heads, FFN 3072,
    non-causal SDPA, exact GELU; Linear weights and biases ~ N(0, 0.02)
    (the bias distribution is not fixed by the config; N(0,0.02) is the
    choice recorded here), LN gamma=1, beta=0, eps 1e-5, seed 1, x ~ N(0,1).
c3  GEMM sweep: A, B ~ U(-1,1), bias ~ N(0,1), seed 2.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn


def make_c1_mlp(seed: int = 0) -> tuple[nn.Module, torch.Tensor]:
    torch.manual_seed(seed)
    m = nn.Sequential(nn.Linear(512, 2048), nn.GELU(), nn.Linear(2048, 512)).eval()
    x = torch.randn(64, 512)
    return m, x


class EncoderBlock(nn.Module):
    """Pre-LN transformer encoder block with separate q/k/v projections."""

    def __init__(self, d_model: int = 768, heads: int = 12, ff: int = 3072):
        super().__init__()
        self.heads = heads
        self.head_dim = d_model // heads
        self.ln1 = nn.LayerNorm(d_model, eps=1e-5)
        self.q = nn.Linear(d_model, d_model)
        self.k = nn.Linear(d_model, d_model)
        self.v = nn.Linear(d_model, d_model)
        self.o = nn.Linear(d_model, d_model)
        self.ln2 = nn.LayerNorm(d_model, eps=1e-5)
        self.fc1 = nn.Linear(d_model, ff)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(ff, d_model)

    def forward(self, x):
        # Token-flattened [b*s, d] projections so the compiler sees rank-2
        # linears (QKV fused into one wide GEMM, FFN-up fused with GELU).
        b, s, d = x.shape
        h = self.ln1(x).reshape(b * s, d)
        q = self.q(h).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        k = self.k(h).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        v = self.v(h).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        a = F.scaled_dot_product_attention(q, k, v)
        a = a.transpose(1, 2).reshape(b * s, d)
        x = x + self.o(a).view(b, s, d)
        h = self.ln2(x).reshape(b * s, d)
        return x + self.fc2(self.act(self.fc1(h))).view(b, s, d)


def make_c2_block(batch: int = 8, seq: int = 512, d_model: int = 768, heads: int = 12, ff: int = 3072,
                  seed: int = 1, dtype: torch.dtype = torch.float32) -> tuple[nn.Module, torch.Tensor]:
    torch.manual_seed(seed)
    m = EncoderBlock(d_model, heads, ff)
    with torch.no_grad():
        for lin in (m.q, m.k, m.v, m.o, m.fc1, m.fc2):
            lin.weight.normal_(0.0, 0.02)
            lin.bias.normal_(0.0, 0.02)
    x = torch.randn(batch, seq, d_model)
    return m.eval().to(dtype), x.to(dtype)


def make_c3_operands(m: int, n: int, k: int, dtype: torch.dtype, *, transposed_b: bool = False,
                     strided_a: bool = False, seed: int = 2, device: str = "cpu"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    if strided_a:
        base = torch.rand(2 * m, k, generator=g) * 2 - 1
        a = base.to(device=device, dtype=dtype)[::2]
    else:
        a = (torch.rand(m, k, generator=g) * 2 - 1).to(device=device, dtype=dtype)
    if transposed_b:
        b = (torch.rand(n, k, generator=g) * 2 - 1).to(device=device, dtype=dtype).t()
    else:
        b = (torch.rand(k, n, generator=g) * 2 - 1).to(device=device, dtype=dtype)
    bias = torch.randn(n, generator=g).to(device=device, dtype=dtype)
    return a, b, bias
