"""Decoder configuration and the monolithic reference-layout decoder.

``DecoderConfig`` and ``TinyDecoder`` keep the reference's fields, validation
and module construction order (src/nebula/model.py:11-100) because the
default-initialised weights must come out bit-identical under the same seed:
``ShardedDecoder(init="reference")`` slices them exactly as the reference
engine does.  TinyDecoder.forward is the plain-torch monolithic forward of the
reference model (pre-LN, causal mask, fp32 softmax, tanh GELU).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass(frozen=True)
class DecoderConfig:
    vocab_size: int = 256
    hidden_size: int = 128
    num_heads: int = 8
    num_layers: int = 4
    intermediate_size: int = 256
    max_seq_len: int = 128
    seed: int = 17

    def __post_init__(self):
        for name in ("vocab_size", "hidden_size", "num_heads", "num_layers", "intermediate_size", "max_seq_len"):
            v = getattr(self, name)
            if not isinstance(v, int) or isinstance(v, bool) or v <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if self.hidden_size % self.num_heads:
            raise ValueError("hidden_size must be divisible by num_heads")

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads


class DecoderBlock(nn.Module):
    def __init__(self, config: DecoderConfig):
        super().__init__()
        h = config.hidden_size
        self.num_heads = config.num_heads
        self.head_dim = h // config.num_heads
        # Construction order fixes the RNG stream: ln1, ln2, q, k, v, o, up, down.
        self.ln1 = nn.LayerNorm(h, eps=1e-5)
        self.ln2 = nn.LayerNorm(h, eps=1e-5)
        self.q = nn.Linear(h, h, bias=False)
        self.k = nn.Linear(h, h, bias=False)
        self.v = nn.Linear(h, h, bias=False)
        self.o = nn.Linear(h, h, bias=False)
        self.up = nn.Linear(h, config.intermediate_size, bias=False)
        self.down = nn.Linear(config.intermediate_size, h, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, t, h = x.shape
        n, hd = self.num_heads, self.head_dim
        h1 = self.ln1(x)
        q = self.q(h1).view(b, t, n, hd).transpose(1, 2)
        k = self.k(h1).view(b, t, n, hd).transpose(1, 2)
        v = self.v(h1).view(b, t, n, hd).transpose(1, 2)
        scores = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(hd)
        scores = scores + torch.full((t, t), float("-inf"), device=x.device).triu(1)
        attn = torch.softmax(scores.float(), dim=-1).to(x.dtype)
        x = x + self.o(torch.matmul(attn, v).transpose(1, 2).reshape(b, t, h))
        return x + self.down(F.gelu(self.up(self.ln2(x)), approximate="tanh"))


class TinyDecoder(nn.Module):
    def __init__(self, config: DecoderConfig):
        super().__init__()
        self.config = config
        with torch.random.fork_rng():
            torch.manual_seed(config.seed)
            self.token_embedding = nn.Embedding(config.vocab_size, config.hidden_size)
            self.position_embedding = nn.Embedding(config.max_seq_len, config.hidden_size)
            self.blocks = nn.ModuleList(DecoderBlock(config) for _ in range(config.num_layers))
            self.final_norm = nn.LayerNorm(config.hidden_size, eps=1e-5)
            self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        if not isinstance(tokens, torch.Tensor) or tokens.dtype != torch.long:
            raise ValueError("tokens must be a long tensor")
        if tokens.dim() != 2 or tokens.shape[0] == 0 or tokens.shape[1] == 0:
            raise ValueError("tokens must have shape [B, T] with B, T >= 1")
        if tokens.shape[1] > self.config.max_seq_len:
            raise ValueError("sequence length exceeds max_seq_len")
        if (tokens < 0).any() or (tokens >= self.config.vocab_size).any():
            raise ValueError("token ids out of range")
        t = tokens.shape[1]
        x = self.token_embedding(tokens) + self.position_embedding(torch.arange(t, device=tokens.device))
        for block in self.blocks:
            x = block(x)
        return self.lm_head(self.final_norm(x))


def _normal_index(key: str) -> int:
    """Generator stream of weight ``key`` in the synthetic initialisation."""
    fixed = {"tok": 0, "pos": 1, "head": 2}
    if key in fixed:
        return fixed[key]
    layer, name = key.split(".")
    return 16 + 8 * int(layer) + ("q", "k", "v", "o", "up", "down").index(name)


def normal_weight_shape(config: DecoderConfig, key: str) -> tuple[int, int]:
    h, f, v = config.hidden_size, config.intermediate_size, config.vocab_size
    if key in ("tok", "head"):
        return (v, h)
    if key == "pos":
        return (config.max_seq_len, h)
    name = key.split(".")[1]
    return {"up": (f, h), "down": (h, f)}.get(name, (h, h))


def normal_weight(config: DecoderConfig, key: str, device, std: float = 0.02) -> torch.Tensor:
    """Full fp32 weight ``key`` of the synthetic benchmark initialisation:
    every matrix ~ N(0, std), drawn on ``device`` from its own generator seeded
    with ``seed * 1_000_003 + stream`` (keys: tok, pos, head, and per layer l
    "l.q", "l.k", "l.v", "l.o", "l.up", "l.down" in nn.Linear [out, in]
    layout).  Every TP rank draws the full tensor and keeps its shard, so the
    shards of one model agree, and a checker can rebuild the whole model."""
    g = torch.Generator(device=device)
    g.manual_seed(config.seed * 1_000_003 + _normal_index(key))
    return torch.empty(normal_weight_shape(config, key), device=device, dtype=torch.float32).normal_(0.0, std, generator=g)

