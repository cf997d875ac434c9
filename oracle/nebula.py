"""Nebula decoder oracle (CPU): restates the TinyDecoder forward of
src/nebula/model.py:37-100 and greedy generation
(src/nebula/benchmarks.py:25-31, tests/test_nebula_runtime.py:25-34) over an
explicit weight dict, plus an incremental decode step over a KV cache with
the absolute-position mask of src/nebula/runtime.py:125-189.

Weights: dict with keys tok, pos, lnf_w, lnf_b, head and per layer l:
  l.ln1_w l.ln1_b l.ln2_w l.ln2_b l.q l.k l.v l.o l.up l.down   (nn.Linear layout [out, in])
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def weights_from_state_dict(sd: dict, num_layers: int) -> dict:
    w = {
        "tok": sd["token_embedding.weight"],
        "pos": sd["position_embedding.weight"],
        "lnf_w": sd["final_norm.weight"],
        "lnf_b": sd["final_norm.bias"],
        "head": sd["lm_head.weight"],
    }
    for i in range(num_layers):
        p = f"blocks.{i}."
        for k_src, k_dst in (("ln1.weight", "ln1_w"), ("ln1.bias", "ln1_b"), ("ln2.weight", "ln2_w"),
                             ("ln2.bias", "ln2_b"), ("q.weight", "q"), ("k.weight", "k"), ("v.weight", "v"),
                             ("o.weight", "o"), ("up.weight", "up"), ("down.weight", "down")):
            w[f"{i}.{k_dst}"] = sd[p + k_src]
    return w


def _block(w, i, x, num_heads, kv=None, start_pos=0):
    b, t, h = x.shape
    hd = h // num_heads
    res = x
    h1 = F.layer_norm(x, (h,), w[f"{i}.ln1_w"], w[f"{i}.ln1_b"], 1e-5)
    q = F.linear(h1, w[f"{i}.q"]).view(b, t, num_heads, hd).transpose(1, 2)
    k = F.linear(h1, w[f"{i}.k"]).view(b, t, num_heads, hd).transpose(1, 2)
    v = F.linear(h1, w[f"{i}.v"]).view(b, t, num_heads, hd).transpose(1, 2)
    if kv is not None:
        kc, vc = kv
        kc[:, :, start_pos:start_pos + t] = k
        vc[:, :, start_pos:start_pos + t] = v
        k = kc[:, :, : start_pos + t]
        v = vc[:, :, : start_pos + t]
    end = k.shape[2]
    scores = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(hd)
    key_pos = torch.arange(end)
    query_pos = start_pos + torch.arange(t)
    scores = scores.masked_fill(key_pos[None, :] > query_pos[:, None], float("-inf"))
    attn = torch.softmax(scores.float(), dim=-1).to(x.dtype)
    out = torch.matmul(attn, v).transpose(1, 2).reshape(b, t, h)
    x = res + F.linear(out, w[f"{i}.o"])
    res = x
    h2 = F.layer_norm(x, (h,), w[f"{i}.ln2_w"], w[f"{i}.ln2_b"], 1e-5)
    return res + F.linear(F.gelu(F.linear(h2, w[f"{i}.up"]), approximate="tanh"), w[f"{i}.down"])


@torch.inference_mode()
def forward(w: dict, tokens: torch.Tensor, num_heads: int, num_layers: int,
            caches=None, start_pos: int = 0) -> torch.Tensor:
    """Logits [B, T, V].  With ``caches`` (list of (k, v) [B,H,S,hd] per layer)
    the call is an incremental step at absolute position ``start_pos``."""
    _, t = tokens.shape
    pos = torch.arange(start_pos, start_pos + t)
    x = F.embedding(tokens, w["tok"]) + F.embedding(pos, w["pos"])
    for i in range(num_layers):
        x = _block(w, i, x, num_heads, None if caches is None else caches[i], start_pos)
    h = x.shape[-1]
    return F.linear(F.layer_norm(x, (h,), w["lnf_w"], w["lnf_b"], 1e-5), w["head"])


@torch.inference_mode()
def greedy(w: dict, prompt: list[int], n: int, num_heads: int, num_layers: int) -> list[int]:
    cur = list(prompt)
    out = []
    for _ in range(n):
        logits = forward(w, torch.tensor([cur], dtype=torch.long), num_heads, num_layers)
        nxt = int(logits[0, -1].argmax())
        out.append(nxt)
        cur.append(nxt)
    return out
