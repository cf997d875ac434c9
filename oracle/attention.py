"""Attention oracles.

sdpa():  softmax(q k^T * scale + mask) v -- the contract of
         F.scaled_dot_product_attention as called by src/forgeml/ops.py:61-70
         (dropout 0, top-left causal, bool or additive mask), in float64.
nebula_attention(): src/nebula/runtime.py:139-144 -- scores q k^T / sqrt(hd)
         over the whole cached prefix, keys at absolute positions
         > start_pos + t masked with -inf, softmax in fp32 or better, then PV.
"""

from __future__ import annotations

import math

import torch


def sdpa(q, k, v, attn_mask=None, is_causal=False, scale=None):
    qd, kd, vd = (t.detach().cpu().double() for t in (q, k, v))
    d = q.shape[-1]
    sc = scale if scale is not None else 1.0 / math.sqrt(d)
    s = (qd @ kd.transpose(-1, -2)) * sc
    sq, sk = q.shape[-2], k.shape[-2]
    if is_causal:
        keep = torch.ones(sq, sk, dtype=torch.bool).tril()
        s = s.masked_fill(~keep, float("-inf"))
    if attn_mask is not None:
        m = attn_mask.detach().cpu()
        if m.dtype == torch.bool:
            s = s.masked_fill(~m, float("-inf"))
        else:
            s = s + m.double()
    p = torch.softmax(s, dim=-1)
    return (p @ vd).to(q.dtype)


def nebula_attention(q, k_all, v_all, start_pos: int):
    """q [B,h,T,hd]; k_all/v_all [B,h,end,hd] with end = start_pos + T."""
    qd, kd, vd = (t.detach().cpu().double() for t in (q, k_all, v_all))
    t = q.shape[2]
    end = k_all.shape[2]
    scores = (qd @ kd.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    key_pos = torch.arange(end)
    query_pos = start_pos + torch.arange(t)
    scores = scores.masked_fill(key_pos[None, :] > query_pos[:, None], float("-inf"))
    p = torch.softmax(scores, dim=-1)
    return (p @ vd).to(q.dtype)
