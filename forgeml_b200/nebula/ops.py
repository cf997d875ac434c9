"""Thin launch wrappers for the Nebula decode-step kernels (C ABI neb_*).

All take device tensors, launch on the current stream of their device and
raise on a nonzero status; none allocates except where an output is created.
"""

from __future__ import annotations

import math

import torch

from forgeml_b200 import _native


def _stream(t: torch.Tensor) -> int:
    return _native.stream_ptr(t.device)


def kv_append(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
              slot_of: torch.Tensor, start_pos: torch.Tensor) -> None:
    """pool[slot_of[b], h, start_pos[b]+t, :] = kv[b, t, h, :] (k, v: [B,T,H,D] views)."""
    b, t, h, d = k.shape
    max_seq = k_pool.shape[2]
    _native.call(
        "neb_kv_append", k.data_ptr(), _native.strides4(k), v.data_ptr(), _native.strides4(v),
        k_pool.data_ptr(), v_pool.data_ptr(), slot_of.data_ptr(), start_pos.data_ptr(),
        b, t, h, d, max_seq, _native.dtype_code(k.dtype), _stream(k),
    )


def attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, slot_of: torch.Tensor,
              start_pos: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Masked attention of q [B,T,H,D] over the cached prefix; returns [B,T,H*D]."""
    b, t, h, d = q.shape
    if out is None:
        out = torch.empty((b, t, h * d), dtype=q.dtype, device=q.device)
    _native.call(
        "neb_attention", q.data_ptr(), _native.strides4(q), k_pool.data_ptr(), v_pool.data_ptr(),
        slot_of.data_ptr(), start_pos.data_ptr(), out.data_ptr(), b, t, h, d, k_pool.shape[2], k_pool.shape[0],
        1.0 / math.sqrt(d), _native.dtype_code(q.dtype), _stream(q),
    )
    return out


def embed(tokens: torch.Tensor, start_pos: torch.Tensor, tok_emb: torch.Tensor, pos_emb: torch.Tensor,
          out: torch.Tensor | None = None) -> torch.Tensor:
    b, t = tokens.shape
    hidden = tok_emb.shape[1]
    if out is None:
        out = torch.empty((b, t, hidden), dtype=tok_emb.dtype, device=tok_emb.device)
    _native.call(
        "neb_embed", tokens.data_ptr(), start_pos.data_ptr(), tok_emb.data_ptr(), pos_emb.data_ptr(),
        out.data_ptr(), b, t, hidden, tok_emb.shape[0], pos_emb.shape[0],
        _native.dtype_code(tok_emb.dtype), _stream(tok_emb),
    )
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-wise argmax of a [rows, cols] view (unit column stride)."""
    rows, cols = logits.shape
    if logits.stride(1) != 1:
        raise ValueError("argmax needs unit column stride")
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    _native.call(
        "neb_argmax", logits.data_ptr(), logits.stride(0), rows, cols, out.data_ptr(),
        _native.dtype_code(logits.dtype), _stream(logits),
    )
    return out


def add(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(a)
    _native.call("neb_add", a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(),
                 _native.dtype_code(a.dtype), _stream(a))
    return out
