"""Constant-weight linear layer on the tcgen05 GEMM with a pre-packed weight.

``PackedLinear(W)`` packs an nn.Linear-layout weight W [N, K] once
(``fml_pack_weight``: 16 KB swizzled tiles, 128 rows x 128 bytes of K) and
then computes ``y = x W^T`` with the fused epilogue of ``fml_gemm`` (bias,
GELU, residual) through ``fml_linear_packed``: the weight streams from HBM as
sequential bulk copies instead of strided row fragments.  16-bit weights
only; fp32 layers use the 3xTF32 ``fml_gemm`` path.
"""

from __future__ import annotations

import ctypes

import torch

from forgeml_b200 import _native


class PackedLinear:
    def __init__(self, weight: torch.Tensor):
        if weight.dim() != 2 or not weight.is_cuda or weight.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("PackedLinear needs a 2-D 16-bit CUDA weight [N, K]")
        if weight.stride(1) != 1:
            raise ValueError("PackedLinear needs K-contiguous rows")
        self.n, self.k = weight.shape
        self.dtype = weight.dtype
        self.code = _native.dtype_code(weight.dtype)
        lib = _native.load()
        nbytes = int(lib.fml_packed_weight_bytes(self.n, self.k, self.code))
        self._buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=weight.device)
        self.ptr = (self._buf.data_ptr() + 1023) // 1024 * 1024
        _native.call("fml_pack_weight", weight.data_ptr(), weight.stride(0), self.n, self.k, self.code, self.ptr,
                     _native.stream_ptr(weight.device))

    def __call__(self, x: torch.Tensor, out: torch.Tensor, act: int = 0, residual: torch.Tensor | None = None,
                 bias: torch.Tensor | None = None, rows: int | None = None, x_stride: int | None = None,
                 tile: tuple[int, int, int] | None = None) -> torch.Tensor:
        """``tile`` = (block_n, block_k, num_stages) hint; None chooses by heuristic."""
        m = x.shape[0] if rows is None else rows
        cfg = None
        if tile is not None:
            cfg = ctypes.byref(_native.fml_tile_cfg(128, tile[0], tile[1], 6, tile[2]))
        _native.call(
            "fml_linear_packed", x.data_ptr(), x.stride(0) if x_stride is None else x_stride, self.ptr, self.n,
            self.k, bias.data_ptr() if bias is not None else None, bias.stride(0) if bias is not None else 0,
            residual.data_ptr() if residual is not None else None,
            residual.stride(0) if residual is not None else 0, out.data_ptr(), out.stride(0), m, self.code, act,
            cfg, _native.stream_ptr(x.device),
        )
        return out

    def fused_ok(self, m: int) -> bool:
        """Whether ``fused`` covers an m-token call on the current device."""
        return bool(_native.load().neb_linear_fused_ok(self.n, self.k, m, self.code))

    def fused(self, x: torch.Tensor, out: torch.Tensor, *, act: int = 0, residual: torch.Tensor | None = None,
              ln: tuple | None = None, ln_fold: tuple | None = None, kv: tuple | None = None, ar_ctx=None,
              rows: int | None = None) -> torch.Tensor:
        """Decode-step linear with its neighbours fused into the one launch
        (``neb_linear_fused``):

        ``ln=(gamma, beta, eps)``: the product reads LayerNorm(x) instead of x.
        ``ln_fold=(wsum, wbias, eps)``: this weight is W diag(gamma) (see
        ``ln_fold_vectors``) and the result is LayerNorm(x) W^T, the row
        statistics computed while the product runs.
        ``kv=(k_pool, v_pool, slot_of, start_pos, q_cols, tq)``: output
        features from ``q_cols`` on are appended to the KV pools
        [slots, heads, max_seq, head_dim] at (slot_of[b], start_pos[b] + t).
        ``ar_ctx``: a ``neb_ar`` context; out = residual + SUM over the TP
        group of this product (every rank calls in the same order).
        """
        m = x.shape[0] if rows is None else rows
        fz = _native.neb_fusion()
        if ln is not None:
            g, b, eps = ln
            fz.ln_gamma, fz.ln_beta, fz.ln_eps = g.data_ptr(), b.data_ptr(), float(eps)
        if ln_fold is not None:
            wsum, wbias, eps = ln_fold
            fz.ln_wsum = wsum.data_ptr()
            fz.ln_wbias = wbias.data_ptr() if wbias is not None else None
            fz.ln_eps = float(eps)
        if kv is not None:
            kp, vp, slots, starts, q_cols, tq = kv
            fz.k_pool, fz.v_pool = kp.data_ptr(), vp.data_ptr()
            fz.slot_of, fz.start_pos = slots.data_ptr(), starts.data_ptr()
            fz.q_cols, fz.tq = int(q_cols), int(tq)
            fz.kv_heads, fz.max_seq, fz.head_dim = kp.shape[1], kp.shape[2], kp.shape[3]
        if ar_ctx is not None:
            fz.ar_ctx = ar_ctx
        _native.call(
            "neb_linear_fused", x.data_ptr(), x.stride(0), self.ptr, self.n, self.k,
            residual.data_ptr() if residual is not None else None,
            residual.stride(0) if residual is not None else 0, out.data_ptr(), out.stride(0), m, self.code, act,
            ctypes.byref(fz), _native.stream_ptr(x.device),
        )
        return out


def ln_fold_vectors(weight: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor):
    """For LayerNorm(x) W^T folded into one product (``PackedLinear.fused``
    with ``ln_fold``): returns (W', wsum, wbias) with W' = W diag(gamma) in
    W's dtype, wsum[n] = sum_k W'[n][k] and wbias[n] = sum_k W[n][k] beta[k]
    (fp32; None when beta is zero).  W' is W itself when gamma is all ones."""
    if bool((gamma == 1).all()):
        wp = weight
    else:
        wp = (weight.float() * gamma.float()[None, :]).to(weight.dtype).contiguous()
    wsum = wp.float().sum(dim=1).contiguous()
    wbias = None if bool((beta == 0).all()) else (weight.float() @ beta.float()).contiguous()
    return wp, wsum, wbias
