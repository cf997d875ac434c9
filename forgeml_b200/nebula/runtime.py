"""Nebula sharded decoder and serving engine on the sm_100a kernels.

Drop-in for src/nebula/runtime.py.  The engine keeps the reference's command
protocol bit-for-bit (CMD_STOP/STEP/RELEASE, int64 header [cmd, B, T,
start_pos], ids, tokens; SHA-256 config handshake; cache preflight agreed by
a MAX all-reduce; poisoning on any failure -- runtime.py:19-27,192-516).

The decoder runs every layer on native kernels (no torch compute on the hot
path).  A layer of at most 32 tokens (every decode step of configs 4 and 5)
runs as fused launches of the tcgen05 GEMM (neb_linear_fused) plus the
attention kernel:

  LN1-folded QKV GEMM + KV append -> attention -> o GEMM (+ TP all-reduce)
  + residual -> LN2-folded up GEMM + tanh-GELU -> down GEMM (+ TP all-reduce)
  + residual

with the K/V columns written into the pools by the GEMM epilogue and the TP
partials summed over NVLink by the standalone peer all-reduce kernel (or, opt
in, exchanged from the GEMM epilogue itself).  The two LayerNorms
are folded into the QKV / up products (decode_ln_mode): gamma is folded into
the packed weight and the GEMM corrects its accumulator with the row
statistics it computes while streaming the weight.  Larger steps (prefill) run the unfused chain:

  LN -> fused QKV GEMM (one [3*h_local*hd, h] weight per rank)
     -> KV append into the slot pool -> attention over the pool (no prefix copy)
     -> o GEMM with the residual add fused in the epilogue (TP=1), or
        o GEMM -> NCCL SUM all-reduce -> residual add (TP>1)
  LN -> up GEMM with tanh-GELU epilogue -> down GEMM (+ residual / all-reduce)
  final LN -> lm_head GEMM (only the last position when generating)

Sharding is the reference's (runtime.py:46-123): whole heads of q/k/v rows
and o columns per TP rank, up rows / down columns per TP rank, contiguous
layer ranges per PP stage, embeddings on stage 0, final norm and lm_head on
the last stage, logits broadcast to the world.  Single-token decode steps of
a batch size are captured once into a CUDA graph and replayed (positions and
cache slots are device inputs, so one graph serves every step).
"""

from __future__ import annotations

import contextlib
import ctypes
import hashlib
import os
import threading
from dataclasses import asdict

import torch
import torch.distributed as dist
from torch import nn
from torch.profiler import record_function

from forgeml_b200 import _native
from forgeml_b200.linear import PackedLinear, ln_fold_vectors
from forgeml_b200.nebula import ops
from forgeml_b200.nebula.cache import CacheError, KVCache
from forgeml_b200.nebula.model import DecoderConfig, TinyDecoder
from forgeml_b200.nebula.parallel import ParallelContext
from forgeml_b200.nebula import peer

CMD_STOP = 0
CMD_STEP = 1
CMD_RELEASE = 2
_GENERATE_ID_BASE = 1 << 62
_MAX_REQUEST_ID = (1 << 62) - 1
_DEFAULT_CONFIG = DecoderConfig()


class EngineFailed(RuntimeError):
    pass


class _Gemm:
    """Launches y = x @ W^T (+ epilogue) for a fixed nn.Linear-layout weight W [N, K]."""

    def __init__(self, weight: torch.Tensor, workspace: "_Workspace"):
        self.w = weight
        self.n, self.k = weight.shape
        self.code = _native.dtype_code(weight.dtype)
        self.ws = workspace

    def __call__(self, x: torch.Tensor, out: torch.Tensor, act: int = 0, residual: torch.Tensor | None = None,
                 rows: int | None = None, x_stride: int | None = None) -> torch.Tensor:
        m = x.shape[0] if rows is None else rows
        lda = x.stride(0) if x_stride is None else x_stride
        lib = _native.load()
        need = lib.fml_gemm_workspace_size(m, self.n, self.k, self.code, lda, 1, 1, self.k, x.data_ptr(),
                                           self.w.data_ptr(), None)
        ws_ptr, ws_n = self.ws.get(int(need))
        _native.call(
            "fml_gemm", x.data_ptr(), lda, 1, self.w.data_ptr(), 1, self.k, None, 0,
            residual.data_ptr() if residual is not None else None,
            residual.stride(0) if residual is not None else 0,
            out.data_ptr(), out.stride(0), m, self.n, self.k, self.code, act, None,
            ws_ptr, ws_n, _native.stream_ptr(x.device),
        )
        return out


class _Workspace:
    """Grow-only scratch for the fp32 (3xTF32) GEMM operand split."""

    def __init__(self, device: torch.device):
        self.device = device
        self.buf: torch.Tensor | None = None

    def get(self, nbytes: int):
        if nbytes <= 0:
            return None, 0
        if self.buf is None or self.buf.numel() < nbytes + 256:
            self.buf = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.device)
        base = (self.buf.data_ptr() + 255) // 256 * 256
        return base, nbytes


def _linear(weight: torch.Tensor, ws: "_Workspace"):
    """16-bit weights are packed once for streaming (PackedLinear); fp32 weights
    run the 3xTF32 GEMM on the fly."""
    if weight.dtype in (torch.bfloat16, torch.float16):
        return PackedLinear(weight)
    return _Gemm(weight, ws)


class _Layer:
    def __init__(self, ln1_w, ln1_b, ln2_w, ln2_b, wqkv, wo, wup, wdown, ws):
        self.ln1_w, self.ln1_b, self.ln2_w, self.ln2_b = ln1_w, ln1_b, ln2_w, ln2_b
        self.wqkv, self.wo, self.wup, self.wdown = wqkv, wo, wup, wdown
        self.qkv = _linear(wqkv, ws)
        self.o = _linear(wo, ws)
        self.up = _linear(wup, ws)
        self.down = _linear(wdown, ws)
        # LayerNorm folded into the QKV / up products of the decode step:
        # W diag(gamma) packed (the same packed weight when gamma is all ones)
        # plus the per-feature sums the epilogue needs.
        self.qkv_ln = self.up_ln = None
        if isinstance(self.qkv, PackedLinear):
            for name, w, g, b, lin in (("qkv_ln", wqkv, ln1_w, ln1_b, self.qkv), ("up_ln", wup, ln2_w, ln2_b, self.up)):
                wp, wsum, wbias = ln_fold_vectors(w, g, b)
                setattr(self, name, (lin if wp is w else PackedLinear(wp), wsum, wbias))


def _ln(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, out: torch.Tensor, rows: int,
        x_stride: int | None = None) -> torch.Tensor:
    cols = w.shape[0]
    _native.call("fml_layernorm", x.data_ptr(), cols if x_stride is None else x_stride, w.data_ptr(), b.data_ptr(),
                 1e-5, out.data_ptr(), cols, rows, cols, _native.dtype_code(x.dtype), _native.stream_ptr(x.device))
    return out


class ShardedDecoder(nn.Module):
    """One TP x PP shard of the decoder, executing on the native kernels.

    init="reference": weights are the reference TinyDecoder default init under
    ``config.seed`` (bit-identical to the reference engine's shards).
    init="normal": every weight matrix ~ N(0, init_std) drawn on the device
    from per-tensor seeded generators (each rank draws the full tensor and
    keeps its shard, so shards agree); LayerNorm gamma=1, beta=0.
    """

    def __init__(self, config: DecoderConfig, context: ParallelContext, *, dtype: torch.dtype = torch.float32,
                 max_requests: int = 32, init: str = "reference", init_std: float = 0.02):
        super().__init__()
        tp, pp = context.tp_size, context.pp_size
        if config.num_heads % tp:
            raise ValueError("num_heads must be divisible by tp_size")
        if config.hidden_size % tp:
            raise ValueError("hidden_size must be divisible by tp_size")
        if config.intermediate_size % tp:
            raise ValueError("intermediate_size must be divisible by tp_size")
        if config.num_layers % pp:
            raise ValueError("num_layers must be divisible by pp_size")
        if context.device.type != "cuda":
            raise ValueError("ShardedDecoder runs on the sm_100a kernels and needs a CUDA device")
        if init not in ("reference", "normal"):
            raise ValueError("init must be 'reference' or 'normal'")
        _native.load()
        self.config = config
        self.context = context
        self.dtype = dtype
        dev = context.device
        h, f = config.hidden_size, config.intermediate_size
        self.num_heads_local = config.num_heads // tp
        self.head_dim = h // config.num_heads
        hl_hd = self.num_heads_local * self.head_dim
        per_stage = config.num_layers // pp
        self.owned_layer_ids = tuple(range(context.pp_rank * per_stage, (context.pp_rank + 1) * per_stage))
        row_lo, row_hi = context.tp_rank * h // tp, (context.tp_rank + 1) * h // tp
        f_lo, f_hi = context.tp_rank * f // tp, (context.tp_rank + 1) * f // tp
        self.workspace = _Workspace(dev)
        self.is_first = context.pp_rank == 0
        self.is_last = context.pp_rank == pp - 1

        def put(t: torch.Tensor) -> torch.Tensor:
            return t.detach().to(device=dev, dtype=dtype).contiguous()

        self.layers: list[_Layer] = []
        if init == "reference":
            ref = TinyDecoder(config).to(dtype=dtype)
            for lid in self.owned_layer_ids:
                s = ref.blocks[lid]
                wqkv = torch.cat([s.q.weight[row_lo:row_hi], s.k.weight[row_lo:row_hi], s.v.weight[row_lo:row_hi]])
                self.layers.append(_Layer(
                    put(s.ln1.weight), put(s.ln1.bias), put(s.ln2.weight), put(s.ln2.bias), put(wqkv),
                    put(s.o.weight[:, row_lo:row_hi]), put(s.up.weight[f_lo:f_hi]), put(s.down.weight[:, f_lo:f_hi]),
                    self.workspace))
            if self.is_first:
                self.tok_emb = put(ref.token_embedding.weight)
                self.pos_emb = put(ref.position_embedding.weight)
            if self.is_last:
                self.lnf_w, self.lnf_b = put(ref.final_norm.weight), put(ref.final_norm.bias)
                self.head = put(ref.lm_head.weight)
            del ref
        else:
            def draw(shape, idx):
                g = torch.Generator(device=dev)
                g.manual_seed(config.seed * 1_000_003 + idx)
                return torch.empty(shape, device=dev, dtype=torch.float32).normal_(0.0, init_std, generator=g)

            ones = torch.ones(h, device=dev, dtype=dtype)
            zeros = torch.zeros(h, device=dev, dtype=dtype)
            for lid in self.owned_layer_ids:
                base = 16 + 8 * lid
                q, k, v = (draw((h, h), base + i)[row_lo:row_hi] for i in range(3))
                self.layers.append(_Layer(
                    ones.clone(), zeros.clone(), ones.clone(), zeros.clone(), put(torch.cat([q, k, v])),
                    put(draw((h, h), base + 3)[:, row_lo:row_hi]), put(draw((f, h), base + 4)[f_lo:f_hi]),
                    put(draw((h, f), base + 5)[:, f_lo:f_hi]), self.workspace))
            if self.is_first:
                self.tok_emb = put(draw((config.vocab_size, h), 0))
                self.pos_emb = put(draw((config.max_seq_len, h), 1))
            if self.is_last:
                self.lnf_w, self.lnf_b = ones.clone(), zeros.clone()
                self.head = put(draw((config.vocab_size, h), 2))
        if self.is_last:
            self.head_gemm = _linear(self.head, self.workspace)
        self.cache = KVCache(layer_ids=self.owned_layer_ids, num_heads=self.num_heads_local, head_dim=self.head_dim,
                             max_seq_len=config.max_seq_len, max_requests=max_requests, device=dev, dtype=dtype)
        self._hl_hd = hl_hd
        self._graphs: dict[int, dict] = {}
        self.use_cuda_graphs = True
        # Decode-step TP reductions (B x 1 x d per call) go through the NVLink
        # peer all-reduce fused with the residual add; collective over the TP
        # group, so every rank builds it here in the same order.
        self._peer_ar = None
        if context.tp_size > 1 and dev.type == "cuda" and peer.enabled():
            es = torch.empty((), dtype=dtype).element_size()
            slot = max(16, (max(max_requests, 32) * h * es + 15) // 16 * 16)
            self._peer_ar = peer.PeerAllReduce(context, max_bytes=slot)
        self._fused_cache: dict[int, bool] = {}

    # ------------------------------------------------------------------ math
    def _fused_ok(self, bt: int) -> bool:
        """Whether a layer of ``bt`` tokens runs as the fused launches
        (LN+QKV+KV append, o+all-reduce, LN+up+GELU, down+all-reduce)."""
        ok = self._fused_cache.get(bt)
        if ok is None:
            ctx = self.context
            L = self.layers[0] if self.layers else None
            ok = (L is not None and fused_enabled() and bt <= 32 and self.dtype in (torch.bfloat16, torch.float16)
                  and self.config.hidden_size % 64 == 0
                  and all(isinstance(g, PackedLinear) and g.fused_ok(bt) for g in (L.qkv, L.o, L.up, L.down))
                  and (ctx.tp_size == 1 or (self._peer_ar is not None and self.config.hidden_size % 16 == 0
                                            and self.config.hidden_size * 64 <= self._peer_ar.max_bytes)))
            self._fused_cache[bt] = ok
        return ok

    def _layer_fused(self, L: _Layer, lid: int, x: torch.Tensor, b: int, t: int, slots: torch.Tensor,
                     starts: torch.Tensor) -> torch.Tensor:
        bt = b * t
        h = self.config.hidden_size
        hl, hd, hl_hd = self.num_heads_local, self.head_dim, self._hl_hd
        dev = x.device
        kp, vp = self.cache.k_pool[lid], self.cache.v_pool[lid]
        ln_mode = decode_ln_mode()
        if ln_mode == "fold":
            lin, wsum, wbias = L.qkv_ln
            q = lin.fused(x, torch.empty((bt, hl_hd), dtype=self.dtype, device=dev), ln_fold=(wsum, wbias, 1e-5),
                          kv=(kp, vp, slots, starts, hl_hd, t))
        elif ln_mode == "prologue":
            q = L.qkv.fused(x, torch.empty((bt, hl_hd), dtype=self.dtype, device=dev), ln=(L.ln1_w, L.ln1_b, 1e-5),
                            kv=(kp, vp, slots, starts, hl_hd, t))
        else:
            h1 = _ln(x, L.ln1_w, L.ln1_b, torch.empty_like(x), bt)
            q = L.qkv.fused(h1, torch.empty((bt, hl_hd), dtype=self.dtype, device=dev),
                            kv=(kp, vp, slots, starts, hl_hd, t))
        attn = ops.attention(q.view(b, t, hl, hd), kp, vp, slots, starts).view(bt, hl_hd)
        tp = self.context.tp_size
        if tp == 1:  # residual add in the plain epilogue
            x = L.o(attn, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x)
        elif fused_ar_enabled(tp):
            x = L.o.fused(attn, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x,
                          ar_ctx=self._peer_ar.handle)
        else:
            x = self._tp_sum_add(L.o(attn, torch.empty((bt, h), dtype=self.dtype, device=dev)), x)
        if ln_mode == "fold":
            lin, wsum, wbias = L.up_ln
            mid = lin.fused(x, torch.empty((bt, L.wup.shape[0]), dtype=self.dtype, device=dev),
                            act=_native.ACT_GELU_TANH, ln_fold=(wsum, wbias, 1e-5))
        elif ln_mode == "prologue":
            mid = L.up.fused(x, torch.empty((bt, L.wup.shape[0]), dtype=self.dtype, device=dev),
                             act=_native.ACT_GELU_TANH, ln=(L.ln2_w, L.ln2_b, 1e-5))
        else:
            h2 = _ln(x, L.ln2_w, L.ln2_b, torch.empty_like(x), bt)
            mid = L.up(h2, torch.empty((bt, L.wup.shape[0]), dtype=self.dtype, device=dev), act=_native.ACT_GELU_TANH)
        if tp == 1:
            return L.down(mid, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x)
        if fused_ar_enabled(tp):
            return L.down.fused(mid, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x,
                                ar_ctx=self._peer_ar.handle)
        return self._tp_sum_add(L.down(mid, torch.empty((bt, h), dtype=self.dtype, device=dev)), x)

    def _layer(self, L: _Layer, lid: int, x: torch.Tensor, b: int, t: int, slots: torch.Tensor,
               starts: torch.Tensor) -> torch.Tensor:
        ctx = self.context
        bt = b * t
        if self._fused_ok(bt):
            with record_function("nebula::layer_fused"):
                return self._layer_fused(L, lid, x, b, t, slots, starts)
        h = self.config.hidden_size
        hl, hd, hl_hd = self.num_heads_local, self.head_dim, self._hl_hd
        dev = x.device
        h1 = _ln(x, L.ln1_w, L.ln1_b, torch.empty_like(x), bt)
        qkv = L.qkv(h1, torch.empty((bt, 3 * hl_hd), dtype=self.dtype, device=dev))
        q = qkv[:, :hl_hd].view(b, t, hl, hd)
        k = qkv[:, hl_hd:2 * hl_hd].view(b, t, hl, hd)
        v = qkv[:, 2 * hl_hd:].view(b, t, hl, hd)
        with record_function("nebula::kv_append"):
            ops.kv_append(k, v, self.cache.k_pool[lid], self.cache.v_pool[lid], slots, starts)
        attn = ops.attention(q, self.cache.k_pool[lid], self.cache.v_pool[lid], slots, starts).view(bt, hl_hd)
        if ctx.tp_size == 1:
            x = L.o(attn, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x)
        else:
            x = self._tp_sum_add(L.o(attn, torch.empty((bt, h), dtype=self.dtype, device=dev)), x)
        h2 = _ln(x, L.ln2_w, L.ln2_b, torch.empty_like(x), bt)
        mid = L.up(h2, torch.empty((bt, L.wup.shape[0]), dtype=self.dtype, device=dev), act=_native.ACT_GELU_TANH)
        if ctx.tp_size == 1:
            x = L.down(mid, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x)
        else:
            x = self._tp_sum_add(L.down(mid, torch.empty((bt, h), dtype=self.dtype, device=dev)), x)
        return x

    def _tp_sum_add(self, part: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """x + SUM-all-reduce(part) over the TP group (reference runtime.py:146,154)."""
        if self._peer_ar is not None and self._peer_ar.fits(part) and x.is_contiguous():
            with record_function("nebula::tp_all_reduce_add"):
                return self._peer_ar(part, x, torch.empty_like(x))
        self.context.all_reduce(part)
        return ops.add(x, part)

    def _core(self, tokens: torch.Tensor, slots: torch.Tensor, starts: torch.Tensor, b: int, t: int,
              last_only: bool) -> torch.Tensor:
        """Stage-local forward + hand-off; returns logits on the last stage, else None."""
        ctx = self.context
        h = self.config.hidden_size
        dev = ctx.device
        if self.is_first:
            x = ops.embed(tokens, starts, self.tok_emb, self.pos_emb).view(b * t, h)
        else:
            x = torch.empty((b * t, h), dtype=self.dtype, device=dev)
            with record_function("nebula::pp_recv"):
                dist.recv(x, src=ctx.rank - ctx.tp_size)
        for L, lid in zip(self.layers, self.owned_layer_ids):
            with record_function("nebula::layer"):
                x = self._layer(L, lid, x, b, t, slots, starts)
        if not self.is_last:
            with record_function("nebula::pp_send"):
                dist.send(x, dst=ctx.rank + ctx.tp_size)
            return None
        rows = b if last_only else b * t
        stride = t * h if last_only else h
        src = x[(t - 1):] if last_only else x  # row (t-1) of each request, stride t*h
        hf = _ln(src, self.lnf_w, self.lnf_b, torch.empty((rows, h), dtype=self.dtype, device=dev), rows, x_stride=stride)
        logits = self.head_gemm(hf, torch.empty((rows, self.config.vocab_size), dtype=self.dtype, device=dev))
        return logits

    # ------------------------------------------------------------------ API
    def forward(self, tokens: torch.Tensor, request_ids: tuple[int, ...], start_pos: int,
                last_only: bool = False) -> torch.Tensor:
        ctx = self.context
        b, t = tokens.shape
        v = self.config.vocab_size
        if start_pos == 0:
            self.cache.reserve(request_ids)
        slots_host = torch.tensor(self.cache.slots(request_ids), dtype=torch.int32)
        if tokens.device != ctx.device:
            tokens = tokens.to(ctx.device)
        # Single-token steps replay a captured graph.  With tensor parallelism the
        # graph also holds the NCCL all-reduces (every TP rank captures and
        # replays the same step in lockstep); pipeline stages run eagerly.
        graphable = (t == 1 and ctx.pp_size == 1 and self.use_cuda_graphs
                     and not torch.cuda.is_current_stream_capturing()
                     and (last_only or ctx.world_size > 1))
        if graphable:
            logits = self._replay(tokens, slots_host, start_pos, b)
        else:
            slots = slots_host.to(ctx.device, non_blocking=True)
            starts = torch.full((b,), start_pos, dtype=torch.int32, device=ctx.device)
            logits = self._core(tokens.contiguous(), slots, starts, b, t, last_only)
        tt = 1 if last_only else t
        if logits is None:
            logits = torch.empty((b * tt, v), dtype=self.dtype, device=ctx.device)
        if ctx.pp_size > 1:
            # Only the last pipeline stage computes logits.  (With tensor
            # parallelism alone every rank already holds the same logits: the
            # TP reductions give bit-identical results on all ranks and the
            # lm_head runs on identical inputs, so the reference's broadcast
            # (runtime.py:188) would copy equal values.)
            dist.broadcast(logits, src=(ctx.pp_size - 1) * ctx.tp_size)
        self.cache.advance(request_ids, start_pos + t)
        return logits.view(b, tt, v)

    def _replay(self, tokens: torch.Tensor, slots_host: torch.Tensor, start_pos: int, b: int) -> torch.Tensor:
        g = self._graphs.get(b)
        if g is None:
            return self._capture(tokens, slots_host, start_pos, b)["logits"]
        g["tokens"].copy_(tokens.view(b, 1), non_blocking=True)
        key = tuple(slots_host.tolist())
        if key != g["slot_key"]:
            g["slots"].copy_(slots_host.to(g["slots"].device))
            g["slot_key"] = key
        g["starts"].fill_(start_pos)
        g["graph"].replay()
        return g["logits"]

    def _capture(self, tokens: torch.Tensor, slots_host: torch.Tensor, start_pos: int, b: int) -> dict:
        """Capture the single-token step for batch size ``b``.

        The static inputs are loaded with this step's real tokens, slots and
        positions, the step is run once eagerly (it loads kernel attributes and
        sizes the workspace, and performs this step's real cache writes), then
        recorded and replayed; the replay recomputes the same step, so its cache
        writes are identical and its logits are the step's result.
        """
        dev = self.context.device
        st = {
            "tokens": tokens.view(b, 1).clone(),
            "slots": slots_host.to(dev),
            "slot_key": tuple(slots_host.tolist()),
            "starts": torch.full((b,), start_pos, dtype=torch.int32, device=dev),
        }
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self._core(st["tokens"], st["slots"], st["starts"], b, 1, True)
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            st["logits"] = self._core(st["tokens"], st["slots"], st["starts"], b, 1, True)
        st["graph"] = graph
        self._graphs[b] = st
        graph.replay()
        return st

    def release_graphs(self) -> None:
        self._graphs.clear()

    def close(self) -> None:
        """Release the captured graphs and the peer all-reduce buffers."""
        self.release_graphs()
        if self._peer_ar is not None:
            self._peer_ar.close()
            self._peer_ar = None


def fused_enabled() -> bool:
    """Decode layers run as fused launches unless FORGEML_FUSED_DECODE=0 (a
    diagnostic switch: the unfused chain computes the same step)."""
    return os.environ.get("FORGEML_FUSED_DECODE", "1") != "0"


def fused_ar_enabled(tp: int) -> bool:
    """TP all-reduce inside the o / down GEMM epilogue (FORGEML_FUSED_AR=1),
    or the standalone peer all-reduce kernel after the GEMM (default).
    Measured on B200 at config 4 with the current GEMM epilogue: TP2 1.006 ms
    per step standalone vs 1.046 ms in the epilogue, TP8 1.13 vs 1.38 ms: the
    exchange waits inside the GEMM's critical path, while the standalone
    kernel's prologue overlaps the GEMM's tail."""
    return os.environ.get("FORGEML_FUSED_AR", "0") == "1"


def decode_ln_mode() -> str:
    """How the decode step's pre-QKV / pre-up LayerNorms run
    (FORGEML_DECODE_LN):
      "fold"     folded into the QKV / up products (gamma in the packed
                 weight, statistics computed by the GEMM while its main loop
                 runs, correction in the epilogue): no LayerNorm launch;
      "prologue" normalised by the GEMM's epilogue warps into the operand
                 stages before the main loop (slower on B200: it lengthens
                 the GEMM's critical path);
      "kernel"   a separate LayerNorm launch before the GEMM."""
    v = os.environ.get("FORGEML_DECODE_LN", "fold")
    return v if v in ("fold", "prologue", "kernel") else "fold"


def _validate_prompt(config: DecoderConfig, prompt: list[int], max_new: int) -> None:
    if not isinstance(prompt, (list, tuple)) or not prompt:
        raise ValueError("prompt must be a non-empty list of token ids")
    for tok in prompt:
        if not isinstance(tok, int) or isinstance(tok, bool):
            raise TypeError("prompt token ids must be ints")
        if tok < 0 or tok >= config.vocab_size:
            raise ValueError(f"token id {tok} out of range")
    if not isinstance(max_new, int) or isinstance(max_new, bool) or max_new < 0:
        raise ValueError("max_new_tokens must be a non-negative int")
    if len(prompt) + max_new > config.max_seq_len:
        raise ValueError("prompt length + max_new_tokens exceeds max_seq_len")


class Engine:
    """Leader/worker serving engine (protocol of src/nebula/runtime.py:206-516).

    ``decoder_factory(config, context, dtype=..., max_requests=...)`` builds the
    decoder; the default is the native ``ShardedDecoder``.  Tests that exercise
    the protocol on CPU (Gloo) inject a CPU decoder here; the product path has
    no CPU decoder.
    """

    def __init__(self, config: DecoderConfig = _DEFAULT_CONFIG, *, context: ParallelContext | None = None,
                 dtype: torch.dtype = torch.float32, max_requests: int = 32, decoder_factory=None,
                 init: str = "reference"):
        self._owns_context = context is None
        if context is None:
            context = ParallelContext.from_env(device="cuda" if torch.cuda.is_available() else "cpu")
        if not isinstance(max_requests, int) or isinstance(max_requests, bool) or max_requests <= 0:
            raise ValueError("max_requests must be a positive integer")
        if dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError(f"unsupported dtype {dtype}")
        if context.device.type != "cuda" and dtype != torch.float32:
            raise ValueError("low-precision dtype requires CUDA")
        self.config = config
        self.context = context
        self.max_requests = max_requests
        if dist.is_available() and dist.is_initialized():
            self._comm_device = context.device if dist.get_backend() == "nccl" else torch.device("cpu")
        else:
            self._comm_device = torch.device("cpu")
        if self._world():
            digest = hashlib.sha256(repr((asdict(config), str(dtype), max_requests)).encode()).digest()
            expected = int.from_bytes(digest[:8], "little", signed=True)
            wire = torch.tensor([expected], dtype=torch.int64, device=self._comm_device)
            dist.broadcast(wire, src=0)
            if int(wire.cpu().item()) != expected:
                raise EngineFailed("engine configuration differs across ranks")
        if decoder_factory is None:
            self.decoder = ShardedDecoder(config, context, dtype=dtype, max_requests=max_requests, init=init)
        else:
            self.decoder = decoder_factory(config, context, dtype=dtype, max_requests=max_requests)
        self._healthy = True
        self._closed = False
        self._lock = threading.RLock()
        self._gen_counter = _GENERATE_ID_BASE

    @property
    def healthy(self) -> bool:
        return self._healthy and not self._closed

    @property
    def _is_leader(self) -> bool:
        return self.context.rank == 0

    def _world(self) -> bool:
        return self.context.world_size > 1 and dist.is_initialized()

    def _validate_request(self, tokens, request_ids, start_pos, internal=False) -> None:
        if not isinstance(tokens, torch.Tensor):
            raise TypeError("tokens must be a torch.Tensor")
        if tokens.dtype != torch.long:
            raise ValueError("tokens must be a long tensor")
        if tokens.dim() != 2 or tokens.shape[0] == 0 or tokens.shape[1] == 0:
            raise ValueError("tokens must have shape [B, T] with B, T >= 1")
        if tokens.shape[0] != len(request_ids):
            raise ValueError("request_ids must match batch size")
        if tokens.shape[0] > self.max_requests:
            raise ValueError("batch exceeds max_requests")
        if not isinstance(start_pos, int) or isinstance(start_pos, bool):
            raise TypeError("start_pos must be an integer")
        if start_pos < 0 or start_pos + tokens.shape[1] > self.config.max_seq_len:
            raise ValueError("sequence exceeds max_seq_len")
        if len(set(request_ids)) != len(request_ids):
            raise ValueError("duplicate request ids")
        for r in request_ids:
            if not isinstance(r, int) or isinstance(r, bool) or r < 0:
                raise ValueError(f"invalid request id {r!r}")
            if r >= 1 << 63:
                raise ValueError("request id exceeds int64 range")
            if r > _MAX_REQUEST_ID and not internal:
                raise ValueError("request id exceeds manual range")
        # Token values produced by the engine's own argmax are in range by
        # construction; caller-supplied tokens are checked (a host sync).
        if not internal and ((tokens < 0).any() or (tokens >= self.config.vocab_size).any()):
            raise ValueError("token ids out of range")

    def _bcast(self, tensor: torch.Tensor) -> None:
        if self._world():
            dist.broadcast(tensor, src=0)

    def _invalidate(self) -> None:
        self._healthy = False
        self.decoder.cache.clear()

    def _collective_forward(self, tokens, request_ids, start_pos, last_only=False) -> torch.Tensor:
        err = 0
        cache = self.decoder.cache
        try:
            if start_pos == 0:
                cache._check_ids(request_ids)
                for r in request_ids:
                    if r in cache._entries:
                        raise CacheError(f"request id {r} already reserved")
                if len(cache._entries) + len(request_ids) > cache.max_requests:
                    raise CacheError("cache capacity exceeded")
            else:
                cache.validate(request_ids, start_pos, tokens.shape[1])
        except CacheError:
            err = 1
        if self._world():
            flag = torch.tensor([err], dtype=torch.int64, device=self._comm_device)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
            err = int(flag.item())
        if err:
            raise EngineFailed("cache preflight failed")
        with torch.inference_mode():
            return self.decoder.forward(tokens, request_ids, start_pos, last_only=last_only)

    def forward(self, tokens: torch.Tensor, request_ids: tuple[int, ...], start_pos: int = 0,
                _internal: bool = False, _last_only: bool = False) -> torch.Tensor:
        with self._lock:
            if not self._healthy or self._closed:
                raise EngineFailed("engine is not healthy")
            self._validate_request(tokens, request_ids, start_pos, internal=_internal)
            if self._world() and not self._is_leader:
                raise EngineFailed("forward must be invoked on rank 0")
            try:
                if self._world():
                    header = torch.tensor([CMD_STEP, tokens.shape[0], tokens.shape[1], start_pos], dtype=torch.int64,
                                          device=self._comm_device)
                    self._bcast(header)
                    self._bcast(torch.tensor(list(request_ids), dtype=torch.int64, device=self._comm_device))
                    self._bcast(tokens.to(self._comm_device).contiguous())
                    # The reference protocol has no "last position only" flag, so with
                    # workers every rank computes (and broadcasts) full logits.
                    _last_only = False
                return self._collective_forward(tokens.to(self.context.device), request_ids, start_pos,
                                                last_only=_last_only)
            except Exception as exc:
                self._invalidate()
                raise EngineFailed("engine execution failed") from exc

    def serve(self) -> None:
        if self._is_leader or not self._world():
            raise EngineFailed("serve() is for non-zero ranks")
        try:
            while True:
                header = torch.zeros(4, dtype=torch.int64, device=self._comm_device)
                dist.broadcast(header, src=0)
                cmd, batch, time_, start_pos = (int(v) for v in header.tolist())
                if cmd == CMD_STOP:
                    if batch != 0 or time_ != 0 or start_pos != 0:
                        raise EngineFailed("malformed STOP header")
                    return
                if cmd == CMD_STEP:
                    if (batch <= 0 or batch > self.max_requests or time_ <= 0 or time_ > self.config.max_seq_len
                            or start_pos < 0 or start_pos + time_ > self.config.max_seq_len):
                        raise EngineFailed("malformed STEP header")
                    ids = torch.zeros(batch, dtype=torch.int64, device=self._comm_device)
                    dist.broadcast(ids, src=0)
                    tokens = torch.zeros(batch, time_, dtype=torch.int64, device=self._comm_device)
                    dist.broadcast(tokens, src=0)
                    self._collective_forward(tokens.to(self.context.device), tuple(int(i) for i in ids.tolist()),
                                             start_pos)
                elif cmd == CMD_RELEASE:
                    if batch < 0 or batch > self.max_requests or time_ != 0 or start_pos != 0:
                        raise EngineFailed("malformed RELEASE header")
                    ids = torch.zeros(batch, dtype=torch.int64, device=self._comm_device)
                    dist.broadcast(ids, src=0)
                    self.decoder.cache.release(tuple(int(i) for i in ids.tolist()))
                else:
                    raise EngineFailed(f"unknown command {cmd}")
        except Exception as exc:
            self._invalidate()
            raise EngineFailed("worker execution failed") from exc

    def release(self, request_ids: tuple[int, ...]) -> None:
        with self._lock:
            if self._closed or not self._healthy:
                raise EngineFailed("engine is not healthy")
            if self._world() and not self._is_leader:
                raise EngineFailed("release must be invoked on rank 0")
            for r in request_ids:
                if not isinstance(r, int) or isinstance(r, bool) or r < 0 or r >= 1 << 63:
                    raise ValueError(f"invalid request id {r!r}")
            if len(request_ids) > self.max_requests:
                raise ValueError("release batch exceeds max_requests")
            if not request_ids:
                return
            try:
                if self._world():
                    header = torch.tensor([CMD_RELEASE, len(request_ids), 0, 0], dtype=torch.int64,
                                          device=self._comm_device)
                    self._bcast(header)
                    self._bcast(torch.tensor(list(request_ids), dtype=torch.int64, device=self._comm_device))
                self.decoder.cache.release(request_ids)
            except Exception as exc:
                self._invalidate()
                raise EngineFailed("engine execution failed") from exc

    def _next_tokens(self, logits: torch.Tensor) -> torch.Tensor:
        last = logits[:, -1, :]
        if last.is_cuda:
            return ops.argmax(last)
        return last.argmax(-1)

    def generate(self, prompts: list[list[int]], max_new_tokens: int) -> list[list[int]]:
        with self._lock:
            if not self._healthy or self._closed:
                raise EngineFailed("engine is not healthy")
            if not self._is_leader and self._world():
                raise EngineFailed("generate must be invoked on rank 0")
            if not isinstance(max_new_tokens, int) or isinstance(max_new_tokens, bool) or max_new_tokens < 0:
                raise ValueError("max_new_tokens must be a non-negative int")
            for p in prompts:
                _validate_prompt(self.config, p, max_new_tokens)
            if len(prompts) > self.max_requests:
                raise ValueError("batch exceeds max_requests")
            if not prompts:
                return []
            if max_new_tokens == 0:
                return [[] for _ in prompts]
            results: list[list[int]] = [[] for _ in prompts]
            cohorts: dict[int, list[int]] = {}
            for i, p in enumerate(prompts):
                cohorts.setdefault(len(p), []).append(i)
            issued: list[int] = []
            try:
                for plen, idxs in cohorts.items():
                    ids = []
                    for _ in idxs:
                        while self._gen_counter in self.decoder.cache._entries:
                            self._gen_counter += 1
                        if self._gen_counter >= 1 << 63:
                            raise EngineFailed("request id space exhausted")
                        ids.append(self._gen_counter)
                        self._gen_counter += 1
                    issued.extend(ids)
                    tokens = torch.tensor([prompts[i] for i in idxs], dtype=torch.long)
                    logits = self.forward(tokens, tuple(ids), 0, _internal=True, _last_only=True)
                    nxt = self._next_tokens(logits)
                    produced = [nxt]
                    for step in range(1, max_new_tokens):
                        logits = self.forward(nxt.view(-1, 1), tuple(ids), plen + step - 1, _internal=True,
                                              _last_only=True)
                        nxt = self._next_tokens(logits)
                        produced.append(nxt)
                    seqs = torch.stack(produced, dim=1).tolist()  # one device->host read per cohort
                    for j, i in enumerate(idxs):
                        results[i] = [int(v) for v in seqs[j]]
            finally:
                if issued and self._healthy:
                    self.release(tuple(issued))
                elif issued:
                    self.decoder.cache.clear()
            return results

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            self._closed = True
            try:
                if self._world() and self._is_leader and self._healthy:
                    header = torch.tensor([CMD_STOP, 0, 0, 0], dtype=torch.int64, device=self._comm_device)
                    with contextlib.suppress(Exception):
                        self._bcast(header)
                self.decoder.cache.clear()
                if hasattr(self.decoder, "close"):
                    self.decoder.close()
                elif hasattr(self.decoder, "release_graphs"):
                    self.decoder.release_graphs()
                self._healthy = False
            finally:
                if self._owns_context:
                    with contextlib.suppress(Exception):
                        self.context.close()
