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
are folded into the QKV / up products (decode_ln): gamma is folded into
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

import ctypes

import torch
import torch.distributed as dist
from torch import nn
from torch.profiler import record_function

from forgeml_b200 import _native
from forgeml_b200.linear import PackedLinear, ln_fold_vectors
from forgeml_b200.nebula import ops
from forgeml_b200.nebula.cache import KVCache
from forgeml_b200.nebula.model import DecoderConfig, TinyDecoder, normal_weight
from forgeml_b200.nebula.parallel import ParallelContext
from forgeml_b200.nebula import peer

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
            def draw(key):
                return normal_weight(config, key, dev, init_std)

            ones = torch.ones(h, device=dev, dtype=dtype)
            zeros = torch.zeros(h, device=dev, dtype=dtype)
            for lid in self.owned_layer_ids:
                q, k, v = (draw(f"{lid}.{n}")[row_lo:row_hi] for n in ("q", "k", "v"))
                self.layers.append(_Layer(
                    ones.clone(), zeros.clone(), ones.clone(), zeros.clone(), put(torch.cat([q, k, v])),
                    put(draw(f"{lid}.o")[:, row_lo:row_hi]), put(draw(f"{lid}.up")[f_lo:f_hi]),
                    put(draw(f"{lid}.down")[:, f_lo:f_hi]), self.workspace))
            if self.is_first:
                self.tok_emb = put(draw("tok"))
                self.pos_emb = put(draw("pos"))
            if self.is_last:
                self.lnf_w, self.lnf_b = ones.clone(), zeros.clone()
                self.head = put(draw("head"))
        if self.is_last:
            self.head_gemm = _linear(self.head, self.workspace)
        self.cache = KVCache(layer_ids=self.owned_layer_ids, num_heads=self.num_heads_local, head_dim=self.head_dim,
                             max_seq_len=config.max_seq_len, max_requests=max_requests, device=dev, dtype=dtype)
        self._hl_hd = hl_hd
        self._graphs: dict[int, dict] = {}
        self._deferred: list[torch.Tensor] = []  # logits awaiting flush_deferred()
        self.use_cuda_graphs = True
        # Decode-step TP reductions (B x 1 x d per call) go through the NVLink
        # peer all-reduce fused with the residual add; collective over the TP
        # group, so every rank builds it here in the same order.
        self._peer_ar = None
        if context.tp_size > 1 and dev.type == "cuda":
            es = torch.empty((), dtype=dtype).element_size()
            slot = max(16, (max(max_requests, 32) * h * es + 15) // 16 * 16)
            self._peer_ar = peer.PeerAllReduce(context, max_bytes=slot)
        # Decode steps of 4 or more TP ranks can run as several batch lanes
        # (_core), each lane reducing through its own peer context, up to
        # MAX_LANES (every rank creates the same contexts, in the same
        # order).  One lane is the default: measured at TP8 on B200s (c4,
        # batch 32), two lanes took 1.32 ms per step against 0.79 ms for
        # one -- the lanes' launches contend instead of filling each other's
        # latency.
        self.decode_lanes = 1
        self._lane_ars = [self._peer_ar]
        self._lane_streams: list = []
        if self._peer_ar is not None and context.pp_size == 1 and context.tp_size >= 4:
            self._lane_ars += [peer.PeerAllReduce(context, max_bytes=self._peer_ar.max_bytes)
                               for _ in range(self.MAX_LANES - 1)]
        self._fused_cache: dict[tuple, bool] = {}
        # Decode-step layout choices (the defaults are the measured best; the
        # alternatives compute the same step and are kept for tests):
        #   fused_decode        layers of <= 32 tokens as fused GEMM launches
        #   decode_ln           "fold": LayerNorms folded into the QKV / up
        #                       products; "prologue": normalised by the GEMM's
        #                       epilogue warps; "kernel": a LayerNorm launch
        #   all_reduce_in_gemm  TP exchange inside the o / down GEMM epilogue
        #                       instead of the standalone peer all-reduce
        #                       (measured slower: the exchange then waits on
        #                       the GEMM's critical path)
        self.fused_decode = True
        self.decode_ln = "fold"
        self.all_reduce_in_gemm = False

    # ------------------------------------------------------------------ math
    MAX_LANES = 4

    def _fused_ok(self, bt: int) -> bool:
        """Whether a layer of ``bt`` tokens runs as the fused launches
        (LN+QKV+KV append, o+all-reduce, LN+up+GELU, down+all-reduce)."""
        key = (bt, self.fused_decode)
        ok = self._fused_cache.get(key)
        if ok is None:
            ctx = self.context
            L = self.layers[0] if self.layers else None
            ok = (L is not None and self.fused_decode and bt <= 32 and self.dtype in (torch.bfloat16, torch.float16)
                  and self.config.hidden_size % 64 == 0
                  and all(isinstance(g, PackedLinear) and g.fused_ok(bt) for g in (L.qkv, L.o, L.up, L.down))
                  and (ctx.tp_size == 1 or (self._peer_ar is not None and self.config.hidden_size % 16 == 0
                                            and self.config.hidden_size * 64 <= self._peer_ar.max_bytes)))
            self._fused_cache[key] = ok
        return ok

    def _layer_fused(self, L: _Layer, lid: int, x: torch.Tensor, b: int, t: int, slots: torch.Tensor,
                     starts: torch.Tensor, ar) -> torch.Tensor:
        bt = b * t
        h = self.config.hidden_size
        hl, hd, hl_hd = self.num_heads_local, self.head_dim, self._hl_hd
        dev = x.device
        kp, vp = self.cache.k_pool[lid], self.cache.v_pool[lid]
        ln_mode = self.decode_ln
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
        elif self.all_reduce_in_gemm:
            x = L.o.fused(attn, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x,
                          ar_ctx=ar.handle)
        else:
            x = self._tp_sum_add(L.o(attn, torch.empty((bt, h), dtype=self.dtype, device=dev)), x, ar)
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
        if self.all_reduce_in_gemm:
            return L.down.fused(mid, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x,
                                ar_ctx=ar.handle)
        return self._tp_sum_add(L.down(mid, torch.empty((bt, h), dtype=self.dtype, device=dev)), x, ar)

    def _layer(self, L: _Layer, lid: int, x: torch.Tensor, b: int, t: int, slots: torch.Tensor,
               starts: torch.Tensor, ar) -> torch.Tensor:
        ctx = self.context
        bt = b * t
        if self._fused_ok(bt):
            with record_function("nebula::layer_fused"):
                return self._layer_fused(L, lid, x, b, t, slots, starts, ar)
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
            x = self._tp_sum_add(L.o(attn, torch.empty((bt, h), dtype=self.dtype, device=dev)), x, ar)
        h2 = _ln(x, L.ln2_w, L.ln2_b, torch.empty_like(x), bt)
        mid = L.up(h2, torch.empty((bt, L.wup.shape[0]), dtype=self.dtype, device=dev), act=_native.ACT_GELU_TANH)
        if ctx.tp_size == 1:
            x = L.down(mid, torch.empty((bt, h), dtype=self.dtype, device=dev), residual=x)
        else:
            x = self._tp_sum_add(L.down(mid, torch.empty((bt, h), dtype=self.dtype, device=dev)), x, ar)
        return x

    def _tp_sum_add(self, part: torch.Tensor, x: torch.Tensor, ar) -> torch.Tensor:
        """x + SUM-all-reduce(part) over the TP group (reference runtime.py:146,154)."""
        if ar is not None and ar.fits(part) and x.is_contiguous():
            with record_function("nebula::tp_all_reduce_add"):
                return ar(part, x, torch.empty_like(x))
        self.context.all_reduce(part)
        return ops.add(x, part)

    def _lanes(self, b: int, t: int) -> list[int]:
        """Rows of each batch lane of a step of ``b`` requests (see _core):
        ``decode_lanes`` contiguous groups of near-equal size, or one."""
        n = min(self.decode_lanes, b, len(self._lane_ars))
        if n <= 1 or t != 1 or self.context.pp_size != 1 or any(a is None for a in self._lane_ars[:n]):
            return [b]
        rows = [b // n + (1 if i < b % n else 0) for i in range(n)]
        return rows if self._fused_ok(max(rows)) else [b]

    def _core(self, tokens: torch.Tensor, slots: torch.Tensor, starts: torch.Tensor, b: int, t: int,
              last_only: bool) -> torch.Tensor:
        """Stage-local forward + hand-off; returns logits on the last stage, else None.

        With tensor parallelism a decode step is a chain of short launches
        whose time is mostly latency (the weights a rank streams shrink with
        the TP degree, a launch's fixed cost does not).  There the batch runs
        as several lanes on their own streams, each with its own peer
        all-reduce context: one lane's GEMMs, attention and reductions fill
        the others' waits.  Every request's arithmetic is that of an unsplit
        step of its lane's rows."""
        lanes = self._lanes(b, t)
        if len(lanes) == 1:
            return self._core_rows(tokens, slots, starts, b, t, last_only, self._peer_ar)
        dev = self.context.device
        main = torch.cuda.current_stream(dev)
        while len(self._lane_streams) < len(lanes) - 1:
            self._lane_streams.append(torch.cuda.Stream(device=dev))
        # the layers per lane (lane 0 on the calling stream); the final
        # LayerNorm and lm_head once for the whole batch (the head's weights
        # are streamed once per step)
        outs, r0 = [], 0
        for i, rows in enumerate(lanes):
            sl = slice(r0, r0 + rows)
            if i == 0:
                outs.append(self._core_rows(tokens[sl], slots[sl], starts[sl], rows, 1, last_only,
                                            self._lane_ars[0], head=False))
            else:
                st = self._lane_streams[i - 1]
                st.wait_stream(main)
                with torch.cuda.stream(st):
                    outs.append(self._core_rows(tokens[sl], slots[sl], starts[sl], rows, 1, last_only,
                                                self._lane_ars[i], head=False))
            r0 += rows
        for st in self._lane_streams[:len(lanes) - 1]:
            main.wait_stream(st)
        return self._head(torch.cat(outs), b, 1, last_only)

    def _core_rows(self, tokens: torch.Tensor, slots: torch.Tensor, starts: torch.Tensor, b: int, t: int,
                   last_only: bool, ar, head: bool = True) -> torch.Tensor:
        """Forward of these rows on this stage (all-reduce context ``ar``):
        logits on the last stage (the hidden rows when ``head`` is False),
        else None."""
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
                x = self._layer(L, lid, x, b, t, slots, starts, ar)
        if not self.is_last:
            with record_function("nebula::pp_send"):
                dist.send(x, dst=ctx.rank + ctx.tp_size)
            return None
        return self._head(x, b, t, last_only) if head else x

    def _head(self, x: torch.Tensor, b: int, t: int, last_only: bool) -> torch.Tensor:
        """Final LayerNorm and lm_head of hidden rows x [b*t, h]."""
        h = self.config.hidden_size
        dev = x.device
        rows = b if last_only else b * t
        stride = t * h if last_only else h
        src = x[(t - 1):] if last_only else x  # row (t-1) of each request, stride t*h
        hf = _ln(src, self.lnf_w, self.lnf_b, torch.empty((rows, h), dtype=self.dtype, device=dev), rows, x_stride=stride)
        return self.head_gemm(hf, torch.empty((rows, self.config.vocab_size), dtype=self.dtype, device=dev))

    # ------------------------------------------------------------------ API
    def forward(self, tokens: torch.Tensor, request_ids: tuple[int, ...], start_pos,
                last_only: bool = False, defer_broadcast: bool = False) -> torch.Tensor:
        """Logits [B, T or 1, V] of one step.  ``start_pos`` is the position of
        the batch's first token (0 reserves the requests), or -- for
        single-token steps of requests already in the cache -- a sequence with
        each request's own position (the kernels take per-request positions)."""
        ctx = self.context
        b, t = tokens.shape
        v = self.config.vocab_size
        if isinstance(start_pos, int):
            if start_pos == 0:
                self.cache.reserve(request_ids)
            positions = [start_pos] * b
        else:
            positions = [int(p) for p in start_pos]
            if t != 1 or len(positions) != b:
                raise ValueError("per-request positions need single-token steps, one position per request")
        slots_host = torch.tensor(self.cache.slots(request_ids), dtype=torch.int32)
        starts_host = torch.tensor(positions, dtype=torch.int32)
        if tokens.device != ctx.device:
            tokens = tokens.to(ctx.device)
        # Single-token steps replay a captured graph.  With tensor parallelism the
        # graph also holds the TP reductions (every TP rank captures and replays
        # the same step in lockstep); pipeline stages run eagerly.
        graphable = (t == 1 and ctx.pp_size == 1 and self.use_cuda_graphs
                     and not torch.cuda.is_current_stream_capturing()
                     and (last_only or ctx.world_size > 1))
        if graphable:
            logits = self._replay(tokens, slots_host, starts_host, b)
        else:
            slots = slots_host.to(ctx.device, non_blocking=True)
            starts = starts_host.to(ctx.device, non_blocking=True)
            logits = self._core(tokens.contiguous(), slots, starts, b, t, last_only)
        tt = 1 if last_only else t
        if logits is None:
            logits = torch.empty((b * tt, v), dtype=self.dtype, device=ctx.device)
        if defer_broadcast:
            # the logits travel later, in order, with flush_deferred()
            self._deferred.append(logits.view(b, 1 if last_only else t, v))
        elif ctx.pp_size > 1:
            # Only the last pipeline stage computes logits.  (With tensor
            # parallelism alone every rank already holds the same logits: the
            # TP reductions give bit-identical results on all ranks and the
            # lm_head runs on identical inputs, so the reference's broadcast
            # (runtime.py:188) would copy equal values.)
            dist.broadcast(logits, src=(ctx.pp_size - 1) * ctx.tp_size)
        if len(set(positions)) == 1:
            self.cache.advance(request_ids, positions[0] + t)
        else:
            for r, p in zip(request_ids, positions):
                self.cache.advance((r,), p + t)
        return logits.view(b, tt, v)

    def flush_deferred(self) -> list[torch.Tensor]:
        """Broadcast, from the last pipeline stage and in call order, the
        logits of every forward(..., defer_broadcast=True) since the last
        flush; returns them ([B, T or 1, V] each).  Deferring lets the stages
        of a pipeline work on consecutive steps at once: no rank waits for the
        last stage between them."""
        out, self._deferred = self._deferred, []
        ctx = self.context
        if ctx.pp_size > 1:
            for lg in out:
                dist.broadcast(lg, src=(ctx.pp_size - 1) * ctx.tp_size)
        return out

    def _replay(self, tokens: torch.Tensor, slots_host: torch.Tensor, starts_host: torch.Tensor,
                b: int) -> torch.Tensor:
        g = self._graphs.get(b)
        if g is None:
            return self._capture(tokens, slots_host, starts_host, b)["logits"]
        g["tokens"].copy_(tokens.view(b, 1), non_blocking=True)
        key = tuple(slots_host.tolist())
        if key != g["slot_key"]:
            g["slots"].copy_(slots_host.to(g["slots"].device))
            g["slot_key"] = key
        first = int(starts_host[0])
        if bool((starts_host == first).all()):
            g["starts"].fill_(first)
        else:
            g["starts"].copy_(starts_host, non_blocking=True)
        g["graph"].replay()
        return g["logits"]

    def _capture(self, tokens: torch.Tensor, slots_host: torch.Tensor, starts_host: torch.Tensor, b: int) -> dict:
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
            "starts": starts_host.to(dev),
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
        for ar in self._lane_ars:  # lane 0 is the step's own context
            if ar is not None:
                ar.close()
        self._lane_ars = [None]
        self._peer_ar = None


# The serving engine lives in engine.py; the reference exposes it from this module.
from forgeml_b200.nebula.engine import (CMD_RELEASE, CMD_STEP, CMD_STOP, Engine, EngineFailed,  # noqa: E402,F401
                                        _validate_prompt)
