"""CPU sharded decoder for exercising the native Engine's host logic on Gloo.

The product decoder (forgeml_b200.nebula.ShardedDecoder) runs only on the
sm_100a kernels.  To test the engine protocol (command broadcasts, config
handshake, cache preflight, poisoning, TP all-reduce, PP send/recv, logits
broadcast) without a GPU, tests inject this decoder through
``Engine(decoder_factory=CpuShardedDecoder)``.  Its arithmetic restates the
reference ShardedDecoder (src/nebula/runtime.py:46-189) with torch CPU ops;
it shares the product KVCache (host bookkeeping + CPU storage).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F

from forgeml_b200.nebula.cache import KVCache
from forgeml_b200.nebula.model import TinyDecoder


class CpuShardedDecoder:
    def __init__(self, config, context, *, dtype=torch.float32, max_requests=32):
        tp, pp = context.tp_size, context.pp_size
        self.config, self.context, self.dtype = config, context, dtype
        h, f = config.hidden_size, config.intermediate_size
        per = config.num_layers // pp
        self.owned_layer_ids = tuple(range(context.pp_rank * per, (context.pp_rank + 1) * per))
        lo, hi = context.tp_rank * h // tp, (context.tp_rank + 1) * h // tp
        flo, fhi = context.tp_rank * f // tp, (context.tp_rank + 1) * f // tp
        ref = TinyDecoder(config).to(dtype)
        self.blocks = []
        for lid in self.owned_layer_ids:
            s = ref.blocks[lid]
            self.blocks.append({
                "ln1": (s.ln1.weight.detach(), s.ln1.bias.detach()), "ln2": (s.ln2.weight.detach(), s.ln2.bias.detach()),
                "q": s.q.weight[lo:hi].detach(), "k": s.k.weight[lo:hi].detach(), "v": s.v.weight[lo:hi].detach(),
                "o": s.o.weight[:, lo:hi].detach(), "up": s.up.weight[flo:fhi].detach(),
                "down": s.down.weight[:, flo:fhi].detach()})
        self.tok = ref.token_embedding.weight.detach()
        self.pos = ref.position_embedding.weight.detach()
        self.lnf = (ref.final_norm.weight.detach(), ref.final_norm.bias.detach())
        self.head = ref.lm_head.weight.detach()
        self._deferred = []
        self.hl = config.num_heads // tp
        self.hd = h // config.num_heads
        self.cache = KVCache(layer_ids=self.owned_layer_ids, num_heads=self.hl, head_dim=self.hd,
                             max_seq_len=config.max_seq_len, max_requests=max_requests,
                             device=torch.device("cpu"), dtype=dtype)

    @torch.inference_mode()
    def forward(self, tokens, request_ids, start_pos, last_only=False, defer_broadcast=False):
        if not isinstance(start_pos, int):  # per-request positions: one request at a time
            return torch.cat([self.forward(tokens[i:i + 1], (r,), int(p), last_only)
                              for i, (r, p) in enumerate(zip(request_ids, start_pos))])
        ctx = self.context
        b, t = tokens.shape
        h = self.config.hidden_size
        if start_pos == 0:
            self.cache.reserve(request_ids)
        if ctx.pp_rank == 0:
            x = F.embedding(tokens, self.tok) + F.embedding(torch.arange(start_pos, start_pos + t), self.pos)
        else:
            x = torch.empty(b, t, h, dtype=self.dtype)
            dist.recv(x, src=ctx.rank - ctx.tp_size)
        for blk, lid in zip(self.blocks, self.owned_layer_ids):
            h1 = F.layer_norm(x, (h,), *blk["ln1"], 1e-5)
            q = F.linear(h1, blk["q"]).view(b, t, self.hl, self.hd).transpose(1, 2)
            k = F.linear(h1, blk["k"]).view(b, t, self.hl, self.hd).transpose(1, 2)
            v = F.linear(h1, blk["v"]).view(b, t, self.hl, self.hd).transpose(1, 2)
            k_all, v_all = self.cache.append(lid, request_ids, k.contiguous(), v.contiguous(), start_pos)
            end = start_pos + t
            s = torch.matmul(q, k_all.transpose(-1, -2)) / math.sqrt(self.hd)
            s = s.masked_fill(torch.arange(end)[None, :] > (start_pos + torch.arange(t))[:, None], float("-inf"))
            a = torch.matmul(torch.softmax(s.float(), -1).to(x.dtype), v_all).transpose(1, 2).reshape(b, t, -1)
            part = F.linear(a, blk["o"])
            ctx.all_reduce(part)
            x = x + part
            h2 = F.layer_norm(x, (h,), *blk["ln2"], 1e-5)
            part = F.linear(F.gelu(F.linear(h2, blk["up"]), approximate="tanh"), blk["down"])
            ctx.all_reduce(part)
            x = x + part
        tt = 1 if last_only else t
        if ctx.pp_rank != ctx.pp_size - 1:
            dist.send(x.contiguous(), dst=ctx.rank + ctx.tp_size)
            logits = torch.empty(b, tt, self.config.vocab_size, dtype=self.dtype)
        else:
            xs = x[:, -1:] if last_only else x
            logits = F.linear(F.layer_norm(xs, (h,), *self.lnf, 1e-5), self.head)
        if defer_broadcast:
            self._deferred.append(logits)
        elif ctx.world_size > 1:
            dist.broadcast(logits, src=(ctx.pp_size - 1) * ctx.tp_size)
        return logits

    def flush_deferred(self):
        out, self._deferred = self._deferred, []
        if self.context.world_size > 1:
            for lg in out:
                dist.broadcast(lg, src=(self.context.pp_size - 1) * self.context.tp_size)
        return out
