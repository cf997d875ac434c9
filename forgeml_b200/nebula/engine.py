"""Nebula serving engine: rank 0 drives, the other ranks follow a command wire.

Public surface of the reference Engine (src/nebula/runtime.py:206-516):
``Engine(config, *, context, dtype, max_requests)``, ``forward``, ``serve``,
``release``, ``generate``, ``close``, ``healthy``; the same argument checks and
exception types, the same request-id spaces (callers below 2^62, ``generate``
from 2^62 up), the same configuration handshake and the same poisoning rule:
any failure leaves the engine unhealthy with an empty cache.

Command wire.  The words are the reference protocol's int64 values in its
order: the header [cmd, B, T, start_pos], then the B request ids, then the
B x T tokens (STEP), the B ids (RELEASE) or nothing (STOP).  They travel in one
broadcast of a fixed frame of 4 + 3 * max_requests words when the message fits
(every decode step), otherwise as the header frame followed by one broadcast
of ids and tokens.  Two commands extend the reference's set: STEP_AT, a
single-token step whose requests each sit at their own position (the decode
phase of ``generate_mixed``), and PREFILL, the prefills of several
equal-length groups in one command with their logits broadcasts deferred
(``generate_mixed`` over pipeline stages: stage s + 1 prefills one group while
stage s prefills the next).  The frame is assembled on the host and copied to
the device once; tokens already on the device (the leader's during
``generate``) are copied into it there, never through the host.  A worker
reads a frame back to the host once.

Cache preflight.  Each rank checks a STEP against its own cache replica
(admission of new requests, or positions of running ones) and the ranks agree
on the outcome with a MAX all-reduce.  The agreed value is not waited for on
the host before the step: a rank whose own check failed raises before it
launches anything; a rank whose check passed launches the step and reads the
agreed value afterwards together with the device error word (``_StepHealth``).
Replicas that follow the same commands always agree: a command the cache
rejects fails on every rank before the step, as in the reference.  A replica
that alone disagrees (only a bug or a lost rank makes one) leaves the step
before launching it; the other ranks run the step and fail at their next
collective with that rank -- at once when its process has ended, otherwise
when the bounded peer wait or the process group's timeout expires.

Device health.  After each step the engine queues copies of the agreed
preflight value and of the library's device error word (bounded waits that
expired, positions or token ids out of range) into pinned host memory.  They
are read without waiting at the next call, and with a wait at the end of
every ``generate`` cohort; a nonzero value poisons the engine.
"""

from __future__ import annotations

import contextlib
import hashlib
import threading
from dataclasses import asdict
from typing import NamedTuple

import torch
import torch.distributed as dist

from forgeml_b200.nebula.cache import CacheError
from forgeml_b200.nebula.model import DecoderConfig
from forgeml_b200.nebula.parallel import ParallelContext

CMD_STOP = 0
CMD_STEP = 1
CMD_RELEASE = 2
# Extension of the reference protocol (generate_mixed): a single-token step in
# which every request sits at its own position.  Header [3, B, 1, 0], then the
# B ids, the B tokens and the B positions.
CMD_STEP_AT = 3
# Extension (generate_mixed over pipeline stages): the prefills of several
# equal-length groups in one command.  Header [4, G, W, 0], then W body words:
# b_1, t_1, ..., b_G, t_G, every group's ids, every group's tokens.  All ranks
# agree on the whole batch once, run the groups back to back and broadcast the
# groups' last-position logits from the last stage only after every group has
# been issued, so that stage s + 1 prefills group g while stage s prefills
# group g + 1.
CMD_PREFILL = 4
_GENERATE_ID_BASE = 1 << 62  # engine-issued request ids start here
_MAX_REQUEST_ID = _GENERATE_ID_BASE - 1  # caller-chosen ids stay at or below this
_ID_LIMIT = 1 << 63
_DEFAULT_CONFIG = DecoderConfig()


class EngineFailed(RuntimeError):
    """The engine cannot serve any more (a step failed on the host, on the
    wire or on the device, or it was closed)."""


def _plain_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _validate_prompt(config: DecoderConfig, prompt, max_new) -> None:
    if not isinstance(prompt, (list, tuple)) or len(prompt) == 0:
        raise ValueError("prompt must be a non-empty list of token ids")
    if not all(_plain_int(t) for t in prompt):
        raise TypeError("prompt token ids must be ints")
    bad = next((t for t in prompt if not 0 <= t < config.vocab_size), None)
    if bad is not None:
        raise ValueError(f"token id {bad} out of range")
    if not _plain_int(max_new) or max_new < 0:
        raise ValueError("max_new_tokens must be a non-negative int")
    if len(prompt) + max_new > config.max_seq_len:
        raise ValueError("prompt length + max_new_tokens exceeds max_seq_len")


class _Command(NamedTuple):
    cmd: int
    batch: int
    steps: int
    start: int
    ids: tuple
    tokens: torch.Tensor | None
    positions: tuple = ()
    groups: tuple = ()  # CMD_PREFILL: ((ids, tokens [b, t]), ...)


class _CommandWire:
    """The leader -> worker command channel over the default process group."""

    def __init__(self, max_requests: int, max_seq_len: int, device: torch.device):
        self.frame_words = 4 + 3 * max_requests
        self.max_requests, self.max_seq_len = max_requests, max_seq_len
        self.device = device
        # the ids of the last command received: equal ids of the next one
        # come back as this same tuple, so the id checks downstream see a
        # tuple they already accepted (both are tuples of plain ints)
        self._last_ids: tuple = ()

    def broadcast(self, t: torch.Tensor) -> None:
        """The transport: every frame and body goes through this one call."""
        dist.broadcast(t, src=0)

    # ------------------------------------------------------------ leader
    def send(self, cmd: int, start: int = 0, ids: tuple = (), tokens: torch.Tensor | None = None,
             positions: tuple = ()) -> None:
        b = len(ids)
        t = 0 if tokens is None else int(tokens.shape[1])
        body_words = b + b * t + len(positions)
        if 4 + body_words <= self.frame_words:
            # the whole message in one frame, assembled on the host and copied
            # to the device once (tokens that already live there are copied
            # on the device)
            host = torch.zeros(self.frame_words, dtype=torch.int64)
            host[:4 + b] = torch.tensor([cmd, b, t, start, *ids], dtype=torch.int64)
            on_host = tokens is not None and tokens.device.type == "cpu"
            if t and on_host:
                host[4 + b:4 + b + b * t] = tokens.reshape(-1)
            if positions:
                host[4 + b + b * t:4 + body_words] = torch.tensor(list(positions), dtype=torch.int64)
            frame = host.to(self.device) if self.device.type == "cuda" else host
            if t and not on_host:
                frame[4 + b:4 + b + b * t].copy_(tokens.reshape(-1))
            self.broadcast(frame)
            return
        frame = torch.zeros(self.frame_words, dtype=torch.int64)
        frame[:4] = torch.tensor([cmd, b, t, start], dtype=torch.int64)
        self.broadcast(frame.to(self.device))
        body = torch.empty(body_words, dtype=torch.int64)
        body[:b] = torch.tensor(list(ids), dtype=torch.int64)
        if positions:
            body[b + b * t:] = torch.tensor(list(positions), dtype=torch.int64)
        body = body.to(self.device)
        if t:
            body[b:b + b * t].copy_(tokens.reshape(-1))
        self.broadcast(body)

    def send_prefill(self, groups: list) -> None:
        """CMD_PREFILL: groups of (ids, host tokens [b, t])."""
        words = [v for ids, tok in groups for v in (len(ids), int(tok.shape[1]))]
        words += [r for ids, _ in groups for r in ids]
        body = torch.tensor(words, dtype=torch.int64)
        body = torch.cat([body] + [tok.reshape(-1).to(torch.int64) for _, tok in groups])
        n = int(body.numel())
        head = torch.tensor([CMD_PREFILL, len(groups), n, 0], dtype=torch.int64)
        if 4 + n <= self.frame_words:
            frame = torch.zeros(self.frame_words, dtype=torch.int64)
            frame[:4], frame[4:4 + n] = head, body
            self.broadcast(frame.to(self.device))
            return
        frame = torch.zeros(self.frame_words, dtype=torch.int64)
        frame[:4] = head
        self.broadcast(frame.to(self.device))
        self.broadcast(body.to(self.device))

    def _receive_prefill(self, frame: torch.Tensor, words: list, g: int, n: int) -> _Command:
        if not (0 < g <= self.max_requests and 0 < n <= 3 * self.max_requests * (self.max_seq_len + 1)):
            raise EngineFailed("malformed PREFILL header")
        if 4 + n <= self.frame_words:
            body = frame[4:4 + n]
            bw = words[4:4 + n]
        else:
            body = torch.zeros(n, dtype=torch.int64, device=self.device)
            self.broadcast(body)
            bw = body.tolist()
        sizes = [(bw[2 * i], bw[2 * i + 1]) for i in range(g)]
        total_ids = sum(b for b, _ in sizes)
        if any(b <= 0 or t <= 0 or t > self.max_seq_len for b, t in sizes) or total_ids > self.max_requests or \
                2 * g + total_ids + sum(b * t for b, t in sizes) != n:
            raise EngineFailed("malformed PREFILL body")
        groups, at_id, at_tok = [], 2 * g, 2 * g + total_ids
        for b, t in sizes:
            groups.append((tuple(bw[at_id:at_id + b]), body[at_tok:at_tok + b * t].view(b, t)))
            at_id, at_tok = at_id + b, at_tok + b * t
        return _Command(CMD_PREFILL, g, 0, 0, (), None, (), tuple(groups))

    # ------------------------------------------------------------ worker
    def receive(self) -> _Command:
        frame = torch.zeros(self.frame_words, dtype=torch.int64, device=self.device)
        self.broadcast(frame)
        words = frame.tolist()  # one device -> host read of the whole frame
        cmd, b, t, start = words[:4]
        if cmd == CMD_STOP:
            if (b, t, start) != (0, 0, 0):
                raise EngineFailed("malformed STOP header")
            return _Command(cmd, 0, 0, 0, (), None)
        if cmd == CMD_PREFILL:
            if start != 0:
                raise EngineFailed("malformed PREFILL header")
            return self._receive_prefill(frame, words, b, t)
        if cmd == CMD_STEP:
            if not (0 < b <= self.max_requests and 0 < t <= self.max_seq_len and start >= 0
                    and start + t <= self.max_seq_len):
                raise EngineFailed("malformed STEP header")
        elif cmd == CMD_STEP_AT:
            if not (0 < b <= self.max_requests and t == 1 and start == 0):
                raise EngineFailed("malformed STEP_AT header")
        elif cmd == CMD_RELEASE:
            if not (0 <= b <= self.max_requests and t == 0 and start == 0):
                raise EngineFailed("malformed RELEASE header")
        else:
            raise EngineFailed(f"unknown command {cmd}")
        extra = b if cmd == CMD_STEP_AT else 0
        body_words = b + b * t + extra
        if 4 + body_words <= self.frame_words:
            body = frame[4:4 + body_words]
            bw = words[4:4 + body_words]
        else:
            body = torch.zeros(body_words, dtype=torch.int64, device=self.device)
            self.broadcast(body)
            bw = body.tolist()
        head = bw[:b] + (bw[b + b * t:] if extra else [])
        tokens = body[b:b + b * t].view(b, t) if t else None
        ids = tuple(head[:b])
        if ids == self._last_ids:
            ids = self._last_ids
        else:
            self._last_ids = ids
        return _Command(cmd, b, t, start, ids, tokens, tuple(head[b:]))


class _StepHealth:
    """Deferred, wait-free check of each step's agreed preflight value and of
    the device error word (see the module docstring)."""

    def __init__(self, device: torch.device):
        self.on_cuda = device.type == "cuda"
        self.device = device
        self.pending = False
        if self.on_cuda:
            self.status = torch.zeros(1, dtype=torch.int32).pin_memory()
            self.agreed = torch.zeros(1, dtype=torch.int64).pin_memory()
            self.event = torch.cuda.Event()

    def after_step(self, agreed: torch.Tensor | None) -> None:
        if not self.on_cuda:
            if agreed is not None and int(agreed.item()):
                raise EngineFailed("cache preflight failed on another rank")
            return
        from forgeml_b200 import _native

        stream = torch.cuda.current_stream(self.device)
        _native.device_status_async(self.status, stream.cuda_stream)
        if agreed is not None:
            self.agreed.copy_(agreed.view(1), non_blocking=True)
        self.event.record(stream)
        self.pending = True

    def check(self, wait: bool) -> None:
        if not self.pending or not (wait or self.event.query()):
            return
        self.event.synchronize()
        self.pending = False
        status, agreed = int(self.status[0]), int(self.agreed[0])
        if status:
            from forgeml_b200 import _native

            _native.device_status()  # clears the sticky word
            raise EngineFailed(f"device error {status:#x} in a decode step")
        if agreed:
            raise EngineFailed("cache preflight failed on another rank")


class Engine:
    """Leader/worker serving engine over the native sharded decoder.

    ``decoder_factory(config, context, dtype=..., max_requests=...)`` builds
    the decoder; the default is the native ``ShardedDecoder`` (with ``init``).
    Protocol tests on CPU (Gloo) inject a CPU decoder here; the product path
    has no CPU decoder.
    """

    def __init__(self, config: DecoderConfig = _DEFAULT_CONFIG, *, context: ParallelContext | None = None,
                 dtype: torch.dtype = torch.float32, max_requests: int = 32, decoder_factory=None,
                 init: str = "reference"):
        self._owns_context = context is None
        if context is None:
            context = ParallelContext.from_env(device="cuda" if torch.cuda.is_available() else "cpu")
        if not _plain_int(max_requests) or max_requests <= 0:
            raise ValueError("max_requests must be a positive integer")
        if dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError(f"unsupported dtype {dtype}")
        if context.device.type != "cuda" and dtype != torch.float32:
            raise ValueError("low-precision dtype requires CUDA")
        self.config, self.context, self.max_requests = config, context, max_requests
        nccl = dist.is_available() and dist.is_initialized() and dist.get_backend() == "nccl"
        self._multi = context.world_size > 1 and dist.is_available() and dist.is_initialized()
        wire_device = context.device if nccl else torch.device("cpu")
        self._wire = _CommandWire(max_requests, config.max_seq_len, wire_device)
        if self._multi:
            self._handshake(dtype)
        if decoder_factory is None:
            from forgeml_b200.nebula.runtime import ShardedDecoder

            self.decoder = ShardedDecoder(config, context, dtype=dtype, max_requests=max_requests, init=init)
        else:
            self.decoder = decoder_factory(config, context, dtype=dtype, max_requests=max_requests)
        self._health = _StepHealth(context.device)
        self._healthy = True
        self._closed = False
        self._lock = threading.RLock()
        self._ids_ok: tuple | None = None  # the last request-id tuple _validate_request accepted
        self._ids_ok_internal = False  # ... and whether under the engine's own (internal) rules
        # generate_mixed over pipeline stages sends its prefill groups as one
        # CMD_PREFILL (stages overlap on consecutive groups); False sends them
        # as separate steps, each waiting for the last stage
        self.pipelined_prefill = context.pp_size > 1
        self._next_generated_id = _GENERATE_ID_BASE

    def _handshake(self, dtype: torch.dtype) -> None:
        """Every rank must hold the same configuration, dtype and capacity
        (SHA-256 of their repr, first 8 bytes as a little-endian int64)."""
        digest = hashlib.sha256(repr((asdict(self.config), str(dtype), self.max_requests)).encode()).digest()
        mine = int.from_bytes(digest[:8], "little", signed=True)
        word = torch.tensor([mine], dtype=torch.int64, device=self._wire.device)
        self._wire.broadcast(word)
        if int(word.item()) != mine:
            raise EngineFailed("engine configuration differs across ranks")

    # ------------------------------------------------------------ state
    @property
    def healthy(self) -> bool:
        return self._healthy and not self._closed

    def _require_healthy(self) -> None:
        if not self._healthy or self._closed:
            raise EngineFailed("engine is not healthy")

    def _require_leader(self, what: str) -> None:
        if self._multi and self.context.rank != 0:
            raise EngineFailed(f"{what} must be invoked on rank 0")

    def _invalidate(self) -> None:
        self._healthy = False
        self.decoder.cache.clear()

    # ------------------------------------------------------------ checks
    def _validate_request(self, tokens, request_ids, start_pos, internal: bool) -> None:
        if not isinstance(tokens, torch.Tensor):
            raise TypeError("tokens must be a torch.Tensor")
        if tokens.dtype != torch.long:
            raise ValueError("tokens must be a long tensor")
        if tokens.dim() != 2 or 0 in tokens.shape:
            raise ValueError("tokens must have shape [B, T] with B, T >= 1")
        b, t = tokens.shape
        if b != len(request_ids):
            raise ValueError("request_ids must match batch size")
        if b > self.max_requests:
            raise ValueError("batch exceeds max_requests")
        if not _plain_int(start_pos):
            raise TypeError("start_pos must be an integer")
        if start_pos < 0 or start_pos + t > self.config.max_seq_len:
            raise ValueError("sequence exceeds max_seq_len")
        # A decode loop passes the same id tuple every step; a tuple of ints
        # cannot change, so one accepted under the same rules is not re-checked.
        # (a tuple accepted by the caller's stricter rules also passes the
        # engine's own; not the other way round)
        if request_ids is not self._ids_ok or (self._ids_ok_internal and not internal):
            if len(set(request_ids)) != b:
                raise ValueError("duplicate request ids")
            for r in request_ids:
                if not _plain_int(r) or r < 0:
                    raise ValueError(f"invalid request id {r!r}")
                if r >= _ID_LIMIT:
                    raise ValueError("request id exceeds int64 range")
                if r > _MAX_REQUEST_ID and not internal:
                    raise ValueError("request id exceeds manual range")
            if type(request_ids) is tuple:
                self._ids_ok, self._ids_ok_internal = request_ids, internal
        # Ids the engine produced itself (generate) are in range by
        # construction; a caller's are checked here (one host sync).
        if not internal and bool(((tokens < 0) | (tokens >= self.config.vocab_size)).any()):
            raise ValueError("token ids out of range")

    def _preflight_error(self, request_ids: tuple, start_pos, steps: int) -> int:
        cache = self.decoder.cache
        try:
            if not isinstance(start_pos, int):  # per-request positions (STEP_AT)
                cache.validate_at(request_ids, start_pos, steps)
            elif start_pos == 0:
                cache.check_admission(request_ids)
            else:
                cache.validate(request_ids, start_pos, steps)
        except (CacheError, ValueError):
            return 1
        return 0

    # ------------------------------------------------------------ steps
    def _run_step(self, tokens: torch.Tensor, request_ids: tuple, start_pos, last_only: bool):
        """One step on this rank: preflight, agreement, decoder, health reads.
        ``start_pos`` is an int, or a tuple of per-request positions."""
        err = self._preflight_error(request_ids, start_pos, tokens.shape[1])
        agreed = None
        if self._multi:
            agreed = torch.tensor([err], dtype=torch.int64, device=self._wire.device)
            dist.all_reduce(agreed, op=dist.ReduceOp.MAX)
        if err:
            raise EngineFailed("cache preflight failed")
        with torch.inference_mode():
            logits = self.decoder.forward(tokens, request_ids, start_pos, last_only=last_only)
        self._health.after_step(agreed)
        return logits

    def _run_prefill(self, groups) -> list:
        """CMD_PREFILL on this rank: one admission check and agreement for
        every group, the groups' prefills back to back with their logits
        broadcasts deferred, then the broadcasts in group order.  Returns each
        group's last-position logits [b, 1, V]."""
        all_ids = tuple(r for ids, _ in groups for r in ids)
        err = self._preflight_error(all_ids, 0, 1)
        agreed = None
        if self._multi:
            agreed = torch.tensor([err], dtype=torch.int64, device=self._wire.device)
            dist.all_reduce(agreed, op=dist.ReduceOp.MAX)
        if err:
            raise EngineFailed("cache preflight failed")
        dev = self.context.device
        with torch.inference_mode():
            for ids, tok in groups:
                self.decoder.forward(tok.to(dev), tuple(ids), 0, last_only=True, defer_broadcast=True)
            logits = self.decoder.flush_deferred()
        self._health.after_step(agreed)
        return logits

    def forward(self, tokens: torch.Tensor, request_ids: tuple[int, ...], start_pos: int = 0,
                _internal: bool = False, _last_only: bool = False) -> torch.Tensor:
        with self._lock:
            self._require_healthy()
            self._validate_request(tokens, request_ids, start_pos, internal=_internal)
            self._require_leader("forward")
            try:
                self._health.check(wait=False)
                if self._multi:
                    self._wire.send(CMD_STEP, start_pos, tuple(request_ids), tokens)
                    # the wire has no "last position only" flag: with workers
                    # every rank computes the full logits, as the reference
                    _last_only = False
                return self._run_step(tokens.to(self.context.device), tuple(request_ids), start_pos, _last_only)
            except Exception as exc:
                self._invalidate()
                raise EngineFailed("engine execution failed") from exc

    def serve(self) -> None:
        if not self._multi or self.context.rank == 0:
            raise EngineFailed("serve() is for non-zero ranks")
        try:
            while True:
                self._health.check(wait=False)
                c = self._wire.receive()
                if c.cmd == CMD_STOP:
                    return
                if c.cmd == CMD_STEP:
                    self._run_step(c.tokens.to(self.context.device), c.ids, c.start, False)
                elif c.cmd == CMD_STEP_AT:
                    self._run_step(c.tokens.to(self.context.device), c.ids, c.positions, False)
                elif c.cmd == CMD_PREFILL:
                    self._run_prefill(c.groups)
                else:
                    self.decoder.cache.release(c.ids)
        except Exception as exc:
            self._invalidate()
            raise EngineFailed("worker execution failed") from exc

    def release(self, request_ids: tuple[int, ...]) -> None:
        with self._lock:
            self._require_healthy()
            self._require_leader("release")
            for r in request_ids:
                if not _plain_int(r) or not 0 <= r < _ID_LIMIT:
                    raise ValueError(f"invalid request id {r!r}")
            if len(request_ids) > self.max_requests:
                raise ValueError("release batch exceeds max_requests")
            if not request_ids:
                return
            try:
                self._health.check(wait=False)
                if self._multi:
                    self._wire.send(CMD_RELEASE, 0, tuple(request_ids))
                self.decoder.cache.release(tuple(request_ids))
            except Exception as exc:
                self._invalidate()
                raise EngineFailed("engine execution failed") from exc

    # ------------------------------------------------------------ generate
    def _argmax(self, logits: torch.Tensor) -> torch.Tensor:
        last = logits[:, -1, :]
        if last.is_cuda:
            from forgeml_b200.nebula import ops

            return ops.argmax(last)
        return last.argmax(-1)

    def _fresh_ids(self, n: int) -> tuple:
        ids = []
        while len(ids) < n:
            if self._next_generated_id >= _ID_LIMIT:
                raise EngineFailed("request id space exhausted")
            if not self.decoder.cache.holds(self._next_generated_id):
                ids.append(self._next_generated_id)
            self._next_generated_id += 1
        return tuple(ids)

    def _decode_cohort(self, prompts: list, ids: tuple, max_new: int) -> list[list[int]]:
        """Prefill one cohort of equal-length prompts, then greedy steps; the
        tokens stay on the device until one read at the end."""
        plen = len(prompts[0])
        logits = self.forward(torch.tensor(prompts, dtype=torch.long), ids, 0, _internal=True, _last_only=True)
        produced = [self._argmax(logits)]
        for k in range(1, max_new):
            logits = self.forward(produced[-1].view(-1, 1), ids, plen + k - 1, _internal=True, _last_only=True)
            produced.append(self._argmax(logits))
        rows = torch.stack(produced, dim=1).tolist()
        try:
            self._health.check(wait=True)
        except EngineFailed:
            self._invalidate()
            raise
        return [[int(v) for v in row] for row in rows]

    def generate(self, prompts: list[list[int]], max_new_tokens: int) -> list[list[int]]:
        with self._lock:
            self._require_healthy()
            self._require_leader("generate")
            if not _plain_int(max_new_tokens) or max_new_tokens < 0:
                raise ValueError("max_new_tokens must be a non-negative int")
            for p in prompts:
                _validate_prompt(self.config, p, max_new_tokens)
            if len(prompts) > self.max_requests:
                raise ValueError("batch exceeds max_requests")
            if not prompts or max_new_tokens == 0:
                return [[] for _ in prompts]
            # cohorts of equal prompt length, in order of first appearance
            cohorts: dict[int, list[int]] = {}
            for i, p in enumerate(prompts):
                cohorts.setdefault(len(p), []).append(i)
            results: list[list[int]] = [[] for _ in prompts]
            issued: list[int] = []
            try:
                for members in cohorts.values():
                    ids = self._fresh_ids(len(members))
                    issued.extend(ids)
                    seqs = self._decode_cohort([prompts[i] for i in members], ids, max_new_tokens)
                    for i, seq in zip(members, seqs):
                        results[i] = seq
            finally:
                if issued:
                    if self._healthy:
                        self.release(tuple(issued))
                    else:
                        self.decoder.cache.clear()
            return results

    def _step_at(self, tokens: torch.Tensor, ids: tuple, positions: tuple) -> torch.Tensor:
        """One single-token step of ``ids`` at their own ``positions`` (leader)."""
        try:
            self._health.check(wait=False)
            if self._multi:
                self._wire.send(CMD_STEP_AT, 0, ids, tokens, positions)
            return self._run_step(tokens.to(self.context.device), ids, positions, not self._multi)
        except Exception as exc:
            self._invalidate()
            raise EngineFailed("engine execution failed") from exc

    def generate_mixed(self, prompts: list[list[int]], max_new_tokens: int) -> list[list[int]]:
        """``generate`` for prompts of different lengths in one decode batch.

        The prompts are prefilled in groups of equal length (as ``generate``
        does), then every later greedy step decodes all of them together, each
        request at its own position (STEP_AT).  Each request's tokens are
        those ``generate`` would produce for it, up to the GEMMs' summation
        order at another batch size.  Not part of the reference API."""
        with self._lock:
            self._require_healthy()
            self._require_leader("generate")
            if not _plain_int(max_new_tokens) or max_new_tokens < 0:
                raise ValueError("max_new_tokens must be a non-negative int")
            for p in prompts:
                _validate_prompt(self.config, p, max_new_tokens)
            if len(prompts) > self.max_requests:
                raise ValueError("batch exceeds max_requests")
            if not prompts or max_new_tokens == 0:
                return [[] for _ in prompts]
            groups: dict[int, list[int]] = {}
            for i, p in enumerate(prompts):
                groups.setdefault(len(p), []).append(i)
            ids = self._fresh_ids(len(prompts))
            try:
                dev = self.context.device
                cur = torch.empty(len(prompts), dtype=torch.long, device=dev)
                if self._multi and self.pipelined_prefill:
                    # pipeline stages: every group's prefill in one command
                    batch = [(tuple(ids[i] for i in members), torch.tensor([prompts[i] for i in members],
                                                                           dtype=torch.long))
                             for members in groups.values()]
                    try:
                        self._health.check(wait=False)
                        self._wire.send_prefill(batch)
                        group_logits = self._run_prefill(batch)
                    except Exception as exc:
                        self._invalidate()
                        raise EngineFailed("engine execution failed") from exc
                    for members, logits in zip(groups.values(), group_logits):
                        cur.index_copy_(0, torch.tensor(members, device=dev), self._argmax(logits))
                else:
                    for plen, members in groups.items():
                        logits = self.forward(torch.tensor([prompts[i] for i in members], dtype=torch.long),
                                              tuple(ids[i] for i in members), 0, _internal=True, _last_only=True)
                        cur.index_copy_(0, torch.tensor(members, device=dev), self._argmax(logits))
                produced = [cur]
                positions = tuple(len(p) for p in prompts)
                for _ in range(1, max_new_tokens):
                    logits = self._step_at(produced[-1].view(-1, 1), ids, positions)
                    produced.append(self._argmax(logits))
                    positions = tuple(p + 1 for p in positions)
                rows = torch.stack(produced, dim=1).tolist()
                try:
                    self._health.check(wait=True)
                except EngineFailed:
                    self._invalidate()
                    raise
                return [[int(v) for v in row] for row in rows]
            finally:
                if self._healthy:
                    self.release(ids)
                else:
                    self.decoder.cache.clear()

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            self._closed = True
            try:
                if self._multi and self.context.rank == 0 and self._healthy:
                    with contextlib.suppress(Exception):
                        self._wire.send(CMD_STOP)
                self.decoder.cache.clear()
                closer = getattr(self.decoder, "close", None) or getattr(self.decoder, "release_graphs", None)
                if closer is not None:
                    closer()
                self._healthy = False
            finally:
                if self._owns_context:
                    with contextlib.suppress(Exception):
                        self.context.close()
