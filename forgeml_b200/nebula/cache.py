"""Per-request KV cache of the Nebula decoder, held in one slot pool per layer.

Public surface of the reference KVCache (src/nebula/cache.py:10-172): the
keyword constructor, ``reserve`` / ``validate`` / ``append`` / ``release`` /
``clear`` / ``active_requests``, CacheError with the same conditions and
message texts.  The storage is designed for the decode kernels instead:

* every owned layer has one K pool and one V pool of shape
  [max_requests, heads, max_seq_len, head_dim], allocated once; a request is
  given a pool slot at ``reserve`` and keeps it until ``release``.  The slot's
  [heads, max_seq_len, head_dim] block has the reference's per-request buffer
  layout, so position p of head h lives where the reference puts it;
* the kernels address a whole batch through an int32 slot table (``slots``)
  and the step's start positions, reading keys in place -- no per-step stack
  of the prefix;
* bookkeeping is one ``_Ticket`` per request: its slot and the number of
  positions held for each owned layer.  The fused decode step writes K/V of
  every layer inside its kernels and records the new length of all layers at
  once (``advance``), so a ticket keeps one count while its layers agree and
  per-layer counts only while the reference-style ``append`` moves them
  apart: a step's bookkeeping is per request, not per request and layer.

``append`` keeps the reference's contract (write [B, heads, T, hd] at
``start_pos``, return the stacked prefixes [B, heads, end, hd] as a copy) for
callers of the reference API; the decoder itself never uses it.
"""

from __future__ import annotations

import heapq

import torch


class CacheError(RuntimeError):
    pass


_ID_LIMIT = 1 << 63


def _plain_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


class _Ticket:
    """A reserved request: its pool slot and the positions held per owned
    layer -- ``level`` while every owned layer holds the same count
    (``per_layer`` None), else ``per_layer`` {layer id: count}."""

    __slots__ = ("slot", "level", "per_layer")

    def __init__(self, slot: int):
        self.slot = slot
        self.level = 0
        self.per_layer: dict[int, int] | None = None

    def counts(self, layer_ids: tuple[int, ...]) -> dict[int, int]:
        """{layer id: positions held}, in ``layer_ids`` order."""
        return dict.fromkeys(layer_ids, self.level) if self.per_layer is None else self.per_layer

    def set_all(self, end: int) -> None:
        self.level, self.per_layer = end, None

    def set_layer(self, layer_ids: tuple[int, ...], layer_id: int, end: int) -> None:
        if self.per_layer is None:
            if end == self.level:
                return
            self.per_layer = dict.fromkeys(layer_ids, self.level)
        self.per_layer[layer_id] = end
        if all(n == end for n in self.per_layer.values()):
            self.set_all(end)


class KVCache:
    def __init__(self, *, layer_ids: tuple[int, ...], num_heads: int, head_dim: int, max_seq_len: int,
                 max_requests: int, device: torch.device, dtype: torch.dtype):
        sizes = {"num_heads": num_heads, "head_dim": head_dim, "max_seq_len": max_seq_len,
                 "max_requests": max_requests}
        bad = next((k for k, v in sizes.items() if not _plain_int(v) or v <= 0), None)
        if bad is not None:
            raise CacheError(f"{bad} must be a positive integer")
        ids = tuple(layer_ids) if layer_ids else ()
        if not ids or len(set(ids)) != len(ids) or not all(_plain_int(i) and i >= 0 for i in ids):
            raise CacheError("layer_ids must be unique non-negative integers")
        if not isinstance(device, torch.device):
            raise CacheError("device must be a torch.device")
        if not isinstance(dtype, torch.dtype):
            raise CacheError("dtype must be a torch.dtype")
        self.layer_ids = ids
        self.num_heads, self.head_dim = num_heads, head_dim
        self.max_seq_len, self.max_requests = max_seq_len, max_requests
        self.device, self.dtype = device, dtype
        pool_shape = (max_requests, num_heads, max_seq_len, head_dim)
        self.k_pool = {lid: torch.empty(pool_shape, device=device, dtype=dtype) for lid in ids}
        self.v_pool = {lid: torch.empty(pool_shape, device=device, dtype=dtype) for lid in ids}
        self._tickets: dict[int, _Ticket] = {}
        self._free_slots = list(range(max_requests))  # min-heap: the lowest free slot goes first
        # the last request-id tuple check_ids accepted: a decode loop passes
        # the same tuple every step, and a tuple of ints cannot change
        self._ids_ok: tuple | None = None

    # ----------------------------------------------------------- inspection
    @property
    def active_requests(self) -> int:
        return len(self._tickets)

    def holds(self, request_id: int) -> bool:
        return request_id in self._tickets

    def slots(self, request_ids: tuple[int, ...]) -> list[int]:
        """Pool slot of each request, in batch order (the kernels' slot table)."""
        return [self._tickets[r].slot for r in request_ids]

    # ---------------------------------------------------------- validation
    def check_ids(self, request_ids: tuple[int, ...]) -> None:
        if request_ids is self._ids_ok:
            return
        if not request_ids:
            raise CacheError("request_ids must be non-empty")
        seen = set()
        for r in request_ids:
            if not _plain_int(r) or not 0 <= r < _ID_LIMIT:
                raise CacheError(f"invalid request id {r!r}")
            if r in seen:
                raise CacheError("duplicate request ids")
            seen.add(r)
        if type(request_ids) is tuple:
            self._ids_ok = request_ids

    def check_admission(self, request_ids: tuple[int, ...]) -> None:
        """Raise CacheError unless ``reserve(request_ids)`` would succeed."""
        self.check_ids(request_ids)
        taken = next((r for r in request_ids if r in self._tickets), None)
        if taken is not None:
            raise CacheError(f"request id {taken} already reserved")
        if len(self._tickets) + len(request_ids) > self.max_requests:
            raise CacheError("cache capacity exceeded")

    def _tickets_of(self, request_ids: tuple[int, ...]) -> list[_Ticket]:
        self.check_ids(request_ids)
        missing = next((r for r in request_ids if r not in self._tickets), None)
        if missing is not None:
            raise CacheError(f"request id {missing} is not reserved")
        return [self._tickets[r] for r in request_ids]

    def validate(self, request_ids: tuple[int, ...], start_pos: int, count: int) -> None:
        """Raise CacheError unless every owned layer of every request holds
        exactly ``start_pos`` positions and ``count`` more fit."""
        tickets = self._tickets_of(request_ids)
        if not _plain_int(start_pos):
            raise CacheError("start_pos must be an integer")
        if not _plain_int(count):
            raise CacheError("count must be an integer")
        if count <= 0:
            raise CacheError("count must be positive")
        if start_pos < 0 or start_pos + count > self.max_seq_len:
            raise CacheError("positions out of range")
        for r, tk in zip(request_ids, tickets):
            if tk.per_layer is None:
                if tk.level != start_pos:
                    raise CacheError(f"layer {self.layer_ids[0]} for request {r} at {tk.level}, expected {start_pos}")
                continue
            for lid, n in tk.per_layer.items():
                if n != start_pos:
                    raise CacheError(f"layer {lid} for request {r} at {n}, expected {start_pos}")

    def validate_at(self, request_ids: tuple[int, ...], positions: tuple[int, ...], count: int) -> None:
        """``validate((r,), p, count)`` for every request r at its own
        position p (a step whose requests sit at different positions), with
        the ids checked once for the batch (duplicates included)."""
        tickets = self._tickets_of(request_ids)
        if len(positions) != len(request_ids):
            raise CacheError("one position per request")
        if not _plain_int(count):
            raise CacheError("count must be an integer")
        if count <= 0:
            raise CacheError("count must be positive")
        for r, p, tk in zip(request_ids, positions, tickets):
            if not _plain_int(p):
                raise CacheError("start_pos must be an integer")
            if p < 0 or p + count > self.max_seq_len:
                raise CacheError("positions out of range")
            if tk.per_layer is None:
                if tk.level != p:
                    raise CacheError(f"layer {self.layer_ids[0]} for request {r} at {tk.level}, expected {p}")
                continue
            for lid, n in tk.per_layer.items():
                if n != p:
                    raise CacheError(f"layer {lid} for request {r} at {n}, expected {p}")

    # -------------------------------------------------------------- updates
    def reserve(self, request_ids: tuple[int, ...]) -> None:
        self.check_admission(request_ids)
        for r in request_ids:
            self._tickets[r] = _Ticket(heapq.heappop(self._free_slots))

    def advance(self, request_ids: tuple[int, ...], end: int) -> None:
        """Record that every owned layer of these requests now holds ``end``
        positions (the decode kernels wrote them)."""
        for r in request_ids:
            self._tickets[r].set_all(end)

    def append(self, layer_id: int, request_ids: tuple[int, ...], key: torch.Tensor, value: torch.Tensor,
               start_pos: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Reference-compatible append: write [B, heads, T, hd] at ``start_pos``
        and return the stacked prefixes [B, heads, start_pos+T, hd] (a copy)."""
        tickets = self._check_append(layer_id, request_ids, key, value, start_pos)
        end = start_pos + key.shape[2]
        kp, vp = self.k_pool[layer_id], self.v_pool[layer_id]
        if self.device.type == "cuda":
            from forgeml_b200.nebula import ops

            b = len(request_ids)
            slot_t = torch.tensor([tk.slot for tk in tickets], dtype=torch.int32, device=self.device)
            start_t = torch.full((b,), start_pos, dtype=torch.int32, device=self.device)
            ops.kv_append(key.transpose(1, 2), value.transpose(1, 2), kp, vp, slot_t, start_t)
        else:
            for i, tk in enumerate(tickets):
                kp[tk.slot, :, start_pos:end].copy_(key[i])
                vp[tk.slot, :, start_pos:end].copy_(value[i])
        for tk in tickets:
            tk.set_layer(self.layer_ids, layer_id, end)
        index = torch.tensor([tk.slot for tk in tickets], device=self.device)
        return kp.index_select(0, index)[:, :, :end], vp.index_select(0, index)[:, :, :end]

    def _check_append(self, layer_id, request_ids, key, value, start_pos) -> list[_Ticket]:
        if layer_id not in self.k_pool:
            raise CacheError(f"layer {layer_id} not owned by this cache")
        tickets = self._tickets_of(request_ids)
        if not isinstance(key, torch.Tensor) or not isinstance(value, torch.Tensor):
            raise CacheError("key/value must be torch.Tensor")
        if not _plain_int(start_pos):
            raise CacheError("start_pos must be an integer")
        if key.dim() != 4 or value.dim() != 4:
            raise CacheError("key/value must be [B, heads, T, head_dim]")
        b, heads, count, hd = key.shape
        if (b, heads, hd) != (len(request_ids), self.num_heads, self.head_dim) or value.shape != key.shape:
            raise CacheError(f"bad key/value shape {tuple(key.shape)}")
        if count <= 0 or start_pos < 0 or start_pos + count > self.max_seq_len:
            raise CacheError("positions out of range")
        if key.dtype != self.dtype or value.dtype != self.dtype:
            raise CacheError("key/value dtype mismatch")
        if key.device != self.device or value.device != self.device:
            raise CacheError("key/value device mismatch")
        # Layers are appended one after another within a step: the layer being
        # written must be at start_pos, the others at start_pos or already past it.
        for r, tk in zip(request_ids, tickets):
            for lid, n in tk.counts(self.layer_ids).items():
                if lid == layer_id and n != start_pos:
                    raise CacheError(f"layer {layer_id} request {r} at {n}, expected {start_pos}")
                if lid != layer_id and n not in (start_pos, start_pos + count):
                    raise CacheError(
                        f"layer {lid} request {r} at {n} while appending layer {layer_id} at {start_pos}+{count}")
        return tickets

    def release(self, request_ids: tuple[int, ...]) -> None:
        for r in request_ids:
            tk = self._tickets.pop(r, None)
            if tk is not None:
                heapq.heappush(self._free_slots, tk.slot)

    def clear(self) -> None:
        self._tickets.clear()
        self._free_slots = list(range(self.max_requests))
