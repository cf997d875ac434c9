"""Contiguous per-request KV cache backed by one pool per layer.

Same API, validation and error behaviour as the reference KVCache
(src/nebula/cache.py:10-172).  Storage differs: instead of allocating two
fresh [heads, max_seq_len, head_dim] tensors per request per layer at
``reserve`` time, each owned layer has one pool [max_requests, heads,
max_seq_len, head_dim] for K and one for V, allocated once; a request owns a
pool slot.  A request's per-layer buffer is therefore a view with exactly the
reference's [heads, max_seq_len, head_dim] layout and indexing, and the
decode kernels address every request of a batch through the slot table
without the reference's per-step ``torch.stack`` of the whole prefix.
"""

from __future__ import annotations

import torch


class CacheError(RuntimeError):
    pass


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


class KVCache:
    def __init__(
        self,
        *,
        layer_ids: tuple[int, ...],
        num_heads: int,
        head_dim: int,
        max_seq_len: int,
        max_requests: int,
        device: torch.device,
        dtype: torch.dtype,
    ):
        for name, v in (("num_heads", num_heads), ("head_dim", head_dim), ("max_seq_len", max_seq_len),
                        ("max_requests", max_requests)):
            if not _is_int(v) or v <= 0:
                raise CacheError(f"{name} must be a positive integer")
        if not layer_ids or any(not _is_int(i) or i < 0 for i in layer_ids) or len(set(layer_ids)) != len(layer_ids):
            raise CacheError("layer_ids must be unique non-negative integers")
        if not isinstance(device, torch.device):
            raise CacheError("device must be a torch.device")
        if not isinstance(dtype, torch.dtype):
            raise CacheError("dtype must be a torch.dtype")
        self.layer_ids = tuple(layer_ids)
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.max_requests = max_requests
        self.device = device
        self.dtype = dtype
        shape = (max_requests, num_heads, max_seq_len, head_dim)
        self.k_pool = {lid: torch.empty(shape, device=device, dtype=dtype) for lid in self.layer_ids}
        self.v_pool = {lid: torch.empty(shape, device=device, dtype=dtype) for lid in self.layer_ids}
        # request id -> {layer id -> [k view, v view, length]} (reference bookkeeping shape)
        self._entries: dict[int, dict[int, list]] = {}
        self._slot: dict[int, int] = {}
        self._free = list(range(max_requests - 1, -1, -1))  # pop() yields the lowest slot

    @property
    def active_requests(self) -> int:
        return len(self._entries)

    def _check_ids(self, request_ids: tuple[int, ...]) -> None:
        if not request_ids:
            raise CacheError("request_ids must be non-empty")
        if len(set(request_ids)) != len(request_ids):
            raise CacheError("duplicate request ids")
        for r in request_ids:
            if not _is_int(r) or r < 0 or r >= 1 << 63:
                raise CacheError(f"invalid request id {r!r}")

    def reserve(self, request_ids: tuple[int, ...]) -> None:
        self._check_ids(request_ids)
        for r in request_ids:
            if r in self._entries:
                raise CacheError(f"request id {r} already reserved")
        if len(self._entries) + len(request_ids) > self.max_requests:
            raise CacheError("cache capacity exceeded")
        for r in request_ids:
            s = self._free.pop()
            self._slot[r] = s
            self._entries[r] = {lid: [self.k_pool[lid][s], self.v_pool[lid][s], 0] for lid in self.layer_ids}

    def validate(self, request_ids: tuple[int, ...], start_pos: int, count: int) -> None:
        self._check_ids(request_ids)
        for r in request_ids:
            if r not in self._entries:
                raise CacheError(f"request id {r} is not reserved")
        for name, v in (("start_pos", start_pos), ("count", count)):
            if not _is_int(v):
                raise CacheError(f"{name} must be an integer")
        if count <= 0:
            raise CacheError("count must be positive")
        if start_pos < 0 or start_pos + count > self.max_seq_len:
            raise CacheError("positions out of range")
        for r in request_ids:
            for lid, (_, _, length) in self._entries[r].items():
                if length != start_pos:
                    raise CacheError(f"layer {lid} for request {r} at {length}, expected {start_pos}")

    def slots(self, request_ids: tuple[int, ...]) -> list[int]:
        """Pool slot of each request (the kernels' slot table)."""
        return [self._slot[r] for r in request_ids]

    def advance(self, request_ids: tuple[int, ...], end: int) -> None:
        """Record that every owned layer of these requests now holds ``end`` positions
        (after a fused forward wrote them through the native append kernel)."""
        for r in request_ids:
            for e in self._entries[r].values():
                e[2] = end

    def _check_append(self, layer_id, request_ids, key, value, start_pos) -> int:
        if layer_id not in self.layer_ids:
            raise CacheError(f"layer {layer_id} not owned by this cache")
        self._check_ids(request_ids)
        for r in request_ids:
            if r not in self._entries:
                raise CacheError(f"request id {r} is not reserved")
        if not isinstance(key, torch.Tensor) or not isinstance(value, torch.Tensor):
            raise CacheError("key/value must be torch.Tensor")
        if not _is_int(start_pos):
            raise CacheError("start_pos must be an integer")
        if key.dim() != 4 or value.dim() != 4:
            raise CacheError("key/value must be [B, heads, T, head_dim]")
        b, heads, count, hd = key.shape
        if b != len(request_ids) or heads != self.num_heads or hd != self.head_dim or value.shape != key.shape:
            raise CacheError(f"bad key/value shape {tuple(key.shape)}")
        if count <= 0 or start_pos < 0 or start_pos + count > self.max_seq_len:
            raise CacheError("positions out of range")
        if key.dtype != self.dtype or value.dtype != self.dtype:
            raise CacheError("key/value dtype mismatch")
        if key.device != self.device or value.device != self.device:
            raise CacheError("key/value device mismatch")
        for r in request_ids:
            for lid, (_, _, length) in self._entries[r].items():
                if lid == layer_id:
                    if length != start_pos:
                        raise CacheError(f"layer {layer_id} request {r} at {length}, expected {start_pos}")
                elif length not in (start_pos, start_pos + count):
                    raise CacheError(
                        f"layer {lid} request {r} at {length} while appending layer {layer_id} at {start_pos}+{count}"
                    )
        return count

    def append(self, layer_id: int, request_ids: tuple[int, ...], key: torch.Tensor, value: torch.Tensor,
               start_pos: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Reference-compatible append: write [B, heads, T, hd] at ``start_pos`` and
        return the stacked prefixes [B, heads, end, hd] (a copy, as the reference)."""
        count = self._check_append(layer_id, request_ids, key, value, start_pos)
        end = start_pos + count
        if self.device.type == "cuda":
            from forgeml_b200.nebula import ops

            slot_t = torch.tensor(self.slots(request_ids), dtype=torch.int32, device=self.device)
            start_t = torch.full((len(request_ids),), start_pos, dtype=torch.int32, device=self.device)
            ops.kv_append(key.transpose(1, 2), value.transpose(1, 2), self.k_pool[layer_id],
                          self.v_pool[layer_id], slot_t, start_t)
        else:
            for i, r in enumerate(request_ids):
                kbuf, vbuf, _ = self._entries[r][layer_id]
                kbuf[:, start_pos:end].copy_(key[i])
                vbuf[:, start_pos:end].copy_(value[i])
        ks, vs = [], []
        for r in request_ids:
            ent = self._entries[r][layer_id]
            ent[2] = end
            ks.append(ent[0][:, :end])
            vs.append(ent[1][:, :end])
        return torch.stack(ks), torch.stack(vs)

    def release(self, request_ids: tuple[int, ...]) -> None:
        for r in request_ids:
            if self._entries.pop(r, None) is not None:
                self._free.append(self._slot.pop(r))
        self._free.sort(reverse=True)

    def clear(self) -> None:
        self._entries.clear()
        self._slot.clear()
        self._free = list(range(self.max_requests - 1, -1, -1))
