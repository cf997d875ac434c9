"""Process layout of a tensor x pipeline parallel Nebula job.

Public surface of the reference ParallelContext (src/nebula/parallel.py:26-123):
``ParallelContext.from_env(tp_size=, pp_size=, device=, timeout_s=)`` with the
fields tp_size, pp_size, rank, world_size, tp_rank, pp_rank, device,
tp_group, owns_process_group; ``all_reduce`` (SUM over the TP group) and
``close``.  The layout is the reference's, because every rank must agree on
it with the reference's workers' view of the world: pipeline stage s holds
ranks [s * tp_size, (s + 1) * tp_size), so ``tp_rank = rank % tp_size`` and
``pp_rank = rank // tp_size``.

On the B200 box a job is one process per GPU (torchrun's WORLD_SIZE, RANK,
LOCAL_RANK), NCCL over NVLink 5 / NVSwitch between them; CPU jobs use Gloo.
The decode step's own TP reductions run over NVLink peer memory
(``peer.PeerAllReduce``); ``all_reduce`` here carries the rest (prefill).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from datetime import timedelta
from typing import Any

import torch
import torch.distributed as dist
from torch.profiler import record_function


def _positive_int(name: str, v) -> int:
    if not isinstance(v, int) or isinstance(v, bool) or v <= 0:
        raise ValueError(f"{name} must be a positive integer")
    return v


def _world_from_environment(device: str) -> tuple[int, int, bool]:
    """(world_size, rank, whether this context must create the process group)."""
    if dist.is_available() and dist.is_initialized():
        backend = dist.get_backend()
        wanted = "gloo" if device == "cpu" else "nccl"
        if backend != wanted:
            raise ValueError(f"preinitialized backend {backend!r} incompatible with {'cpu' if wanted == 'gloo' else 'cuda'}")
        return dist.get_world_size(), dist.get_rank(), False
    if "WORLD_SIZE" not in os.environ:
        return 1, 0, False
    return int(os.environ["WORLD_SIZE"]), int(os.environ.get("RANK", "0")), True


def _bind_device(device: str, world_size: int) -> torch.device:
    dev = torch.device(device)
    if dev.type != "cuda":
        return dev
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA device requested but unavailable")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world_size > 1 and dev.index is not None and dev.index != local:
        raise ValueError(f"device index {dev.index} != LOCAL_RANK {local}")
    dev = torch.device("cuda", local if dev.index is None else dev.index)
    torch.cuda.set_device(dev)
    return dev


@dataclass
class ParallelContext:
    tp_size: int
    pp_size: int
    rank: int
    world_size: int
    tp_rank: int
    pp_rank: int
    device: torch.device
    tp_group: Any
    owns_process_group: bool

    @classmethod
    def from_env(cls, *, tp_size: int = 1, pp_size: int = 1, device: str = "cpu",
                 timeout_s: float = 30.0) -> "ParallelContext":
        _positive_int("tp_size", tp_size)
        _positive_int("pp_size", pp_size)
        if isinstance(timeout_s, bool) or not isinstance(timeout_s, (int, float)) or not (
                math.isfinite(timeout_s) and timeout_s > 0):
            raise ValueError("timeout_s must be a finite positive number")
        if not (device in ("cpu", "cuda") or (isinstance(device, str) and device.startswith("cuda:"))):
            raise ValueError("device must be 'cpu' or 'cuda'")
        world_size, rank, owns = _world_from_environment(device)
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} out of range for world_size {world_size}")
        if world_size != tp_size * pp_size:
            raise ValueError(f"world_size {world_size} != tp_size {tp_size} * pp_size {pp_size}")
        dev = _bind_device(device, world_size)
        timeout = timedelta(seconds=timeout_s)
        if world_size > 1 and owns:
            if not dist.is_available():
                raise RuntimeError("torch.distributed is not available")
            if dev.type == "cuda":
                if not dist.is_nccl_available():
                    raise RuntimeError("nccl backend unavailable")
                dist.init_process_group(backend="nccl", timeout=timeout, device_id=dev)
            else:
                if not dist.is_gloo_available():
                    raise RuntimeError("gloo backend unavailable")
                dist.init_process_group(backend="gloo", timeout=timeout)
        tp_group = None
        if world_size > 1:
            # new_group is collective: every rank creates every stage's group
            groups = [dist.new_group(list(range(s * tp_size, (s + 1) * tp_size)), timeout=timeout)
                      for s in range(pp_size)]
            tp_group = groups[rank // tp_size]
        return cls(tp_size=tp_size, pp_size=pp_size, rank=rank, world_size=world_size, tp_rank=rank % tp_size,
                   pp_rank=rank // tp_size, device=dev, tp_group=tp_group, owns_process_group=owns)

    def all_reduce(self, tensor: torch.Tensor) -> torch.Tensor:
        """In-place SUM over this rank's TP group (a no-op without one)."""
        if self.tp_size > 1 and self.tp_group is not None:
            with record_function("nebula::tp_all_reduce"):
                dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=self.tp_group)
        return tensor

    def close(self) -> None:
        """Destroy the process group if this context created it."""
        if not (self.owns_process_group and dist.is_available() and dist.is_initialized()):
            return
        try:
            dist.destroy_process_group()
        finally:
            self.owns_process_group = False
