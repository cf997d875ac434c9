"""Tensor/pipeline-parallel process layout over torch.distributed.

Same contract as the reference ParallelContext (src/nebula/parallel.py:26-123):
torchrun environment (WORLD_SIZE / RANK / LOCAL_RANK), NCCL for CUDA and
Gloo for CPU, TP groups as contiguous rank blocks per pipeline stage,
``tp_rank = rank % tp_size`` and ``pp_rank = rank // tp_size``, SUM
all-reduce over the TP group.  On B200 the NCCL communicator runs over
NVLink 5 / NVSwitch (one process per GPU).
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
        for name, v in (("tp_size", tp_size), ("pp_size", pp_size)):
            if not isinstance(v, int) or isinstance(v, bool) or v <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if (not isinstance(timeout_s, (int, float)) or isinstance(timeout_s, bool)
                or not math.isfinite(timeout_s) or timeout_s <= 0):
            raise ValueError("timeout_s must be a finite positive number")
        if device not in ("cpu", "cuda") and not (isinstance(device, str) and device.startswith("cuda:")):
            raise ValueError("device must be 'cpu' or 'cuda'")
        if dist.is_available() and dist.is_initialized():
            world_size, rank, owns = dist.get_world_size(), dist.get_rank(), False
            backend = dist.get_backend()
            if device == "cpu" and backend != "gloo":
                raise ValueError(f"preinitialized backend {backend!r} incompatible with cpu")
            if device != "cpu" and backend != "nccl":
                raise ValueError(f"preinitialized backend {backend!r} incompatible with cuda")
        elif os.environ.get("WORLD_SIZE") is None:
            world_size, rank, owns = 1, 0, False
        else:
            world_size = int(os.environ["WORLD_SIZE"])
            rank = int(os.environ.get("RANK", "0"))
            owns = True
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} out of range for world_size {world_size}")
        if world_size != tp_size * pp_size:
            raise ValueError(f"world_size {world_size} != tp_size {tp_size} * pp_size {pp_size}")
        dev = torch.device(device)
        if dev.type == "cuda":
            if not torch.cuda.is_available():
                raise RuntimeError("CUDA device requested but unavailable")
            local_rank = int(os.environ.get("LOCAL_RANK", "0"))
            if dev.index is not None and world_size > 1 and dev.index != local_rank:
                raise ValueError(f"device index {dev.index} != LOCAL_RANK {local_rank}")
            dev = torch.device("cuda", dev.index if dev.index is not None else local_rank)
            torch.cuda.set_device(dev)
        if world_size > 1 and owns:
            if not dist.is_available():
                raise RuntimeError("torch.distributed is not available")
            backend = "nccl" if dev.type == "cuda" else "gloo"
            if dev.type == "cpu" and not dist.is_gloo_available():
                raise RuntimeError("gloo backend unavailable")
            if dev.type == "cuda" and not dist.is_nccl_available():
                raise RuntimeError("nccl backend unavailable")
            kw = {"device_id": dev} if dev.type == "cuda" else {}
            dist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_s), **kw)
        tp_group = None
        if world_size > 1:
            for stage in range(pp_size):
                ranks = list(range(stage * tp_size, (stage + 1) * tp_size))
                g = dist.new_group(ranks, timeout=timedelta(seconds=timeout_s))
                if rank in ranks:
                    tp_group = g
        return cls(tp_size=tp_size, pp_size=pp_size, rank=rank, world_size=world_size,
                   tp_rank=rank % tp_size, pp_rank=rank // tp_size, device=dev, tp_group=tp_group,
                   owns_process_group=owns)

    def all_reduce(self, tensor: torch.Tensor) -> torch.Tensor:
        if self.tp_size > 1 and self.tp_group is not None:
            with record_function("nebula::tp_all_reduce"):
                dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=self.tp_group)
        return tensor

    def close(self) -> None:
        if self.owns_process_group and dist.is_available() and dist.is_initialized():
            try:
                dist.destroy_process_group()
            finally:
                self.owns_process_group = False
