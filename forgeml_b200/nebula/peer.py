"""NVLink peer-memory collectives for the tensor-parallel decode step.

``PeerAllReduce`` wraps the native one-shot SUM all-reduce fused with the
residual add (``neb_ar_*`` in include/forgeml_b200.h): each TP rank owns a
symmetric device buffer, the ranks exchange CUDA IPC handles once over the
TP process group, and every call is a single kernel per rank (stream-ordered,
CUDA-graph capturable) that pushes its partial into every peer's buffer over
NVLink and sums the rank slots in rank order, so all ranks hold bit-identical
results.  It replaces ParallelContext.all_reduce + ``x + part``
(src/nebula/parallel.py:112-116, src/nebula/runtime.py:146,154) for messages
up to ``max_bytes``; larger messages (prefill) go through NCCL.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from forgeml_b200 import _native

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


class PeerAllReduce:
    PROTOCOLS = {"auto": 0, "one_shot": 1, "two_shot": 2}

    def __init__(self, context, max_bytes: int = 1 << 20, timeout_ms: float = 5000.0, protocol: str = "auto"):
        if protocol not in self.PROTOCOLS:
            raise ValueError(f"protocol must be one of {sorted(self.PROTOCOLS)}")
        if context.tp_size < 2 or context.device.type != "cuda":
            raise ValueError("PeerAllReduce needs a CUDA tensor-parallel group of 2 or more ranks")
        lib = _native.load()
        hb = int(lib.neb_ar_handle_bytes())
        handle = (ctypes.c_uint8 * hb)()
        ptr = ctypes.c_void_p()
        _native.call("neb_ar_create", int(max_bytes), context.tp_size, context.tp_rank, float(timeout_ms),
                     ctypes.byref(ptr), handle)
        self._ctx = ptr
        self.max_bytes = int(max_bytes)
        _native.call("neb_ar_set_protocol", self._ctx, self.PROTOCOLS[protocol])
        gathered: list = [None] * context.tp_size
        dist.all_gather_object(gathered, bytes(handle), group=context.tp_group)
        self._blob = ctypes.create_string_buffer(b"".join(gathered), hb * context.tp_size)
        try:
            _native.call("neb_ar_open", self._ctx, ctypes.cast(self._blob, ctypes.c_void_p))
        except Exception:
            self.close()
            raise

    @property
    def handle(self) -> int | None:
        """The native context pointer (for the fused GEMM all-reduce epilogue)."""
        return None if self._ctx is None else self._ctx.value

    def fits(self, t: torch.Tensor) -> bool:
        nbytes = t.numel() * t.element_size()
        return (self._ctx is not None and t.is_cuda and t.is_contiguous() and t.dtype in _DTYPES
                and 0 < nbytes <= self.max_bytes and nbytes % 16 == 0 and t.data_ptr() % 16 == 0)

    def __call__(self, part: torch.Tensor, residual: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
        """out = round(round(sum over ranks of part) + residual)."""
        _native.call("neb_ar_all_reduce", self._ctx, part.data_ptr(),
                     residual.data_ptr() if residual is not None else None, out.data_ptr(), part.numel(),
                     _native.dtype_code(part.dtype), torch.cuda.current_stream(part.device).cuda_stream)
        return out

    def close(self) -> None:
        if self._ctx is not None:
            _native.call("neb_ar_destroy", self._ctx)
            self._ctx = None

