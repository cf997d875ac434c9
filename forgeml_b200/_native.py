"""ctypes binding of ``libforgeml_b200.so`` (the C ABI in include/forgeml_b200.h).

The product path has no fallback: if the library is missing or a call returns
a nonzero status, the caller gets an exception carrying ``fml_last_error()``.
Tensors cross the boundary as raw device pointers, element strides and the
current CUDA stream handle.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libforgeml_b200.so"

FML_F32, FML_F16, FML_BF16 = 0, 1, 2
ACT_NONE, ACT_GELU_ERF, ACT_GELU_TANH = 0, 1, 2
STATUS_NAMES = {
    1: "invalid argument",
    2: "unsupported layout",
    3: "CUDA error",
    4: "workspace too small",
    5: "device-side error",
}

# Capacity of the library-owned scratch used by fml_gemm_noalloc (bytes).
GEMM_NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024

_DTYPE_CODE = {torch.float32: FML_F32, torch.float16: FML_F16, torch.bfloat16: FML_BF16}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_load_error: str | None = None


class NativeError(RuntimeError):
    """A forgeml_b200 C-ABI call failed (status code and library message)."""

    def __init__(self, name: str, code: int, message: str):
        self.code = code
        super().__init__(f"{name} failed ({STATUS_NAMES.get(code, code)}): {message}")


class fml_tile_cfg(ctypes.Structure):
    _fields_ = [
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("block_k", ctypes.c_int32),
        ("num_warps", ctypes.c_int32),
        ("num_stages", ctypes.c_int32),
    ]


class neb_fusion(ctypes.Structure):
    """Fusions of neb_linear_fused (include/forgeml_b200.h)."""

    _fields_ = [
        ("ln_gamma", ctypes.c_void_p),
        ("ln_beta", ctypes.c_void_p),
        ("ln_eps", ctypes.c_float),
        ("ln_wsum", ctypes.c_void_p),
        ("ln_wbias", ctypes.c_void_p),
        ("k_pool", ctypes.c_void_p),
        ("v_pool", ctypes.c_void_p),
        ("slot_of", ctypes.c_void_p),
        ("start_pos", ctypes.c_void_p),
        ("q_cols", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("max_seq", ctypes.c_int32),
        ("tq", ctypes.c_int32),
        ("ar_ctx", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_S4 = ctypes.POINTER(ctypes.c_int64)

_SIGNATURES = {
    "fml_gemm_workspace_size": (
        ctypes.c_size_t, [_I64, _I64, _I64, _I, _I64, _I64, _I64, _I64, _P, _P, ctypes.POINTER(fml_tile_cfg)]
    ),
    "fml_gemm": (
        _I,
        [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I, _I,
         ctypes.POINTER(fml_tile_cfg), _P, ctypes.c_size_t, _P],
    ),
    "fml_gemm_packed_b_bytes": (ctypes.c_size_t, [_I64, _I64, _I]),
    "fml_gemm_pack_b": (_I, [_P, _I64, _I64, _I64, _I64, _I, _P, ctypes.c_size_t, _P]),
    "fml_gemm_packed_b_workspace_size": (
        ctypes.c_size_t, [_I64, _I64, _I64, _I, _I64, _I64, _P, ctypes.POINTER(fml_tile_cfg)]
    ),
    "fml_gemm_packed_b": (
        _I,
        [_P, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I, _I,
         ctypes.POINTER(fml_tile_cfg), _P, ctypes.c_size_t, _P],
    ),
    "fml_gemm_noalloc": (
        _I,
        [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I, _I,
         ctypes.POINTER(fml_tile_cfg), _P],
    ),
    "fml_packed_weight_bytes": (ctypes.c_size_t, [_I64, _I64, _I]),
    "fml_pack_weight": (_I, [_P, _I64, _I64, _I64, _I, _P, _P]),
    "fml_linear_packed": (
        _I, [_P, _I64, _P, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I, _I, ctypes.POINTER(fml_tile_cfg), _P]
    ),
    "fml_layernorm": (_I, [_P, _I64, _P, _P, _F, _P, _I64, _I64, _I64, _I, _P]),
    "fml_sdpa": (
        _I,
        [_P, _S4, _P, _S4, _P, _S4, _P, _S4, _I, _I, _F, _P, _S4, _I64, _I64, _I64, _I64, _I64, _I, _P],
    ),
    "neb_attention": (_I, [_P, _S4, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _F, _I, _P]),
    "neb_kv_append": (_I, [_P, _S4, _P, _S4, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    "neb_embed": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    "neb_argmax": (_I, [_P, _I64, _I64, _I64, _P, _I, _P]),
    "neb_add": (_I, [_P, _P, _P, _I64, _I, _P]),
    "neb_ar_handle_bytes": (_I64, []),
    "neb_ar_create": (_I, [_I64, _I, _I, ctypes.c_double, ctypes.POINTER(ctypes.c_void_p), _P]),
    "neb_ar_open": (_I, [_P, _P]),
    "neb_ar_set_peers": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "neb_ar_buffer": (_P, [_P]),
    "neb_ar_set_protocol": (_I, [_P, _I]),
    "neb_ar_all_reduce": (_I, [_P, _P, _P, _P, _I64, _I, _P]),
    "neb_ar_destroy": (_I, [_P]),
    "neb_linear_fused": (
        _I, [_P, _I64, _P, _I64, _I64, _P, _I64, _P, _I64, _I64, _I, _I, ctypes.POINTER(neb_fusion), _P]
    ),
    "neb_linear_fused_ok": (_I, [_I64, _I64, _I64, _I]),
    "fml_last_error": (ctypes.c_char_p, []),
    "fml_device_status": (_I, []),
    "fml_device_status_async": (_I, [_P, _P]),
    "fml_launch_count": (_I64, []),
    "fml_version": (ctypes.c_char_p, []),
}

EXPORTED = tuple(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load the shared library once; raise with the reason if it is unusable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("FORGEML_B200_LIB", LIB_PATH))
        if not path.exists():
            _load_error = (
                f"{path} is missing; build it with `python -m forgeml_b200.build` "
                "(there is no non-native fallback)"
            )
            raise RuntimeError(_load_error)
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def is_loadable() -> bool:
    try:
        load()
        return True
    except (OSError, RuntimeError):
        return False


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"dtype {dtype} is not supported by the native kernels") from None


def strides4(t_or_strides) -> ctypes.Array:
    s = t_or_strides.stride() if isinstance(t_or_strides, torch.Tensor) else tuple(t_or_strides)
    if len(s) != 4:
        raise ValueError("expected 4 strides")
    return (ctypes.c_int64 * 4)(*[int(v) for v in s])


def stream_ptr(device: torch.device | None = None) -> int:
    return int(torch.cuda.current_stream(device).cuda_stream)


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.fml_last_error().decode(errors="replace")
        raise NativeError(name, int(rc), msg)


def device_status() -> int:
    """Read and clear the device error word (synchronises the current device)."""
    return int(load().fml_device_status())


def device_status_async(host_dst: torch.Tensor, stream: int) -> None:
    """Queue a copy of the device error word into ``host_dst`` (a pinned
    int32 host tensor) on ``stream``; read it once the stream has passed."""
    call("fml_device_status_async", host_dst.data_ptr(), stream)


def launch_count() -> int:
    return int(load().fml_launch_count())


def version() -> str:
    return load().fml_version().decode()
