"""Kernel front door: validation + launch of the sm_100a kernels.

Drop-in for the reference module src/forgeml/kernels.py.  ``matmul`` keeps the
reference signature, validation order and error substrings
(src/forgeml/kernels.py:52-116) but launches the tcgen05 GEMM of
``libforgeml_b200.so`` (C ABI ``fml_gemm``) instead of the Triton template.
``layer_norm`` and ``sdpa`` are new native front doors for the ops the
reference evaluated through torch (src/forgeml/ops.py:54-70).

Backend naming: the plan label ``"triton"`` and ``compile(...,
backend="triton")`` keep the reference's public names for API compatibility.
No Triton code exists in this package; the label selects the native sm_100a
kernels.  There is no silent fallback: a node planned for the native backend
either runs the native kernel or raises ``GraphError``.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from pathlib import Path

import torch

from forgeml_b200 import _native
from forgeml_b200.forgeml.ir import Graph, GraphError


@dataclass(frozen=True)
class KernelConfig:
    """Tile hints for the native GEMM (fields as in src/forgeml/kernels.py:12-18).

    ``block_n`` is the UMMA N tile (16..256) and ``num_stages`` the shared-memory
    pipeline depth of single-CTA tiles.  ``block_m`` 256 (with ``block_n``
    256) asks for CTA-pair tiles (``cta_group::2``, 256 x 256 per pair, the
    deepest ring that fits); other ``block_m`` values are the 128-row UMMA
    tile.  ``block_k`` (128-byte K slab) and ``num_warps`` (TMA, MMA and
    epilogue warps) are fixed by the kernel design and only validated.
    """

    block_m: int = 128
    block_n: int = 256
    block_k: int = 64
    num_warps: int = 6
    num_stages: int = 4


DEFAULT_CONFIG = KernelConfig()
CANDIDATES = (
    KernelConfig(128, 256, 64, 6, 4),
    KernelConfig(256, 256, 64, 6, 7),
    KernelConfig(128, 128, 64, 6, 6),
    KernelConfig(128, 64, 64, 6, 8),
    KernelConfig(128, 32, 64, 6, 8),
)

_TILES_M = {16, 32, 64, 128, 256}
_TILES_N = {16, 32, 64, 128, 256}
_TILES_K = {16, 32, 64, 128, 256}
_WARPS = {4, 6, 8}
_STAGES = {2, 3, 4, 5, 6, 7, 8}
_DTYPES = {torch.float16, torch.bfloat16, torch.float32}
_GEMM_OPS = ("matmul", "linear", "fused_linear_gelu")
_NATIVE_OPS = _GEMM_OPS + ("layer_norm", "sdpa")


_SM100: dict = {}


def _sm100(device: torch.device | int | None = None) -> bool:
    key = device.index if isinstance(device, torch.device) else device
    hit = _SM100.get(key)
    if hit is None:
        hit = _SM100[key] = torch.cuda.get_device_capability(device) == (10, 0)
    return hit


def available() -> bool:
    """True when a CUDA sm_100 device is present and the native library loads."""
    if not torch.cuda.is_available():
        return False
    try:
        if not _sm100():
            return False
    except (RuntimeError, AssertionError):
        return False
    return _native.is_loadable()


def _check_config(config: KernelConfig) -> None:
    if not isinstance(config, KernelConfig):
        raise GraphError(f"config must be a KernelConfig, got {type(config).__name__}")
    for name, allowed in (("block_m", _TILES_M), ("block_n", _TILES_N), ("block_k", _TILES_K)):
        v = getattr(config, name)
        if not isinstance(v, int) or isinstance(v, bool) or v not in allowed:
            raise GraphError(f"{name} must be one of {sorted(allowed)}, got {v!r}")
    if config.num_warps not in _WARPS:
        raise GraphError(f"num_warps must be one of {sorted(_WARPS)}")
    if config.num_stages not in _STAGES:
        raise GraphError(f"num_stages must be one of {sorted(_STAGES)}")


def _require_native(device: torch.device) -> None:
    if not _sm100(device):
        raise GraphError(
            f"native kernels require an sm_100a (B200) GPU, got capability "
            f"{torch.cuda.get_device_capability(device)}"
        )
    try:
        _native.load()
    except (OSError, RuntimeError) as e:
        raise GraphError(f"native library unavailable: {e}") from e


class _NoContext:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_CONTEXT = _NoContext()


def _workspace(nbytes: int, device: torch.device) -> tuple[torch.Tensor | None, int, int]:
    if nbytes <= 0:
        return None, 0, 0
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    base = ws.data_ptr()
    aligned = (base + 255) // 256 * 256
    return ws, aligned, nbytes


_FML_EWORKSPACE = 4


def _launch_gemm(a, b, bias, out, act: int, config: KernelConfig, residual=None) -> None:
    m, k = a.shape
    n = b.shape[1]
    code = _native.dtype_code(a.dtype)
    lib = _native.load()
    cfg = None
    if config is not DEFAULT_CONFIG and config != DEFAULT_CONFIG:
        cfg = ctypes.byref(
            _native.fml_tile_cfg(config.block_m, config.block_n, config.block_k, config.num_warps, config.num_stages)
        )
    args = (a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
            bias.data_ptr() if bias is not None else None, bias.stride(0) if bias is not None else 0,
            residual.data_ptr() if residual is not None else None, residual.stride(0) if residual is not None else 0,
            out.data_ptr(), out.stride(0), m, n, k, code, act, cfg)
    stream = torch.cuda.current_stream(a.device).cuda_stream
    # 16-bit operands TMA can address need no workspace: try that first (one
    # native call); fp32 (3xTF32 split) and unaddressable layouts ask for it.
    if a.dtype != torch.float32:
        rc = lib.fml_gemm(*args, None, 0, stream)
        if rc == 0:
            return
        if rc != _FML_EWORKSPACE:
            raise _native.NativeError("fml_gemm", int(rc), lib.fml_last_error().decode(errors="replace"))
    ws_bytes = lib.fml_gemm_workspace_size(
        m, n, k, code, a.stride(0), a.stride(1), b.stride(0), b.stride(1), a.data_ptr(), b.data_ptr(), cfg
    )
    ws, ws_ptr, ws_n = _workspace(int(ws_bytes), a.device)
    _native.call("fml_gemm", *args, ws_ptr or None, ws_n, stream)
    del ws  # the caching allocator keeps it alive until the stream is done with it


def _version_of(t: torch.Tensor) -> int | None:
    """The tensor's in-place version counter; None for inference tensors
    (made under torch.inference_mode), which carry none: a compiled graph's
    weights made that way are taken as constant."""
    try:
        return t._version
    except RuntimeError:
        return None


def _aligned(buf: torch.Tensor, align: int) -> int:
    return (buf.data_ptr() + align - 1) // align * align


class PreparedGemm:
    """A GEMM launch whose validation was done once (by the compiler, from the
    graph's specs): each call passes the current pointers straight to
    ``fml_gemm``.  Keeps its own grow-only workspace (fp32 operand split,
    operands TMA cannot address), so a call allocates nothing once warm."""

    def __init__(self, dtype: torch.dtype, activation: str = "none", approximate: str = "none",
                 config: KernelConfig = DEFAULT_CONFIG):
        _check_config(config)
        self.config = config
        self.code = _native.dtype_code(dtype)
        self.act = _native.ACT_NONE
        if activation == "gelu":
            self.act = _native.ACT_GELU_TANH if approximate == "tanh" else _native.ACT_GELU_ERF
        self.cfg = None
        if config != DEFAULT_CONFIG:
            self._cfg_obj = _native.fml_tile_cfg(config.block_m, config.block_n, config.block_k, config.num_warps,
                                                 config.num_stages)
            self.cfg = ctypes.byref(self._cfg_obj)
        self.lib = _native.load()
        self.ws: torch.Tensor | None = None
        self._b_const: torch.Tensor | None = None  # fp32 constant B and its 3xTF32 image
        self._b_image: torch.Tensor | None = None
        self._b_version = -1

    def pack_constant_b(self, b: torch.Tensor) -> None:
        """Split a constant fp32 B [K, N] into its 3xTF32 image once
        (fml_gemm_pack_b); calls with this tensor then split only A.  Other
        dtypes read B directly and keep no image."""
        if self.code != _native.dtype_code(torch.float32) or b.dtype != torch.float32 or not b.is_cuda:
            return
        k, n = b.shape
        nbytes = int(self.lib.fml_gemm_packed_b_bytes(n, k, self.code))
        img = torch.empty(nbytes + 256, dtype=torch.uint8, device=b.device)
        with torch.cuda.device(b.device):
            _native.call("fml_gemm_pack_b", b.data_ptr(), b.stride(0), b.stride(1), k, n, self.code,
                         _aligned(img, 256), nbytes, torch.cuda.current_stream(b.device).cuda_stream)
        self._b_const, self._b_image, self._b_version = b, img, _version_of(b)

    def _packed_call(self, a, b, bias, out, residual) -> bool:
        """Run on B's image when b is the packed constant (re-split first if
        it was written in place since); False when b is another tensor."""
        if b is not self._b_const:
            return False
        if _version_of(b) != self._b_version:
            self.pack_constant_b(b)
        m, k = a.shape
        n = b.shape[1]
        lib = self.lib
        need = int(lib.fml_gemm_packed_b_workspace_size(m, n, k, self.code, a.stride(0), a.stride(1),
                                                        a.data_ptr(), self.cfg))
        ws_ptr = None
        if need > 0:
            if self.ws is None or self.ws.numel() < need + 256:
                self.ws = torch.empty(need + 256, dtype=torch.uint8, device=a.device)
            ws_ptr = _aligned(self.ws, 256)
        rc = lib.fml_gemm_packed_b(a.data_ptr(), a.stride(0), a.stride(1), _aligned(self._b_image, 256),
                                   bias.data_ptr() if bias is not None else None,
                                   bias.stride(0) if bias is not None else 0,
                                   residual.data_ptr() if residual is not None else None,
                                   residual.stride(0) if residual is not None else 0,
                                   out.data_ptr(), out.stride(0), m, n, k, self.code, self.act, self.cfg,
                                   ws_ptr, need, torch.cuda.current_stream(a.device).cuda_stream)
        if rc != 0:
            raise GraphError(f"fml_gemm_packed_b failed ({rc}): {lib.fml_last_error().decode(errors='replace')}")
        return True

    def __call__(self, a, b, bias, out, residual=None):
        if not (a.is_cuda and b.is_cuda and out.is_cuda):
            raise GraphError("native GEMM operands must be CUDA tensors")
        if self._b_const is not None and self._packed_call(a, b, bias, out, residual):
            return out
        m, k = a.shape
        n = b.shape[1]
        lib = self.lib
        need = int(lib.fml_gemm_workspace_size(m, n, k, self.code, a.stride(0), a.stride(1), b.stride(0),
                                               b.stride(1), a.data_ptr(), b.data_ptr(), self.cfg))
        ws_ptr = None
        if need > 0:
            if self.ws is None or self.ws.numel() < need + 256:
                self.ws = torch.empty(need + 256, dtype=torch.uint8, device=a.device)
            ws_ptr = _aligned(self.ws, 256)
        rc = lib.fml_gemm(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                          bias.data_ptr() if bias is not None else None, bias.stride(0) if bias is not None else 0,
                          residual.data_ptr() if residual is not None else None,
                          residual.stride(0) if residual is not None else 0,
                          out.data_ptr(), out.stride(0), m, n, k, self.code, self.act, self.cfg,
                          ws_ptr, need, torch.cuda.current_stream(a.device).cuda_stream)
        if rc != 0:
            raise GraphError(f"fml_gemm failed ({rc}): {lib.fml_last_error().decode(errors='replace')}")
        return out


def matmul(
    a: torch.Tensor,
    b: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    activation: str = "none",
    approximate: str = "none",
    config: KernelConfig = DEFAULT_CONFIG,
    out: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    """``act(round(round(a @ b) + bias))`` on the tcgen05 GEMM.

    Validation mirrors src/forgeml/kernels.py:62-112.  ``residual`` (an
    extension used by Nebula) adds a [M, N] tensor after the activation with
    one more rounding to the output dtype.
    """
    if not torch.cuda.is_available():
        raise GraphError("native matmul requires CUDA")
    if not isinstance(a, torch.Tensor) or not isinstance(b, torch.Tensor):
        raise GraphError("matmul inputs must be tensors")
    if not a.is_cuda or not b.is_cuda or a.device != b.device:
        raise GraphError("matmul inputs must be CUDA tensors on the same device")
    if a.dtype not in _DTYPES or a.dtype != b.dtype:
        raise GraphError(f"matmul dtype {a.dtype} not supported or mismatched")
    if a.dim() != 2 or b.dim() != 2:
        raise GraphError("matmul requires rank-2 inputs")
    m, k = a.shape
    k2, n = b.shape
    if k != k2 or m <= 0 or n <= 0 or k <= 0:
        raise GraphError(f"matmul incompatible shapes {a.shape} x {b.shape}")
    if activation not in ("none", "gelu"):
        raise GraphError(f"activation must be 'none' or 'gelu', got {activation!r}")
    if approximate not in ("none", "tanh"):
        raise GraphError(f"approximate must be 'none' or 'tanh', got {approximate!r}")
    if activation == "none" and approximate != "none":
        raise GraphError("approximate only applies when activation='gelu'")
    if bias is not None and (
        not isinstance(bias, torch.Tensor)
        or not bias.is_cuda
        or bias.device != a.device
        or bias.dtype != a.dtype
        or bias.dim() != 1
        or bias.shape[0] != n
    ):
        raise GraphError("bias must be a 1-D CUDA tensor of output width matching dtype/device")
    if residual is not None and (
        not isinstance(residual, torch.Tensor)
        or residual.device != a.device
        or residual.dtype != a.dtype
        or tuple(residual.shape) != (m, n)
        or residual.stride(1) != 1
    ):
        raise GraphError("residual must be a row-major (M, N) tensor matching dtype/device")
    if config is not DEFAULT_CONFIG:
        _check_config(config)
    _require_native(a.device)
    if out is None:
        out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    else:
        if (
            not isinstance(out, torch.Tensor)
            or tuple(out.shape) != (m, n)
            or out.dtype != a.dtype
            or out.device != a.device
            or not out.is_contiguous()
        ):
            raise GraphError("out must be a contiguous tensor of shape (M, N) matching dtype/device")
        out_ptr = out.untyped_storage().data_ptr()
        for src in (a, b, bias, residual):
            if src is not None and src.untyped_storage().data_ptr() == out_ptr:
                raise GraphError("out must not share storage with inputs")
    act = _native.ACT_NONE
    if activation == "gelu":
        act = _native.ACT_GELU_TANH if approximate == "tanh" else _native.ACT_GELU_ERF
    ctx = torch.cuda.device(a.device) if torch.cuda.current_device() != a.device.index else _NO_CONTEXT
    with ctx:
        try:
            _launch_gemm(a, b, bias, out, act, config, residual)
        except _native.NativeError as e:
            raise GraphError(str(e)) from e
    return out


def layer_norm(
    x: torch.Tensor,
    normalized_shape: int | tuple[int, ...],
    weight: torch.Tensor | None,
    bias: torch.Tensor | None,
    eps: float,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Native LayerNorm over the trailing ``normalized_shape`` dims."""
    norm = (normalized_shape,) if isinstance(normalized_shape, int) else tuple(normalized_shape)
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise GraphError("native layer_norm requires a CUDA tensor")
    if x.dtype not in _DTYPES:
        raise GraphError(f"layer_norm dtype {x.dtype} not supported")
    if x.dim() < len(norm) or tuple(x.shape[-len(norm):]) != norm:
        raise GraphError(f"layer_norm shape {tuple(x.shape)} does not end with {norm}")
    if (weight is None) != (bias is None):
        raise GraphError("layer_norm needs weight and bias together")
    cols = math.prod(norm)
    rows = x.numel() // cols
    if weight is not None:
        for t in (weight, bias):
            if t.device != x.device or t.dtype != x.dtype or tuple(t.shape) != norm or not t.is_contiguous():
                raise GraphError("layer_norm weight/bias must be contiguous and match x")
    _require_native(x.device)
    xv = x.reshape(rows, cols) if x.is_contiguous() else None
    if xv is None:
        raise GraphError("native layer_norm requires a contiguous input")
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    elif tuple(out.shape) != tuple(x.shape) or out.dtype != x.dtype or not out.is_contiguous():
        raise GraphError("layer_norm out must be contiguous and match x")
    with torch.cuda.device(x.device):
        try:
            _native.call(
                "fml_layernorm", xv.data_ptr(), cols,
                weight.data_ptr() if weight is not None else None,
                bias.data_ptr() if bias is not None else None,
                float(eps), out.data_ptr(), cols, rows, cols,
                _native.dtype_code(x.dtype), _native.stream_ptr(x.device),
            )
        except _native.NativeError as e:
            raise GraphError(str(e)) from e
    return out


def sdpa(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    attn_mask: torch.Tensor | None = None,
    *,
    is_causal: bool = False,
    scale: float | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Native rank-4 scaled-dot-product attention (strided q/k/v allowed)."""
    for t in (q, k, v):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dim() != 4:
            raise GraphError("native sdpa requires rank-4 CUDA tensors")
        if t.stride(3) != 1:
            raise GraphError("native sdpa requires unit stride in the head dimension")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in _DTYPES:
        raise GraphError("sdpa dtype mismatch or unsupported")
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if tuple(k.shape) != (B, H, Sk, D) or tuple(v.shape) != (B, H, Sk, D):
        raise GraphError("sdpa batch/head/key-value shapes are incompatible")
    if D > 256:
        raise GraphError("native sdpa supports head dim <= 256")
    mask_kind = 0
    mptr = None
    mstr = None
    if attn_mask is not None:
        if is_causal:
            raise GraphError("sdpa attn_mask cannot be combined with is_causal")
        if attn_mask.dtype == torch.bool:
            mask_kind = 1
        elif attn_mask.dtype == q.dtype:
            mask_kind = 2
        else:
            raise GraphError("sdpa attn_mask must be bool or match the query dtype")
        mexp = attn_mask.expand(B, H, Sq, Sk)
        mptr = mexp.data_ptr()
        mstr = _native.strides4(mexp)
    _require_native(q.device)
    if out is None:
        out = torch.empty((B, H, Sq, D), dtype=q.dtype, device=q.device)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    with torch.cuda.device(q.device):
        try:
            _native.call(
                "fml_sdpa", q.data_ptr(), _native.strides4(q), k.data_ptr(), _native.strides4(k),
                v.data_ptr(), _native.strides4(v), mptr, mstr, mask_kind, 1 if is_causal else 0, sc,
                out.data_ptr(), _native.strides4(out), B, H, Sq, Sk, D,
                _native.dtype_code(q.dtype), _native.stream_ptr(q.device),
            )
        except _native.NativeError as e:
            raise GraphError(str(e)) from e
    return out


def _native_ok(node, specs) -> bool:
    if node.spec.dtype not in _DTYPES:
        return False
    if not all(torch.device(specs[i].device).type == "cuda" for i in node.inputs):
        return False
    if node.op == "sdpa":
        return node.spec.shape[-1] <= 256
    if node.op in _GEMM_OPS:  # the tcgen05 GEMM takes rank-2 operands
        return all(len(specs[i].shape) == 2 for i in node.inputs[:2])
    return True


def select_kernels(graph: Graph, backend: str) -> dict[str, str]:
    """Per-node backend plan (src/forgeml/kernels.py:119-155 contract).

    GEMM-family nodes go native as in the reference; LayerNorm and SDPA nodes
    also go native (the reference ran them through torch).
    """
    if backend == "torch":
        return {n.name: "torch" for n in graph.nodes}
    if backend == "auto":
        can = available()
        specs = graph.specs()
        return {
            n.name: "triton" if (can and n.op in _NATIVE_OPS and _native_ok(n, specs)) else "torch"
            for n in graph.nodes
        }
    if backend == "triton":
        if not available():
            raise GraphError("backend 'triton' requires CUDA on an sm_100a GPU and the native library")
        specs = graph.specs()
        if not all(torch.device(s.device).type == "cuda" for s in graph.inputs.values()):
            raise GraphError("backend 'triton' requires CUDA graph inputs")
        return {
            n.name: "triton" if (n.op in _NATIVE_OPS and _native_ok(n, specs)) else "torch"
            for n in graph.nodes
        }
    raise GraphError(f"unsupported backend {backend!r}; expected 'torch', 'triton', or 'auto'")


def kernel_source() -> str:
    """CUDA source of the GEMM kernel family (the reference returned its Triton source)."""
    csrc = Path(__file__).resolve().parent.parent / "csrc"
    return (csrc / "common.cuh").read_text() + "\n" + (csrc / "gemm.cu").read_text()
