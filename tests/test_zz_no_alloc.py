"""fml_gemm_noalloc: the GEMM entry point for callers that cannot allocate
device memory (a host runtime that owns all GPU memory through its own
allocator, or a latency-critical caller that must not go through
cudaMalloc/cudaFree).  Instead of a caller workspace it stages operand packing
in a library-owned device array of GEMM_NOALLOC_SCRATCH_BYTES.

The test calls it through the C ABI and compares it with fml_gemm (the
workspace-taking entry point) on two calls in a row, in the same tolerances as
the other GEMM tests: fp32 rtol 1e-5 / atol 1e-4, bf16 rtol 2e-2 / atol 2e-2.
Both problems need scratch (the fp32 3xTF32 split; a bf16 operand whose rows
TMA cannot address).  This file is collected last so that a run stopping at
the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

from forgeml_b200 import _native

pytestmark = pytest.mark.gpu


def _run(name, a, b, out, bias=None, residual=None, act=_native.ACT_NONE):
    m, k = a.shape
    n = b.shape[1]
    code = _native.dtype_code(a.dtype)
    args = [a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
            bias.data_ptr() if bias is not None else None, bias.stride(0) if bias is not None else 0,
            residual.data_ptr() if residual is not None else None, residual.stride(0) if residual is not None else 0,
            out.data_ptr(), out.stride(0), m, n, k, code, act, None]
    ws = None
    if name == "fml_gemm":
        need = _workspace_bytes(a, b)
        assert need > 0, "the comparison must exercise the scratch path"
        ws = torch.empty(need + 256, dtype=torch.uint8, device=a.device)
        args += [(ws.data_ptr() + 255) // 256 * 256, need]
    _native.call(name, *args, _native.stream_ptr(a.device))
    return ws


def _workspace_bytes(a, b) -> int:
    m, k = a.shape
    return int(_native.load().fml_gemm_workspace_size(m, b.shape[1], k, _native.dtype_code(a.dtype), a.stride(0),
                                                      a.stride(1), b.stride(0), b.stride(1), a.data_ptr(),
                                                      b.data_ptr(), None))


@pytest.mark.parametrize("dtype,shape,tol,epilogue", [
    (torch.float32, (96, 80, 200), (1e-5, 1e-4), False),
    (torch.bfloat16, (40, 72, 9), (2e-2, 2e-2), False),  # K=9: 18-byte rows, packed in scratch
    (torch.float32, (64, 48, 136), (1e-5, 1e-4), True),  # bias + exact GELU + residual
    (torch.bfloat16, (33, 40, 7), (2e-2, 2e-2), True),
])
def test_noalloc_matches_workspace_gemm_two_calls(cuda, dtype, shape, tol, epilogue):
    m, n, k = shape
    for call in range(2):
        g = torch.Generator().manual_seed(100 * call + m)
        a = torch.randn(m, k, generator=g).to(dtype).to(cuda)
        b = torch.randn(k, n, generator=g).to(dtype).to(cuda)
        extra = {}
        if epilogue:
            extra = {"bias": torch.randn(n, generator=g).to(dtype).to(cuda),
                     "residual": torch.randn(m, n, generator=g).to(dtype).to(cuda), "act": _native.ACT_GELU_ERF}
        want = torch.empty(m, n, dtype=dtype, device=cuda)
        got = torch.full((m, n), float("nan"), dtype=dtype, device=cuda)
        ws = _run("fml_gemm", a, b, want, **extra)
        _run("fml_gemm_noalloc", a, b, got, **extra)
        torch.cuda.synchronize()
        del ws
        torch.testing.assert_close(got.float(), want.float(), rtol=tol[0], atol=tol[1])


def test_noalloc_just_under_the_scratch_limit_matches_the_oracle(cuda):
    """An fp32 problem whose packing needs just under the scratch size runs
    (the library's size check and fml_gemm's workspace rule agree) and is
    right, checked against the fp64-accumulated oracle contract."""
    from oracle.gemm import matmul_epilogue

    n = k = 1024
    limit = _native.GEMM_NOALLOC_SCRATCH_BYTES
    probe_b = torch.empty(k, n, device=cuda)
    lo, hi = 1, 4096
    while lo < hi:  # the largest m whose packing fits
        mid = (lo + hi + 1) // 2
        if _workspace_bytes(torch.empty(mid, k, device=cuda), probe_b) <= limit:
            lo = mid
        else:
            hi = mid - 1
    m = lo
    g = torch.Generator().manual_seed(11)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(k, n, generator=g)
    need = _workspace_bytes(a.to(cuda), b.to(cuda))
    assert limit - (1 << 20) < need <= limit
    got = torch.empty(m, n, device=cuda)
    _run("fml_gemm_noalloc", a.to(cuda), b.to(cuda), got)
    torch.testing.assert_close(got.cpu(), matmul_epilogue(a, b), rtol=1e-5, atol=1e-4)
    big = torch.empty(m + 64, k, device=cuda)
    with pytest.raises(_native.NativeError, match="static scratch"):
        _run("fml_gemm_noalloc", big, b.to(cuda), torch.empty(m + 64, n, device=cuda))


def test_noalloc_rejects_problems_beyond_scratch(cuda):
    m = n = k = 1024  # fp32 3xTF32 packing needs ~25 MB > 16 MiB
    a = torch.zeros(m, k, device=cuda)
    b = torch.zeros(k, n, device=cuda)
    out = torch.zeros(m, n, device=cuda)
    with pytest.raises(_native.NativeError, match="static scratch"):
        _run("fml_gemm_noalloc", a, b, out)
    assert _native.GEMM_NOALLOC_SCRATCH_BYTES == 16 * 1024 * 1024
    assert ctypes.sizeof(ctypes.c_void_p) == 8
