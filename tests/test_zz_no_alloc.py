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


def _run(name, a, b, out, ws=None):
    m, k = a.shape
    n = b.shape[1]
    code = _native.dtype_code(a.dtype)
    args = [a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1), None, 0, None, 0,
            out.data_ptr(), out.stride(0), m, n, k, code, _native.ACT_NONE, None]
    if name == "fml_gemm":
        lib = _native.load()
        need = lib.fml_gemm_workspace_size(m, n, k, code, a.stride(0), a.stride(1), b.stride(0), b.stride(1),
                                           a.data_ptr(), b.data_ptr(), None)
        assert need > 0, "the comparison must exercise the scratch path"
        ws = torch.empty(need + 256, dtype=torch.uint8, device=a.device)
        args += [(ws.data_ptr() + 255) // 256 * 256, need]
    _native.call(name, *args, _native.stream_ptr(a.device))
    return ws


@pytest.mark.parametrize("dtype,shape,tol", [
    (torch.float32, (96, 80, 200), (1e-5, 1e-4)),
    (torch.bfloat16, (40, 72, 9), (2e-2, 2e-2)),  # K=9: 18-byte rows, packed in scratch
])
def test_noalloc_matches_workspace_gemm_two_calls(cuda, dtype, shape, tol):
    m, n, k = shape
    for call in range(2):
        g = torch.Generator().manual_seed(100 * call + m)
        a = torch.randn(m, k, generator=g).to(dtype).to(cuda)
        b = torch.randn(k, n, generator=g).to(dtype).to(cuda)
        want = torch.empty(m, n, dtype=dtype, device=cuda)
        got = torch.full((m, n), float("nan"), dtype=dtype, device=cuda)
        ws = _run("fml_gemm", a, b, want)
        _run("fml_gemm_noalloc", a, b, got)
        torch.cuda.synchronize()
        del ws
        torch.testing.assert_close(got.float(), want.float(), rtol=tol[0], atol=tol[1])


def test_noalloc_rejects_problems_beyond_scratch(cuda):
    m = n = k = 1024  # fp32 3xTF32 packing needs ~25 MB > 16 MiB
    a = torch.zeros(m, k, device=cuda)
    b = torch.zeros(k, n, device=cuda)
    out = torch.zeros(m, n, device=cuda)
    with pytest.raises(_native.NativeError, match="static scratch"):
        _run("fml_gemm_noalloc", a, b, out)
    assert _native.GEMM_NOALLOC_SCRATCH_BYTES == 16 * 1024 * 1024
    assert ctypes.sizeof(ctypes.c_void_p) == 8
