"""Peer all-reduce on one GPU: the bounded peer wait.

Two contexts of a two-rank group live in this process; only rank 0
launches, so its wait for rank 1's flag can never end.  The kernel must give
up after the context's timeout, raise the all-reduce bit (32) in the device
error word, and leave the CUDA context usable.  No GPU fault is involved.
"""

import ctypes

import pytest
import torch

from forgeml_b200 import _native

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_without_hanging(cuda):
    lib = _native.load()
    hb = int(lib.neb_ar_handle_bytes())
    ctxs, handles = [], []
    for rank in range(2):
        c = ctypes.c_void_p()
        h = (ctypes.c_uint8 * hb)()
        _native.call("neb_ar_create", 1 << 16, 2, rank, 200.0, ctypes.byref(c), h)
        ctxs.append(c)
        handles.append(h)
    try:
        bases = (ctypes.c_void_p * 2)(lib.neb_ar_buffer(ctxs[0]), lib.neb_ar_buffer(ctxs[1]))
        _native.call("neb_ar_set_peers", ctxs[0], bases)
        assert _native.device_status() == 0
        part = torch.ones(1024, dtype=torch.bfloat16, device=cuda)
        out = torch.empty_like(part)
        _native.call("neb_ar_all_reduce", ctxs[0], part.data_ptr(), None, out.data_ptr(), 1024,
                     _native.dtype_code(torch.bfloat16), torch.cuda.current_stream().cuda_stream)
        status = _native.device_status()  # synchronizes; returns once the bounded waits gave up
        assert status & 32
        # the context is still usable
        x = torch.arange(8, device=cuda, dtype=torch.float32)
        assert float((x * 2).sum()) == 56.0
        assert _native.device_status() == 0
    finally:
        for c in ctxs:
            _native.call("neb_ar_destroy", c)


def test_peer_validation(cuda):
    lib = _native.load()
    hb = int(lib.neb_ar_handle_bytes())
    c = ctypes.c_void_p()
    h = (ctypes.c_uint8 * hb)()
    with pytest.raises(_native.NativeError):
        _native.call("neb_ar_create", 1 << 16, 9, 0, 100.0, ctypes.byref(c), h)
    with pytest.raises(_native.NativeError):
        _native.call("neb_ar_create", 100, 2, 0, 100.0, ctypes.byref(c), h)
    _native.call("neb_ar_create", 1 << 16, 2, 0, 100.0, ctypes.byref(c), h)
    try:
        part = torch.ones(1024, dtype=torch.bfloat16, device=cuda)
        with pytest.raises(_native.NativeError, match="peers not opened"):
            _native.call("neb_ar_all_reduce", c, part.data_ptr(), None, part.data_ptr(), 1024,
                         _native.dtype_code(torch.bfloat16), 0)
    finally:
        _native.call("neb_ar_destroy", c)
