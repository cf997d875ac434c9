"""Fused decode linear (neb_linear_fused) on one GPU, through the C ABI.

* LayerNorm prologue: against the unfused chain fml_layernorm ->
  fml_linear_packed.  The fused statistics are summed in another order, so
  an LN output may land on the neighbouring bf16 value; with an identity
  weight the product returns LN(x) itself, which must match fml_layernorm to
  one bf16 step (and exactly for nearly every element).
* LayerNorm fold (gamma in the packed weight, statistics by the GEMM,
  rstd * (acc - mean * sum W') + W beta in the epilogue): against the unfused
  chain within bf16 tolerance, and no further from an fp32 LN(x) W^T.
* KV epilogue: bit-exact against the same kernel writing every feature to
  `out` (the pools receive exactly the K and V columns; other pool rows stay
  untouched).
* All-reduce epilogue with a one-rank group: bit-exact against the residual
  epilogue of the same kernel, eagerly and replayed from a CUDA graph.
* The all-reduce peer wait is bounded: a two-rank group in which only one
  rank launches gives up after the context's timeout with status bit 32.
"""

import ctypes

import pytest
import torch

from forgeml_b200 import _native
from forgeml_b200.linear import PackedLinear

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _ln_ref(x, g, b):
    out = torch.empty_like(x)
    _native.call("fml_layernorm", x.data_ptr(), x.stride(0), g.data_ptr(), b.data_ptr(), 1e-5, out.data_ptr(),
                 out.stride(0), x.shape[0], x.shape[1], _native.dtype_code(x.dtype),
                 torch.cuda.current_stream().cuda_stream)
    return out


def _data(n, k, m, dev, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).to(BF).to(dev)
    x = (torch.randn(m, k, generator=g) * 1.5 + 0.3).to(BF).to(dev)
    gam = (1 + 0.1 * torch.randn(k, generator=g)).to(BF).to(dev)
    bet = (0.1 * torch.randn(k, generator=g)).to(BF).to(dev)
    return w, x, gam, bet


@pytest.mark.parametrize("n,k,m", [(6144, 2048, 32), (768, 2048, 32), (8192, 2048, 7), (256, 128, 18),
                                   (2048, 4096, 1), (1536, 2048, 16)])
def test_ln_prologue_matches_unfused(cuda, n, k, m):
    w, x, gam, bet = _data(n, k, m, cuda, n + k + m)
    lin = PackedLinear(w)
    assert lin.fused_ok(m)
    act = _native.ACT_GELU_TANH if n == 8192 else 0
    got = lin.fused(x, torch.empty(m, n, dtype=BF, device=cuda), act=act, ln=(gam, bet, 1e-5))
    want = lin(_ln_ref(x, gam, bet), torch.empty(m, n, dtype=BF, device=cuda), act=act)
    assert _native.device_status() == 0
    scale = float(want.float().abs().max())
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2 * scale)
    assert (got == want).float().mean() > 0.95


@pytest.mark.parametrize("k,m", [(2048, 32), (4096, 5), (512, 16)])
def test_ln_prologue_identity_weight_is_layernorm(cuda, k, m):
    _, x, gam, bet = _data(8, k, m, cuda, 7 * k + m)
    lin = PackedLinear(torch.eye(k, dtype=BF, device=cuda))
    got = lin.fused(x, torch.empty(m, k, dtype=BF, device=cuda), ln=(gam, bet, 1e-5))
    want = _ln_ref(x, gam, bet)
    assert _native.device_status() == 0
    # one bf16 step at most, and almost always exact
    step = torch.maximum(want.float().abs(), torch.full_like(want.float(), 1e-3)) * 2.0 ** -7
    assert torch.all((got.float() - want.float()).abs() <= step * 1.01)
    assert (got == want).float().mean() > 0.98


@pytest.mark.parametrize("n,k,m,identity", [(6144, 2048, 32, False), (8192, 2048, 7, False), (768, 2048, 32, True),
                                            (2048, 4096, 1, False), (256, 128, 18, True)])
def test_ln_fold_matches_unfused(cuda, n, k, m, identity):
    """LayerNorm folded into the product: LN(x) W^T = rstd (x W'^T - mean sum W') + W beta.
    Against the unfused chain within bf16 tolerance, and no further from an
    fp32 evaluation of LN(x) W^T than the unfused chain (which rounds LN(x))."""
    from forgeml_b200.linear import ln_fold_vectors

    w, x, gam, bet = _data(n, k, m, cuda, 3 * n + k + m)
    if identity:
        gam, bet = torch.ones_like(gam), torch.zeros_like(bet)
    wp, wsum, wbias = ln_fold_vectors(w, gam, bet)
    assert (wp is w) == identity and (wbias is None) == identity
    act = _native.ACT_GELU_TANH if n == 8192 else 0
    lin = PackedLinear(w)
    lin_f = lin if wp is w else PackedLinear(wp)
    got = lin_f.fused(x, torch.empty(m, n, dtype=BF, device=cuda), act=act, ln_fold=(wsum, wbias, 1e-5))
    want = lin(_ln_ref(x, gam, bet), torch.empty(m, n, dtype=BF, device=cuda), act=act)
    assert _native.device_status() == 0
    scale = float(want.float().abs().max())
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2 * scale)
    ln32 = torch.nn.functional.layer_norm(x.float(), (k,), gam.float(), bet.float(), 1e-5)
    ref = ln32 @ w.float().t()
    if act:
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    err_f = (got.float() - ref).abs().mean()
    err_u = (want.float() - ref).abs().mean()
    assert err_f <= 1.5 * err_u + 1e-6 * scale


@pytest.mark.parametrize("b,t,heads", [(32, 1, 16), (4, 3, 2), (1, 1, 8)])
def test_kv_epilogue_writes_the_pools(cuda, b, t, heads):
    hd, max_seq, slots_n = 128, 64, 40
    q_cols = heads * hd
    n, k, m = 3 * q_cols, 2048, b * t
    w, x, gam, bet = _data(n, k, m, cuda, 11 * b + t)
    lin = PackedLinear(w)
    full = lin.fused(x, torch.empty(m, n, dtype=BF, device=cuda), ln=(gam, bet, 1e-5))
    kp = torch.randn(slots_n, heads, max_seq, hd, device=cuda).to(BF)
    vp = torch.randn(slots_n, heads, max_seq, hd, device=cuda).to(BF)
    kp0, vp0 = kp.clone(), vp.clone()
    slots = torch.randperm(slots_n)[:b].to(torch.int32).to(cuda)
    starts = torch.randint(0, max_seq - t, (b,), dtype=torch.int32).to(cuda)
    q = lin.fused(x, torch.empty(m, q_cols, dtype=BF, device=cuda), ln=(gam, bet, 1e-5),
                  kv=(kp, vp, slots, starts, q_cols, t))
    assert _native.device_status() == 0
    assert torch.equal(q, full[:, :q_cols])
    want_k, want_v = kp0.clone(), vp0.clone()
    fk = full[:, q_cols:2 * q_cols].view(b, t, heads, hd)
    fv = full[:, 2 * q_cols:].view(b, t, heads, hd)
    for i in range(b):
        s, p0 = int(slots[i]), int(starts[i])
        want_k[s, :, p0:p0 + t] = fk[i].transpose(0, 1)
        want_v[s, :, p0:p0 + t] = fv[i].transpose(0, 1)
    assert torch.equal(kp, want_k)
    assert torch.equal(vp, want_v)


def test_kv_epilogue_position_out_of_range_is_reported(cuda):
    heads, hd, max_seq = 2, 64, 8
    q_cols = heads * hd
    w, x, gam, bet = _data(3 * q_cols, 256, 2, cuda, 3)
    lin = PackedLinear(w)
    kp = torch.zeros(2, heads, max_seq, hd, dtype=BF, device=cuda)
    vp = torch.zeros_like(kp)
    slots = torch.tensor([0, 1], dtype=torch.int32, device=cuda)
    starts = torch.tensor([0, max_seq], dtype=torch.int32, device=cuda)  # request 1 is past the end
    lin.fused(x, torch.empty(2, q_cols, dtype=BF, device=cuda), kv=(kp, vp, slots, starts, q_cols, 1))
    assert _native.device_status() & 4
    assert torch.all(kp[1] == 0) and torch.all(vp[1] == 0)


def _ar_context(world, rank, max_bytes, timeout_ms=5000.0):
    lib = _native.load()
    c = ctypes.c_void_p()
    h = (ctypes.c_uint8 * int(lib.neb_ar_handle_bytes()))()
    _native.call("neb_ar_create", max_bytes, world, rank, timeout_ms, ctypes.byref(c), h)
    return c


@pytest.mark.parametrize("n,k,m", [(2048, 2048, 32), (2048, 8192, 32), (4096, 1024, 9), (256, 128, 18)])
def test_all_reduce_epilogue_single_rank(cuda, n, k, m):
    w, x, _, _ = _data(n, k, m, cuda, n * 3 + m)
    res = torch.randn(m, n, device=cuda).to(BF)
    lin = PackedLinear(w)
    ctx = _ar_context(1, 0, n * 64)
    try:
        want = lin.fused(x, torch.empty(m, n, dtype=BF, device=cuda), residual=res)
        for _ in range(3):  # epochs advance
            got = lin.fused(x, torch.empty(m, n, dtype=BF, device=cuda), residual=res, ar_ctx=ctx.value)
            assert torch.equal(got, want)
        out = torch.empty(m, n, dtype=BF, device=cuda)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            lin.fused(x, out, residual=res, ar_ctx=ctx.value)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            lin.fused(x, out, residual=res, ar_ctx=ctx.value)
            lin.fused(x, out, residual=res, ar_ctx=ctx.value)
        for _ in range(3):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want)
        del graph
        assert _native.device_status() == 0
    finally:
        _native.call("neb_ar_destroy", ctx)


def test_all_reduce_epilogue_peer_wait_times_out(cuda):
    lib = _native.load()
    n, k, m = 2048, 1024, 32
    ctxs = [_ar_context(2, r, n * 64, timeout_ms=200.0) for r in range(2)]
    try:
        bases = (ctypes.c_void_p * 2)(lib.neb_ar_buffer(ctxs[0]), lib.neb_ar_buffer(ctxs[1]))
        _native.call("neb_ar_set_peers", ctxs[0], bases)
        assert _native.device_status() == 0
        w, x, _, _ = _data(n, k, m, cuda, 5)
        lin = PackedLinear(w)
        lin.fused(x, torch.empty(m, n, dtype=BF, device=cuda), ar_ctx=ctxs[0].value)  # rank 1 never launches
        assert _native.device_status() & 32
        y = lin.fused(x, torch.empty(m, n, dtype=BF, device=cuda))  # the context is still usable
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
    finally:
        for c in ctxs:
            _native.call("neb_ar_destroy", c)


def test_fused_rejects_what_it_does_not_cover(cuda):
    w, x, gam, bet = _data(256, 128, 33, cuda, 1)
    lin = PackedLinear(w)
    assert not lin.fused_ok(33)
    with pytest.raises(_native.NativeError, match="32 tokens"):
        lin.fused(x, torch.empty(33, 256, dtype=BF, device=cuda))
    w2 = (torch.randn(256, 96, device=cuda) * 0.02).to(BF)
    x2 = torch.randn(4, 96, device=cuda).to(BF)
    with pytest.raises(_native.NativeError, match="multiple of 64"):
        PackedLinear(w2).fused(x2, torch.empty(4, 256, dtype=BF, device=cuda),
                               ln=(torch.ones(96, dtype=BF, device=cuda), torch.zeros(96, dtype=BF, device=cuda), 1e-5))
