"""Parity of the non-GEMM kernels on the B200 against the CPU oracle.

LayerNorm (ForgeML c2 and Nebula shapes), ForgeML SDPA (strided views of a
fused QKV slot, causal, bool and additive masks), Nebula attention over the
KV pool (decode and multi-token steps at absolute positions), KV append
(bit-exact), embedding, argmax (bit-exact, ties) and residual add.

Tolerances: fp32 rtol 1e-5 / atol 1e-4 (LN: atol 1e-5); bf16 rtol 2e-2 /
atol 2e-2; fp16 1e-2 / 1e-2.  Index and copy kernels: exact.
"""

import math

import pytest
import torch

from oracle.attention import nebula_attention, sdpa as sdpa_ref
from oracle.layernorm import layer_norm as ln_ref
from forgeml_b200.forgeml import kernels
from forgeml_b200.nebula import ops as nops

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-4), torch.float16: (1e-2, 1e-2), torch.bfloat16: (2e-2, 2e-2)}


def close(got, want, dtype, atol=None):
    rtol, a = TOL[dtype]
    torch.testing.assert_close(got.float().cpu(), want.float().cpu(), rtol=rtol, atol=a if atol is None else atol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(4096, 768), (32, 2048), (7, 100), (3, 4096), (1, 16), (5, 33)])
@pytest.mark.parametrize("affine", [True, False])
def test_layernorm(cuda, dtype, rows, cols, affine):
    g = torch.Generator().manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=g) * 3 + 1).to(dtype)
    w = (torch.randn(cols, generator=g)).to(dtype) if affine else None
    b = (torch.randn(cols, generator=g)).to(dtype) if affine else None
    got = kernels.layer_norm(x.to(cuda), cols, w.to(cuda) if affine else None, b.to(cuda) if affine else None, 1e-5)
    close(got, ln_ref(x, cols, w, b, 1e-5), dtype)


def _qkv_views(b, s, h, d, dtype, device, seed):
    """q/k/v as strided [B,H,S,D] views of one [B*S, 3*H*D] slot (fused QKV)."""
    g = torch.Generator().manual_seed(seed)
    wide = torch.randn(b * s, 3 * h * d, generator=g).to(dtype)
    wd = wide.to(device)
    views = []
    for i in range(3):
        part = wd.narrow(1, i * h * d, h * d).reshape(b, s, h, d).transpose(1, 2)
        views.append(part)
    cpu = [wide.narrow(1, i * h * d, h * d).reshape(b, s, h, d).transpose(1, 2) for i in range(3)]
    return views, cpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,s,h,d", [(2, 128, 12, 64), (1, 77, 3, 32), (2, 40, 2, 128), (1, 16, 4, 4)])
@pytest.mark.parametrize("mode", ["plain", "causal", "bool_mask", "add_mask"])
def test_sdpa(cuda, dtype, b, s, h, d, mode):
    (q, k, v), (qc, kc, vc) = _qkv_views(b, s, h, d, dtype, cuda, seed=b * s + h * d)
    mask = None
    if mode == "bool_mask":
        g = torch.Generator().manual_seed(9)
        mask = torch.rand(b, 1, s, s, generator=g) > 0.3
        mask[..., 0] = True  # no fully-masked rows
    elif mode == "add_mask":
        g = torch.Generator().manual_seed(11)
        mask = torch.randn(s, s, generator=g).to(dtype)
    got = kernels.sdpa(q, k, v, mask.to(cuda) if mask is not None else None, is_causal=(mode == "causal"))
    want = sdpa_ref(qc, kc, vc, mask, is_causal=(mode == "causal"))
    close(got, want, dtype)


@pytest.mark.parametrize("dtype,b,s,h,d,causal", [
    (torch.bfloat16, 2, 512, 12, 64, False),   # config 2 shape (two batch elements)
    (torch.bfloat16, 1, 512, 12, 64, True),
    (torch.float16, 2, 300, 4, 128, True),     # Nebula prefill head size, partial key block
    (torch.bfloat16, 1, 129, 2, 128, False),   # one position past a 128-block
])
def test_sdpa_tensor_core_path(cuda, dtype, b, s, h, d, causal):
    """16-bit attention without an explicit mask runs on the tcgen05 kernel
    (sdpa_tc.cu); checked against the oracle at the dtype's tolerance."""
    (q, k, v), (qc, kc, vc) = _qkv_views(b, s, h, d, dtype, cuda, seed=3 * s + d)
    got = kernels.sdpa(q, k, v, is_causal=causal)
    want = sdpa_ref(qc, kc, vc, is_causal=causal)
    close(got, want, dtype)
    # written through strides into a [B, S, H, D] buffer (the compiled block's layout)
    buf = torch.empty(b, s, h, d, dtype=dtype, device=cuda)
    kernels.sdpa(q, k, v, is_causal=causal, out=buf.transpose(1, 2))
    close(buf.transpose(1, 2), want, dtype)


@pytest.mark.parametrize("dtype,s,causal", [(torch.bfloat16, 1000, False), (torch.float16, 777, True)])
def test_sdpa_tensor_core_sharp_scores(cuda, dtype, s, causal):
    """Large scores (q scaled by 6) over many key blocks: row maxima keep
    moving, so the running output in TMEM is rescaled block after block."""
    (q, k, v), (qc, kc, vc) = _qkv_views(1, s, 3, 64, dtype, cuda, seed=11 + s)
    q, qc = (q * 6).to(dtype), (qc.float() * 6).to(dtype)
    got = kernels.sdpa(q, k, v, is_causal=causal)
    want = sdpa_ref(qc, kc, vc, is_causal=causal)
    close(got, want, dtype)


def test_sdpa_matches_torch_cpu_c2_slice(cuda):
    """c2 shapes (head_dim 64, 12 heads) on one batch element vs torch's own CPU SDPA."""
    (q, k, v), (qc, kc, vc) = _qkv_views(1, 512, 12, 64, torch.float32, cuda, seed=1)
    got = kernels.sdpa(q, k, v)
    want = torch.nn.functional.scaled_dot_product_attention(qc, kc, vc)
    close(got, want, torch.float32)


def _pool(slots, h, max_seq, d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    kp = torch.randn(slots, h, max_seq, d, generator=g).to(dtype)
    vp = torch.randn(slots, h, max_seq, d, generator=g).to(dtype)
    return kp, vp


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("b,t,h,d,max_seq,start", [
    (32, 1, 16, 128, 2048, 600),   # c4 decode step shape
    (4, 1, 8, 128, 4096, 2000),    # c5-like context
    (3, 5, 4, 64, 256, 17),        # multi-token step at an offset
    (2, 3, 4, 4, 16, 0),           # tiny config prefill (head_dim 4)
    (2, 1, 4, 4, 16, 9),
    (1, 1, 2, 80, 300, 299),       # odd head size, last position
])
def test_nebula_attention(cuda, dtype, b, t, h, d, max_seq, start):
    slots = b + 2
    kp, vp = _pool(slots, h, max_seq, d, dtype, seed=b * 7 + t)
    slot_of = torch.tensor([(i * 3 + 1) % slots for i in range(b)], dtype=torch.int32)
    starts = torch.full((b,), start, dtype=torch.int32)
    g = torch.Generator().manual_seed(5)
    # q as a strided [B,T,H,D] view of a wider projection output
    qkv = torch.randn(b, t, 3 * h * d, generator=g).to(dtype)
    q = qkv[..., : h * d].reshape(b, t, h, d)
    got = nops.attention(q.to(cuda) if q.is_contiguous() else qkv.to(cuda)[..., : h * d].reshape(b, t, h, d),
                         kp.to(cuda), vp.to(cuda), slot_of.to(cuda), starts.to(cuda))
    assert got.shape == (b, t, h * d)
    for i in range(b):
        s = int(slot_of[i])
        k_all = kp[s, :, : start + t].unsqueeze(0)
        v_all = vp[s, :, : start + t].unsqueeze(0)
        want = nebula_attention(q[i : i + 1].transpose(1, 2), k_all, v_all, start)  # [1,h,t,d]
        close(got[i].view(t, h, d).transpose(0, 1), want[0], dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("b,t,h,d,max_seq,start", [(32, 1, 16, 128, 2048, 512), (3, 7, 4, 4, 16, 2), (2, 2, 3, 40, 64, 10)])
def test_kv_append_exact(cuda, dtype, b, t, h, d, max_seq, start):
    slots = b + 1
    kp = torch.zeros(slots, h, max_seq, d, dtype=dtype, device=cuda)
    vp = torch.zeros_like(kp)
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(b, t, 3 * h * d, generator=g).to(dtype).to(cuda)
    k = qkv[..., h * d: 2 * h * d].reshape(b, t, h, d)
    v = qkv[..., 2 * h * d:].reshape(b, t, h, d)
    slot_of = torch.tensor([(i + 1) % slots for i in range(b)], dtype=torch.int32, device=cuda)
    starts = torch.full((b,), start, dtype=torch.int32, device=cuda)
    nops.kv_append(k, v, kp, vp, slot_of, starts)
    want_k = torch.zeros_like(kp)
    want_v = torch.zeros_like(vp)
    for i in range(b):
        s = int(slot_of[i])
        want_k[s, :, start:start + t] = k[i].transpose(0, 1)
        want_v[s, :, start:start + t] = v[i].transpose(0, 1)
    assert torch.equal(kp, want_k) and torch.equal(vp, want_v)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_embed(cuda, dtype):
    g = torch.Generator().manual_seed(2)
    te = torch.randn(100, 64, generator=g).to(dtype)
    pe = torch.randn(40, 64, generator=g).to(dtype)
    toks = torch.randint(0, 100, (3, 5), generator=g)
    starts = torch.tensor([0, 7, 30], dtype=torch.int32)
    got = nops.embed(toks.to(cuda), starts.to(cuda), te.to(cuda), pe.to(cuda))
    pos = starts[:, None].long() + torch.arange(5)[None, :]
    want = te[toks] + pe[pos]  # torch rounds the sum to dtype once, like the reference
    assert torch.equal(got.cpu(), want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(32, 32000), (3, 17), (1, 1)])
def test_argmax_exact_with_ties(cuda, dtype, rows, cols):
    g = torch.Generator().manual_seed(rows)
    x = torch.randn(rows, cols, generator=g).to(dtype)
    if cols > 4:
        x[:, cols // 2] = 50.0
        x[:, cols - 2] = 50.0  # tie: first index wins
    got = nops.argmax(x.to(cuda))
    assert torch.equal(got.cpu(), x.argmax(-1))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_argmax_nan_wins_first(cuda, dtype):
    x = torch.randn(4, 32000, generator=torch.Generator().manual_seed(6)).to(dtype)
    x[1, 777] = float("nan")
    x[1, 20000] = float("nan")
    x[2, 31999] = float("inf")
    assert torch.equal(nops.argmax(x.to(cuda)).cpu(), x.argmax(-1))


def test_add_rounding(cuda):
    g = torch.Generator().manual_seed(4)
    a = torch.randn(1000, generator=g).to(torch.bfloat16)
    b = torch.randn(1000, generator=g).to(torch.bfloat16)
    assert torch.equal(nops.add(a.to(cuda), b.to(cuda)).cpu(), a + b)


def test_device_status_after_ops(cuda):
    from forgeml_b200 import _native

    assert _native.device_status() == 0
