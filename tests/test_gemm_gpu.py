"""GEMM parity on the B200: native tcgen05 GEMM vs the CPU oracle and the
golden vectors generated from the reference (tests/golden/make_golden.py).

Mirrors the reference's GPU kernel tests (tests/test_kernels.py:101-181 of the
reference) and extends them to the headline shapes' layouts: skinny M (swap
+ cluster split-K), transposed B, row-strided A, K not a multiple of the
slab, fused residual.

Tolerances (written here, per dtype):
  fp32 (3xTF32): rtol 1e-5, atol 1e-4     (north-star fp32 bar)
  fp16         : rtol 1e-2, atol 1e-2
  bf16         : rtol 2e-2, atol 2e-2     (north-star bf16 bar; reference gate was 5e-2)
"""

import pytest
import torch

from oracle.gemm import matmul_epilogue
from forgeml_b200.forgeml.ir import GraphError
from forgeml_b200.forgeml import kernels
from tests.golden_io import load_gemm_golden

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-4), torch.float16: (1e-2, 1e-2), torch.bfloat16: (2e-2, 2e-2)}


def close(got, want, dtype):
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(got.float().cpu(), want.float().cpu(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("idx", range(len(load_gemm_golden()["cases"])))
def test_golden_cases(cuda, idx):
    case = load_gemm_golden()["cases"][idx]
    a, b = case["a"].to(cuda), case["b"].to(cuda)
    if case["kind"] == "transposed":
        a, b = a.t(), b.t()
    bias = case["bias"]
    if bias is not None:
        bias = bias.to(cuda)
        if case.get("bias_step"):
            bias = bias[:: case["bias_step"]]
    got = kernels.matmul(a, b, bias, activation=case["activation"], approximate=case["approximate"])
    close(got, case["want"], a.dtype)
    # the torch-backend evaluation of the reference agrees within the same gate
    close(got, case["want_torch"], a.dtype)


SHAPES = [
    (128, 256, 64),
    (256, 512, 1024),
    (300, 700, 513),
    (1, 4096, 4096),
    (16, 4096, 4096),
    (128, 4096, 4096),
    (32, 2048, 8192),
    (32, 6144, 2048),
    (1024, 1024, 1024),
    (4096, 2304, 768),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("variant", ["plain", "bias_gelu", "bias_tanh", "transposed_b", "strided_a"])
def test_shapes_vs_oracle(cuda, dtype, m, n, k, variant):
    if dtype == torch.float32 and m * n * k > 2**31:
        pytest.skip("fp32 oracle cost bounded to keep the suite short")
    g = torch.Generator().manual_seed(m * 31 + n * 7 + k)
    if variant == "strided_a":
        a_cpu = (torch.rand(2 * m, k, generator=g) * 2 - 1).to(dtype)[::2]
    else:
        a_cpu = (torch.rand(m, k, generator=g) * 2 - 1).to(dtype)
    if variant == "transposed_b":
        b_cpu = (torch.rand(n, k, generator=g) * 2 - 1).to(dtype).t()
    else:
        b_cpu = (torch.rand(k, n, generator=g) * 2 - 1).to(dtype)
    bias_cpu = torch.randn(n, generator=g).to(dtype)
    act = "gelu" if variant in ("bias_gelu", "bias_tanh") else "none"
    approx = "tanh" if variant == "bias_tanh" else "none"
    use_bias = variant != "plain"
    if variant == "strided_a":
        base = torch.empty(2 * m, k, dtype=dtype, device=cuda)
        base[::2] = a_cpu.to(cuda)
        a = base[::2]
    else:
        a = a_cpu.to(cuda)
    if variant == "transposed_b":
        b = b_cpu.t().contiguous().to(cuda).t()
    else:
        b = b_cpu.to(cuda)
    bias = bias_cpu.to(cuda) if use_bias else None
    got = kernels.matmul(a, b, bias, activation=act, approximate=approx)
    want = matmul_epilogue(a_cpu, b_cpu, bias_cpu if use_bias else None, activation=act, approximate=approx)
    close(got, want, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("m,n,k", [(32, 2048, 2048), (32, 2048, 8192), (5, 300, 70), (64, 512, 2048)])
def test_residual_epilogue(cuda, dtype, m, n, k):
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(m, k, generator=g) * 0.5).to(dtype)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dtype)  # nn.Linear layout [out, in]
    r = torch.randn(m, n, generator=g).to(dtype)
    got = kernels.matmul(x.to(cuda), w.to(cuda).t(), residual=r.to(cuda))
    want = matmul_epilogue(x, w.t(), residual=r)
    close(got, want, dtype)


def test_out_buffer_and_overlap_reject(cuda):
    a = torch.randn(16, 16, device=cuda)
    b = torch.randn(16, 16, device=cuda)
    out = torch.empty(16, 16, device=cuda)
    got = kernels.matmul(a, b, out=out)
    assert got.data_ptr() == out.data_ptr()
    close(out, matmul_epilogue(a.cpu(), b.cpu()), torch.float32)
    with pytest.raises(GraphError, match="storage"):
        kernels.matmul(a, b, out=a)


@pytest.mark.parametrize("cfg", kernels.CANDIDATES)
def test_candidates_agree(cuda, cfg):
    g = torch.Generator().manual_seed(3)
    a = torch.randn(200, 320, generator=g).to(torch.bfloat16)
    b = torch.randn(320, 520, generator=g).to(torch.bfloat16)
    bias = torch.randn(520, generator=g).to(torch.bfloat16)
    got = kernels.matmul(a.to(cuda), b.to(cuda), bias.to(cuda), activation="gelu", config=cfg)
    close(got, matmul_epilogue(a, b, bias, activation="gelu"), torch.bfloat16)


def test_repeat_is_deterministic(cuda):
    g = torch.Generator().manual_seed(5)
    a = torch.randn(32, 8192, generator=g).to(torch.bfloat16).to(cuda)
    b = torch.randn(8192, 2048, generator=g).to(torch.bfloat16).to(cuda)
    r1 = kernels.matmul(a, b)
    r2 = kernels.matmul(a, b)
    assert torch.equal(r1, r2)


def test_device_status_clean(cuda):
    from forgeml_b200 import _native

    a = torch.randn(256, 256, device=cuda, dtype=torch.bfloat16)
    kernels.matmul(a, a)
    assert _native.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(32, 6144, 2048), (32, 2048, 8192), (1, 300, 70), (5, 32000, 2048),
                                   (130, 1000, 1000), (512, 2048, 2048)])
@pytest.mark.parametrize("epi", ["plain", "gelu_tanh", "residual", "bias"])
def test_packed_linear(cuda, dtype, m, n, k, epi):
    """Pre-packed constant-weight GEMM (Nebula decode path) vs the oracle contract."""
    from forgeml_b200.linear import PackedLinear

    g = torch.Generator().manual_seed(m + n + k)
    x = (torch.randn(m, k, generator=g) * 0.5).to(dtype)
    w = (torch.randn(n, k, generator=g) * 0.05).to(dtype)
    r = torch.randn(m, n, generator=g).to(dtype) if epi == "residual" else None
    bias = torch.randn(n, generator=g).to(dtype) if epi == "bias" else None
    lin = PackedLinear(w.to(cuda))
    out = torch.empty(m, n, dtype=dtype, device=cuda)
    act = 2 if epi == "gelu_tanh" else 0
    lin(x.to(cuda), out, act=act, residual=r.to(cuda) if r is not None else None,
        bias=bias.to(cuda) if bias is not None else None)
    want = matmul_epilogue(x, w.t(), bias, activation="gelu" if act else "none",
                           approximate="tanh" if act else "none", residual=r)
    close(out, want, dtype)


@pytest.mark.parametrize("m,n,k", [(64, 2048, 512), (64, 512, 2048), (300, 700, 513), (4096, 768, 768),
                                   (1, 1000, 33)])
@pytest.mark.parametrize("epi", ["plain", "bias_gelu", "residual"])
@pytest.mark.parametrize("layout", ["linear_t", "row_major"])
def test_packed_b_fp32(cuda, m, n, k, epi, layout):
    """fp32 B split once (fml_gemm_pack_b) then used by fml_gemm_packed_b:
    same product as fml_gemm, checked against the oracle at the fp32 bar;
    a B written in place is split again before the next call."""
    g = torch.Generator().manual_seed(m + 3 * n + 11 * k)
    a_cpu = torch.rand(m, k, generator=g) * 2 - 1
    w_cpu = torch.rand(n, k, generator=g) * 2 - 1
    b_cpu = w_cpu.t() if layout == "linear_t" else w_cpu.t().contiguous()
    bias_cpu = torch.randn(n, generator=g) if epi != "plain" else None
    res_cpu = torch.randn(m, n, generator=g) if epi == "residual" else None
    act = "gelu" if epi == "bias_gelu" else "none"
    b = w_cpu.to(cuda).t() if layout == "linear_t" else b_cpu.to(cuda)
    launch = kernels.PreparedGemm(torch.float32, act)
    launch.pack_constant_b(b)
    out = torch.empty(m, n, device=cuda)
    args = (a_cpu.to(cuda), b, None if bias_cpu is None else bias_cpu.to(cuda), out)
    launch(*args, residual=None if res_cpu is None else res_cpu.to(cuda))
    want = matmul_epilogue(a_cpu, b_cpu, bias_cpu, activation=act, residual=res_cpu)
    close(out, want, torch.float32)
    b.mul_(0.5)  # in place: the image must follow
    launch(*args, residual=None if res_cpu is None else res_cpu.to(cuda))
    want = matmul_epilogue(a_cpu, b_cpu * 0.5, bias_cpu, activation=act, residual=res_cpu)
    close(out, want, torch.float32)


@pytest.mark.parametrize("approximate", ["none", "tanh"])
def test_gelu_epilogue_accuracy(cuda, approximate):
    """The epilogue's GELU against torch's (fp64) over [-8, 8): an fp32
    identity product passes the values through exactly (multiples of 1/64
    are exact in the 3xTF32 split), so out = gelu(b) elementwise.  The erf
    form uses the Abramowitz & Stegun 7.1.26 erf (|error| <= 1.5e-7)."""
    xs = (torch.arange(1024, dtype=torch.float64) / 64 - 8).to(torch.float32)
    b = xs.view(8, 128).t().contiguous()          # [K=128, N=8]: every value in some column
    a = torch.eye(128, dtype=torch.float32)
    got = kernels.matmul(a.to(cuda), b.to(cuda), activation="gelu", approximate=approximate).cpu().double()
    want = torch.nn.functional.gelu(b.double(), approximate=approximate)
    err = (got - want).abs()
    assert float(err.max()) <= 2e-7 * max(1.0, float(b.abs().max())) + 1e-7, float(err.max())


@pytest.mark.parametrize("m,n,k,epi", [(512, 1024, 768, "bias_gelu"), (1024, 768, 3072, "residual"),
                                       (384, 512, 256, "plain")])
def test_cta_pair_tiles(cuda, m, n, k, epi):
    """CTA-pair tiles (tile hint block_m = 256: cta_group::2, 256 x 256 per
    pair) against the oracle, including an M that leaves half a pair tile."""
    g = torch.Generator().manual_seed(m + n + k)
    a = (torch.rand(m, k, generator=g) * 2 - 1).to(torch.bfloat16)
    w = (torch.rand(n, k, generator=g) * 2 - 1).to(torch.bfloat16)
    bias = torch.randn(n, generator=g).to(torch.bfloat16) if epi == "bias_gelu" else None
    res = torch.randn(m, n, generator=g).to(torch.bfloat16) if epi == "residual" else None
    act = "gelu" if epi == "bias_gelu" else "none"
    cfg = kernels.KernelConfig(256, 256, 64, 6, 7)
    got = kernels.matmul(a.to(cuda), w.to(cuda).t(), None if bias is None else bias.to(cuda), activation=act,
                         residual=None if res is None else res.to(cuda), config=cfg)
    close(got, matmul_epilogue(a, w.t(), bias, activation=act, residual=res), torch.bfloat16)


def test_packed_b_inference_tensors(cuda):
    """A graph compiled under torch.inference_mode holds inference-tensor
    weights (no version counter): the fp32 split is made once and used."""
    from forgeml_b200.forgeml import compile as fml_compile

    with torch.inference_mode():
        lin = torch.nn.Linear(96, 160).to(cuda)
        x = torch.randn(8, 96, device=cuda)
        c = fml_compile(torch.nn.Sequential(lin), (x,), backend="triton")
        got = c(x)
        want = lin(x)
    close(got, want.cpu(), torch.float32)
