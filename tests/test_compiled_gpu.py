"""Compiled forward pass on the B200 with the native backend (configs 1 and 2).

GEMM-family, LayerNorm and SDPA nodes run the sm_100a kernels and write the
slot arena (GEMMs) or the extension arena (LN, SDPA).  Parity against the
reference's torch CPU path on identical seeded inputs:
  fp32: rtol 1e-5, atol 1e-4
  bf16: rtol 2e-2, atol 2e-2 * max|expected|
"""

import pytest
import torch
from torch import nn

from forgeml_b200.forgeml import compile
from forgeml_b200.forgeml.memory import plan_memory
from forgeml_b200.workloads import EncoderBlock, make_c1_mlp, make_c2_block

pytestmark = pytest.mark.gpu


def _native_nodes(c):
    return {n.op for n in c.graph.nodes if c.kernel_plan[n.name] == "triton"}


def test_c1_mlp_fp32(cuda):
    m, x = make_c1_mlp()
    with torch.no_grad():
        want = m(x)
    c = compile(m.to(cuda), (x.to(cuda),), backend="triton")
    assert _native_nodes(c) == {"fused_linear_gelu", "linear"}
    got = c(x.to(cuda))
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-4)
    # slot plan is the reference's, independent of the backend
    assert c.memory_plan.to_dict() == plan_memory(c.graph).to_dict()


def test_c2_block_fp32(cuda):
    m, x = make_c2_block()
    with torch.no_grad():
        want = m(x)
    c = compile(m.to(cuda), (x.to(cuda),), backend="triton")
    assert _native_nodes(c) == {"linear", "fused_linear_gelu", "layer_norm", "sdpa"}
    got = c(x.to(cuda))
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-4)
    again = c(x.to(cuda))  # arena reuse across calls
    torch.testing.assert_close(again.cpu(), want, rtol=1e-5, atol=1e-4)


def test_c2_block_bf16(cuda):
    m, x = make_c2_block(dtype=torch.bfloat16)
    with torch.no_grad():
        want = m.float()(x.float())  # fp32 evaluation of the bf16 weights and inputs
    m = m.to(torch.bfloat16)
    c = compile(m.to(cuda), (x.to(cuda),), backend="auto")
    assert "sdpa" in _native_nodes(c)
    got = c(x.to(cuda)).float().cpu()
    torch.testing.assert_close(got, want, rtol=2e-2, atol=2e-2 * float(want.abs().max()))


def test_small_blocks_causal_and_odd_sizes(cuda):
    torch.manual_seed(3)

    class Blk(nn.Module):
        def __init__(self):
            super().__init__()
            self.inner = EncoderBlock(96, 3, 200)

        def forward(self, x):
            y = self.inner(x)
            q = y.view(2, 37, 3, 32).transpose(1, 2)
            a = torch.nn.functional.scaled_dot_product_attention(q, q, q, is_causal=True)
            return a.transpose(1, 2).reshape(2, 37, 96) + y

    m = Blk().eval()
    x = torch.randn(2, 37, 96)
    with torch.no_grad():
        want = m(x)
    c = compile(m.to(cuda), (x.to(cuda),), backend="triton")
    torch.testing.assert_close(c(x.to(cuda)).cpu(), want, rtol=1e-5, atol=1e-4)


def test_mixed_plan(cuda):
    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(16, 16)

        def forward(self, x):
            return torch.relu(self.lin(x)) + x

    m = M().eval().to(cuda)
    x = torch.randn(4, 16, device=cuda)
    c = compile(m, (x,), backend="auto")
    assert "triton" in c.kernel_plan.values() and "torch" in c.kernel_plan.values()
    torch.testing.assert_close(c(x), m(x), rtol=1e-5, atol=1e-4)


def test_autotune_selects_valid_candidates(cuda):
    m, x = make_c1_mlp()
    c = compile(m.to(cuda), (x.to(cuda),), backend="triton")
    rep = c.autotune(x.to(cuda), warmup=1, repeats=2)
    assert set(rep["nodes"]) == {n.name for n in c.graph.nodes if c.kernel_plan[n.name] == "triton"}
    assert all(r["winner"] in r["candidates"] for r in rep["nodes"].values())
    with torch.no_grad():
        want = m.cpu()(x)
    torch.testing.assert_close(c(x.to(cuda)).cpu(), want, rtol=1e-5, atol=1e-4)
