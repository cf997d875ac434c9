"""Parity at the shapes the headline numbers are quoted on.

Config 4 (the decode benchmark): the full 12-layer d2048 decoder in bf16 at
batch 32 on one B200 -- the M=32 tile choices, LayerNorm-folded QKV / up
launches, KV-append epilogue and CUDA-graph step the benchmark times -- run
greedily for 16 steps and compared, step by step, with the reference's own
TinyDecoder forward on the host in fp32 over the bf16-rounded weights,
teacher-forced with the engine's tokens (bench.decode_parity):
  logits      max |got - want| <= 2e-2 * max |want|   (north-star bf16 bar)
  greedy      argmax agreement >= 0.9 of (request, step) pairs, reported
              (bf16 rounding may flip near-ties)

Config 3 (the GEMM sweep): the square 4096^3 / 8192^3 products with bias +
exact GELU in bf16 and fp32 (3xTF32), transposed-B and row-strided-A at
4096^3, checked on a seeded sample of output rows against the fp64-accumulated
oracle contract (the full fp64 product would take minutes on the host):
  bf16 rtol 2e-2 / atol 2e-2,  fp32 rtol 1e-5 / atol 1e-4.
"""

import pytest
import torch

from oracle.gemm import matmul_epilogue

pytestmark = pytest.mark.gpu

C4 = dict(vocab_size=32000, hidden_size=2048, num_heads=16, num_layers=12, intermediate_size=8192,
          max_seq_len=2048, seed=3)


def test_c4_full_model_greedy_parity(cuda):
    import bench
    from forgeml_b200.nebula import DecoderConfig, ParallelContext
    from forgeml_b200.nebula.runtime import ShardedDecoder

    dec = ShardedDecoder(DecoderConfig(**C4), ParallelContext.from_env(device="cuda"), dtype=torch.bfloat16,
                         max_requests=32, init="normal")
    try:
        res = bench.decode_parity(dec, cuda, batch=32, prompt_len=16, steps=16)
    finally:
        dec.close()
    print(f"c4 full model: max_rel_err {res['max_rel_err']:.3e}, greedy agreement {res['greedy_agree']:.4f}")
    assert res["max_rel_err"] <= 2e-2, res
    assert res["greedy_agree"] >= 0.9, res


CASES = [
    (4096, torch.bfloat16, "plain"),
    (8192, torch.bfloat16, "plain"),
    (4096, torch.bfloat16, "transposed_b"),
    (4096, torch.bfloat16, "strided_a"),
    (4096, torch.float32, "plain"),
    (8192, torch.float32, "plain"),
]


@pytest.mark.parametrize("size,dtype,variant", CASES)
def test_c3_square_sampled_rows(cuda, size, dtype, variant):
    from forgeml_b200.forgeml import kernels
    from forgeml_b200.workloads import make_c3_operands

    a, b, bias = make_c3_operands(size, size, size, dtype, transposed_b=variant == "transposed_b",
                                  strided_a=variant == "strided_a", device="cuda")
    out = kernels.matmul(a, b, bias, activation="gelu")
    rows = torch.randperm(size, generator=torch.Generator().manual_seed(size))[:48].sort().values
    want = matmul_epilogue(a[rows.to(cuda)].cpu(), b.cpu(), bias.cpu(), activation="gelu")
    rtol, atol = (2e-2, 2e-2) if dtype == torch.bfloat16 else (1e-5, 1e-4)
    torch.testing.assert_close(out[rows.to(cuda)].float().cpu(), want.float(), rtol=rtol, atol=atol)
