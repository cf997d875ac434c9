"""The CPU oracle is pinned against golden vectors produced by running the
reference itself (tests/golden/make_golden.py).  CPU only."""

import math

import pytest
import torch

from oracle import memory as orc_memory
from oracle import nebula as orc_nebula
from oracle.attention import nebula_attention, sdpa
from oracle.gemm import matmul_epilogue
from oracle.layernorm import layer_norm
from tests.golden_io import load_gemm_golden, load_memory_plans, load_nebula_small

TOL = {torch.float32: (1e-5, 1e-5), torch.float16: (1e-2, 1e-2), torch.bfloat16: (2e-2, 2e-2)}


@pytest.mark.parametrize("idx", range(len(load_gemm_golden()["cases"])))
def test_gemm_oracle_matches_reference_contract(idx):
    c = load_gemm_golden()["cases"][idx]
    a, b = c["a"], c["b"]
    if c["kind"] == "transposed":
        a, b = a.t(), b.t()
    bias = c["bias"]
    if bias is not None and c.get("bias_step"):
        bias = bias[:: c["bias_step"]]
    got = matmul_epilogue(a, b, bias, activation=c["activation"], approximate=c["approximate"])
    rtol, atol = TOL[a.dtype]
    torch.testing.assert_close(got.float(), c["want"].float(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", sorted(load_memory_plans()))
def test_planner_oracle_matches_reference_plans(name):
    rec = load_memory_plans()[name]
    g = rec["graph"]
    assert orc_memory.plan(g["nodes"], g["outputs"]) == rec["plan"]


def test_nebula_oracle_matches_reference_engine():
    gold = load_nebula_small()
    cfg = gold["config"]
    w = orc_nebula.weights_from_state_dict(gold["state_dict"], cfg["num_layers"])
    got = orc_nebula.forward(w, gold["prefill_tokens"], cfg["num_heads"], cfg["num_layers"])
    torch.testing.assert_close(got, gold["prefill_logits"], rtol=1e-5, atol=1e-6)
    full = torch.cat([gold["prefill_tokens"], gold["decode_tokens"]], 1)
    got_d = orc_nebula.forward(w, full, cfg["num_heads"], cfg["num_layers"])[:, -1:]
    torch.testing.assert_close(got_d, gold["decode_logits"], rtol=1e-5, atol=1e-6)
    toks = [orc_nebula.greedy(w, p, 3, cfg["num_heads"], cfg["num_layers"]) for p in gold["generate_prompts"]]
    assert toks == gold["generate_tokens"]
    long = orc_nebula.greedy(w, gold["generate_long_prompt"][0], 8, cfg["num_heads"], cfg["num_layers"])
    assert [long] == gold["generate_long_tokens"]


def test_nebula_oracle_incremental_matches_full():
    gold = load_nebula_small()
    cfg = gold["config"]
    w = orc_nebula.weights_from_state_dict(gold["state_dict"], cfg["num_layers"])
    hd = cfg["hidden_size"] // cfg["num_heads"]
    caches = [(torch.zeros(2, cfg["num_heads"], 16, hd), torch.zeros(2, cfg["num_heads"], 16, hd))
              for _ in range(cfg["num_layers"])]
    p = orc_nebula.forward(w, gold["prefill_tokens"], cfg["num_heads"], cfg["num_layers"], caches=caches, start_pos=0)
    torch.testing.assert_close(p, gold["prefill_logits"], rtol=1e-5, atol=1e-6)
    d = orc_nebula.forward(w, gold["decode_tokens"], cfg["num_heads"], cfg["num_layers"], caches=caches, start_pos=3)
    torch.testing.assert_close(d, gold["decode_logits"], rtol=1e-5, atol=1e-6)


def test_layernorm_and_sdpa_oracles_match_torch():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(7, 33, generator=g)
    w, b = torch.randn(33, generator=g), torch.randn(33, generator=g)
    torch.testing.assert_close(layer_norm(x, 33, w, b), torch.nn.functional.layer_norm(x, (33,), w, b, 1e-5),
                               rtol=1e-5, atol=1e-5)
    q, k, v = (torch.randn(2, 3, 9, 8, generator=g) for _ in range(3))
    mask = torch.rand(2, 1, 9, 9, generator=g) > 0.3
    mask[..., 0] = True
    for kw in ({}, {"is_causal": True}, {"attn_mask": mask}):
        torch.testing.assert_close(sdpa(q, k, v, **kw), torch.nn.functional.scaled_dot_product_attention(q, k, v, **kw),
                                   rtol=1e-5, atol=1e-5)
    # decode attention at an absolute offset equals the full masked computation
    kk, vv = torch.randn(1, 3, 12, 8, generator=g), torch.randn(1, 3, 12, 8, generator=g)
    qq = torch.randn(1, 3, 2, 8, generator=g)
    got = nebula_attention(qq, kk, vv, start_pos=10)
    s = (qq @ kk.transpose(-1, -2)) / math.sqrt(8)
    s[..., 0, 11] = float("-inf")
    torch.testing.assert_close(got, torch.softmax(s, -1) @ vv, rtol=1e-5, atol=1e-6)
