"""Correctness-gated autotuning (forgeml_b200/forgeml/autotune.py) on the CPU
with the kernel launch and the timer replaced by fakes, as the reference's
tests/test_measurement.py:58-149 does: a candidate that returns a wrong
result or raises is rejected, the fastest survivor wins, the choice stays on
the compiled-model instance, and a node with no valid candidate is an error."""

import pytest
import torch
from torch import nn

from forgeml_b200.forgeml import autotune, compile, kernels
from forgeml_b200.forgeml.kernels import CANDIDATES


def _mlp():
    torch.manual_seed(0)
    m = nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 8)).eval()
    return m, torch.randn(4, 16)


def _native_plan(c):
    c.kernel_plan = {n.name: ("triton" if n.op in ("linear", "fused_linear_gelu", "matmul") else "torch")
                     for n in c.graph.nodes}


def _fake_launch(bad=(), raising=()):
    """torch stand-in for PreparedGemm.__call__; candidates in `bad` return a
    wrong result, those in `raising` fail to launch."""

    def fake(self, a, b, bias, out, residual=None):
        if self.config in raising:
            raise RuntimeError("launch failed (fake)")
        y = a @ b if bias is None else torch.addmm(bias, a, b)
        if self.act:
            y = torch.nn.functional.gelu(y, approximate="tanh" if self.act == 2 else "none")
        if residual is not None:
            y = y + residual
        if self.config in bad:
            y = y + 1.0
        return out.copy_(y)

    return fake


def _fake_timer(order):
    """_time_candidates stand-in: candidate_i gets median order[i] ms."""

    def fake(runs, *, device, warmup, repeats):
        out = {}
        for name, fn in runs.items():
            fn()
            idx = int(name.split("_")[1])
            out[name] = {"median_ms": order[idx], "samples_ms": [order[idx]] * repeats}
        return out

    return fake


def test_fastest_correct_candidate_wins(monkeypatch):
    m, x = _mlp()
    c = compile(m, (x,), backend="torch")
    _native_plan(c)
    monkeypatch.setattr(kernels.PreparedGemm, "__call__", _fake_launch(bad={CANDIDATES[1]}, raising={CANDIDATES[2]}))
    # candidate 1 is the fastest but wrong, 2 fails to launch, 3 is the fastest survivor
    monkeypatch.setattr(autotune, "_time_candidates", _fake_timer([4.0, 0.5, 0.1, 1.0, 2.0]))
    rep = autotune.tune_graph(c, (x,), warmup=0, repeats=2)
    assert rep["scope"] == "this_compiled_model_instance_only"
    assert rep["nodes"], "no native GEMM node was tuned"
    for name, rec in rep["nodes"].items():
        assert rec["winner"] == "candidate_3"
        assert set(rec["rejected"]) == {"candidate_1", "candidate_2"}
        assert "launch failed" in rec["rejected"]["candidate_2"]
        assert "wrong result" in rec["rejected"]["candidate_1"]
        assert set(rec["candidates"]) == {"candidate_0", "candidate_3", "candidate_4"}
        assert all(v["correctness"]["passed"] for v in rec["candidates"].values())
        assert c.kernel_configs[name] == CANDIDATES[3]
    other = compile(m, (x,), backend="torch")
    assert not other.kernel_configs  # selections live on the tuned instance only
    torch.testing.assert_close(c(x), m(x), rtol=1e-5, atol=1e-5)


def test_no_valid_candidate_is_an_error(monkeypatch):
    m, x = _mlp()
    c = compile(m, (x,), backend="torch")
    _native_plan(c)
    monkeypatch.setattr(kernels.PreparedGemm, "__call__", _fake_launch(bad=set(CANDIDATES)))
    monkeypatch.setattr(autotune, "_time_candidates", _fake_timer([1.0] * len(CANDIDATES)))
    with pytest.raises(RuntimeError, match="no numerically valid kernel candidate"):
        autotune.tune_graph(c, (x,), warmup=0, repeats=2)


def test_autotune_argument_checks():
    m, x = _mlp()
    c = compile(m, (x,), backend="torch")
    with pytest.raises(ValueError):
        autotune.tune_graph(c, (x,), warmup=-1, repeats=2)
    with pytest.raises(ValueError):
        autotune.tune_graph(c, (x,), warmup=0, repeats=1)
