"""Cached loaders for the committed golden fixtures (tests/golden/)."""

import functools
import json
from pathlib import Path

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


@functools.lru_cache(maxsize=None)
def load_gemm_golden() -> dict:
    return torch.load(GOLDEN / "gemm.pt", weights_only=False)


@functools.lru_cache(maxsize=None)
def load_memory_plans() -> dict:
    return json.loads((GOLDEN / "memory_plans.json").read_text())


@functools.lru_cache(maxsize=None)
def load_nebula_small() -> dict:
    return torch.load(GOLDEN / "nebula_small.pt", weights_only=False)
