"""Nebula tensor-/pipeline-parallel decoding on sm_100a kernels (drop-in for `nebula`)."""

from forgeml_b200.nebula.cache import CacheError, KVCache
from forgeml_b200.nebula.model import DecoderConfig, TinyDecoder
from forgeml_b200.nebula.parallel import ParallelContext
from forgeml_b200.nebula.runtime import Engine, EngineFailed, ShardedDecoder

__all__ = [
    "CacheError",
    "DecoderConfig",
    "Engine",
    "EngineFailed",
    "KVCache",
    "ParallelContext",
    "ShardedDecoder",
    "TinyDecoder",
]
