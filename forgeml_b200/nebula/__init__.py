"""Nebula tensor-/pipeline-parallel decoding on sm_100a kernels (drop-in for `nebula`)."""

from forgeml_b200.nebula.cache import CacheError, KVCache
from forgeml_b200.nebula.model import DecoderConfig, TinyDecoder
from forgeml_b200.nebula.parallel import ParallelContext
from forgeml_b200.nebula.engine import Engine, EngineFailed
from forgeml_b200.nebula.runtime import ShardedDecoder
from forgeml_b200.nebula.scheduler import AsyncBatcher, QueueFull, ServiceClosed

__all__ = [
    "AsyncBatcher",
    "QueueFull",
    "ServiceClosed",
    "CacheError",
    "DecoderConfig",
    "Engine",
    "EngineFailed",
    "KVCache",
    "ParallelContext",
    "ShardedDecoder",
    "TinyDecoder",
]
