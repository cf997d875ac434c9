"""forgeml_b200: sm_100a (B200) kernels behind ForgeML's compiled forward pass
and Nebula's tensor-/pipeline-parallel decode step.

Subpackages mirror the reference's public modules:
  forgeml_b200.forgeml  -- compile / CompiledModel / kernels.matmul / autotune
  forgeml_b200.nebula   -- Engine / ShardedDecoder / KVCache / ParallelContext / AsyncBatcher
The compute runs in ``_lib/libforgeml_b200.so`` (C ABI: include/forgeml_b200.h).
"""

__version__ = "0.1.0"
