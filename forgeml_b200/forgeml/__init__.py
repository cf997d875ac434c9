"""ForgeML compiled-forward path on sm_100a kernels (drop-in for the `forgeml` package)."""

from forgeml_b200.forgeml.compiler import CompiledModel, compile
from forgeml_b200.forgeml.frontend import from_torch
from forgeml_b200.forgeml.ir import Graph, GraphBuilder, GraphError, Node, TensorSpec

__all__ = ["CompiledModel", "Graph", "GraphBuilder", "GraphError", "Node", "TensorSpec", "compile",
           "from_torch"]
