"""ForgeML compiled-forward path on sm_100a kernels (drop-in for the `forgeml` package)."""

from forgeml_b200.forgeml.ir import Graph, GraphBuilder, GraphError, Node, TensorSpec

__all__ = ["Graph", "GraphBuilder", "GraphError", "Node", "TensorSpec"]
