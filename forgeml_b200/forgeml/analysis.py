"""Static cost model used by CompiledModel.explain().

Same accounting as the reference (src/forgeml/analysis.py:14-105): GEMM
2*M*N*K (+ bias, + 8/elt for GELU), elementwise 1/elt, GELU 8, softmax 5,
LayerNorm 6, SDPA 2*pairs*2*hd + 5 (6 with a mask) per query/key pair
(causal pairs counted once), conv2d 2*MAC; view ops move no bytes.
"""

from __future__ import annotations

import math
from collections import Counter

from forgeml_b200.forgeml.ir import Graph
from forgeml_b200.forgeml.memory import VIEW_LIKE_OPS


def node_flops(node, ins) -> int:
    elems = math.prod(node.spec.shape)
    op = node.op
    if op in ("matmul", "linear", "fused_linear_gelu"):
        (m, k), n = ins[0].shape, ins[1].shape[1]
        f = 2 * m * k * n
        if op != "matmul" and len(ins) == 3:
            f += elems
        return f + (8 * elems if op == "fused_linear_gelu" else 0)
    if op in ("add", "mul", "relu"):
        return elems
    if op == "gelu":
        return 8 * elems
    if op == "softmax":
        return 5 * elems
    if op == "layer_norm":
        return 6 * elems
    if op == "sdpa":
        b, h, sq, hd = ins[0].shape
        sk = ins[1].shape[2]
        pairs = b * h * sq * sk
        if node.attrs.get("is_causal"):
            pairs = min(pairs, b * h * (sq * (sq + 1) // 2))
        return 4 * hd * pairs + (6 if len(ins) == 4 else 5) * pairs
    if op == "conv2d":
        _, _, oh, ow = node.spec.shape
        oc, ipg, kh, kw = ins[1].shape
        return 2 * ins[0].shape[0] * oh * ow * oc * ipg * kh * kw + (elems if len(ins) == 3 else 0)
    return 0


def graph_analysis(graph: Graph) -> dict:
    graph.validate()
    specs = graph.specs()
    rows, depth = [], {}
    flops = byts = 0
    for n in graph.nodes:
        ins = [specs[i] for i in n.inputs]
        f = node_flops(n, ins)
        lb = 0 if n.op in VIEW_LIKE_OPS else sum(specs[i].nbytes for i in dict.fromkeys(n.inputs)) + n.spec.nbytes
        depth[n.name] = 1 + max((depth.get(i, 0) for i in n.inputs), default=0)
        rows.append({"name": n.name, "op": n.op, "flops": f, "logical_bytes": lb,
                     "arithmetic_intensity": f / max(lb, 1), "depth": depth[n.name],
                     "output_shape": list(n.spec.shape)})
        flops += f
        byts += lb
    return {
        "model": "static_operator_cost_bounds_not_measured_hardware_counters",
        "nodes": len(graph.nodes),
        "op_counts": dict(sorted(Counter(n.op for n in graph.nodes).items())),
        "flops": flops,
        "logical_bytes": byts,
        "arithmetic_intensity": flops / max(byts, 1),
        "critical_path_ops": max(depth.values(), default=0),
        "input_bytes": sum(s.nbytes for s in graph.inputs.values()),
        "constant_bytes": sum(t.numel() * t.element_size() for t in graph.constants.values()),
        "output_bytes": sum(specs[o].nbytes for o in graph.outputs),
        "dominant_nodes": sorted(rows, key=lambda r: (r["flops"], r["logical_bytes"], r["name"]), reverse=True)[:5],
        "per_node": rows,
    }
