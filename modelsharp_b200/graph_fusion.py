"""Engine-level fusion of a decoder graph onto the fused decode GEMV.

`fuse_decode_graph` rewrites three patterns of an INT4 decoder graph into
`MatMulNBitsFused` nodes (msq_matmul_fused: the decode GEMV with RMSNorm or SwiGLU folded into
its activation pass and a residual-accumulating store), so the engine runs a decode step with
the same five launches per layer as the fused decode step:

1. SwiGLU. gate = MatMulNBits(h, Wg), up = MatMulNBits(h, Wu), silu = Mul(gate, Sigmoid(gate)),
   act = Mul(silu, up), y = MatMulNBits(act, Wd)  ->  gu = MatMulNBits(h, [Wg; Wu]) (one GEMV over
   the concatenated weights, rows [gate | up]), y = MatMulNBitsFused(gu, Wd, swiglu=1).
2. Norm into its consumers. SimplifiedLayerNormalization(x, g) whose output feeds only
   MatMulNBits nodes (as A)  ->  each of them MatMulNBitsFused(x, W, gamma=g).
3. Residual add into its producer. SkipSimplifiedLayerNormalization(a, skip, g) -> [h, -, -, s]
   where `a` comes from a MatMulNBits(-Fused) node P used only here and `h` feeds only
   MatMulNBits nodes  ->  P accumulates into `skip` in place (output s = skip + P's product)
   and the consumers of h become MatMulNBitsFused(s, W, gamma=g). In place only when every
   other reader of `skip` runs before P and `skip` is not a graph input, output or initializer.

A pattern whose conditions do not hold is left as it is. Values are not renamed: every value
the rest of the graph reads keeps its name and meaning.
"""
from __future__ import annotations

from collections import defaultdict

import torch

from .kernels import GraphNode, ModelGraph

_MNB = ("MatMulNBits", "MatMulNBitsFused")


def _consumers(nodes: list[GraphNode]) -> dict[str, list[int]]:
    c: dict[str, list[int]] = defaultdict(list)
    for i, n in enumerate(nodes):
        for v in n.inputs:
            if v:
                c[v].append(i)
    return c


def _producers(nodes: list[GraphNode]) -> dict[str, int]:
    return {o: i for i, n in enumerate(nodes) for o in n.outputs if o}


def _fused_from(node: GraphNode, a: str, *, gamma: str = "", residual: str = "", swiglu: int = 0,
                epsilon: float | None = None, out: str | None = None) -> GraphNode:
    """node (MatMulNBits or MatMulNBitsFused) with A = a and the given fusion fields added."""
    ins = list(node.inputs[:4]) + [""] * (4 - len(node.inputs[:4]))
    attrs = {k: node.attributes[k] for k in ("N", "K", "bits", "block_size") if k in node.attributes}
    if node.op_type == "MatMulNBitsFused":
        old = list(node.inputs) + [""] * (6 - len(node.inputs))
        gamma, residual = gamma or old[4], residual or old[5]
        swiglu = swiglu or int(node.attributes.get("swiglu", 0))
        if epsilon is None:
            epsilon = node.attributes.get("epsilon")
    attrs["swiglu"] = swiglu
    if epsilon is not None:
        attrs["epsilon"] = float(epsilon)
    ins[0] = a
    return GraphNode("MatMulNBitsFused", node.name, ins + [gamma, residual], [out or node.outputs[0]], attrs)


def _fuse_swiglu(g: ModelGraph) -> bool:
    nodes = g.nodes
    cons, prod = _consumers(nodes), _producers(nodes)
    for i, act_mul in enumerate(nodes):
        if act_mul.op_type != "Mul":
            continue
        down_users = cons.get(act_mul.outputs[0], [])
        if len(down_users) != 1 or nodes[down_users[0]].op_type != "MatMulNBits" \
                or nodes[down_users[0]].inputs[0] != act_mul.outputs[0]:
            continue
        for silu_name, up_name in (tuple(act_mul.inputs), tuple(reversed(act_mul.inputs))):
            si = prod.get(silu_name)
            up = prod.get(up_name)
            if si is None or up is None or nodes[si].op_type != "Mul" or nodes[up].op_type != "MatMulNBits":
                continue
            a, b = nodes[si].inputs
            for gate_name, sig_name in ((a, b), (b, a)):
                sg, gt = prod.get(sig_name), prod.get(gate_name)
                if sg is None or gt is None or nodes[sg].op_type != "Sigmoid" or nodes[sg].inputs[0] != gate_name \
                        or nodes[gt].op_type != "MatMulNBits":
                    continue
                gate, upn, down = nodes[gt], nodes[up], nodes[down_users[0]]
                same = all(gate.attributes.get(k) == upn.attributes.get(k) for k in ("K", "bits", "block_size"))
                if not same or gate.inputs[0] != upn.inputs[0] or gate.attributes.get("N") != upn.attributes.get("N") \
                        or int(down.attributes.get("K", -1)) != int(gate.attributes.get("N", -2)):
                    continue
                if len(gate.inputs) < 4 or len(upn.inputs) < 4 or not gate.inputs[3] or not upn.inputs[3]:
                    continue  # zero points on both, so the concatenated layout stays one packed tensor
                if sorted(cons[gate_name]) != sorted([sg, si]) or cons[up_name] != [i] \
                        or cons[sig_name] != [si] or cons[silu_name] != [i]:
                    continue
                base = gate.name + "+" + upn.name
                init = g.initializers
                init[base + ".B"] = torch.cat([torch.as_tensor(init[gate.inputs[1]]),
                                               torch.as_tensor(init[upn.inputs[1]])])
                init[base + ".scales"] = torch.cat([torch.as_tensor(init[gate.inputs[2]]).reshape(-1),
                                                    torch.as_tensor(init[upn.inputs[2]]).reshape(-1)])
                init[base + ".zero_points"] = torch.cat([torch.as_tensor(init[gate.inputs[3]]),
                                                         torch.as_tensor(init[upn.inputs[3]])])
                n = int(gate.attributes["N"])
                merged = GraphNode("MatMulNBits", base, [gate.inputs[0], base + ".B", base + ".scales",
                                                         base + ".zero_points"], [base],
                                   dict(gate.attributes, N=2 * n))
                fused_down = _fused_from(down, base, swiglu=1)
                drop = {gt, up, sg, si, i}
                out = []
                for j, n_ in enumerate(nodes):
                    if j == gt:
                        out.append(merged)
                    elif j == down_users[0]:
                        out.append(fused_down)
                    elif j not in drop:
                        out.append(n_)
                g.nodes = out
                return True
    return False


def _norm_consumers_ok(nodes, cons, h: str) -> bool:
    users = cons.get(h, [])
    return bool(users) and all(nodes[u].op_type in _MNB and nodes[u].inputs[0] == h
                               and int(nodes[u].attributes.get("swiglu", 0)) == 0
                               and not (nodes[u].op_type == "MatMulNBitsFused"
                                        and len(nodes[u].inputs) > 4 and nodes[u].inputs[4]) for u in users)


def _fuse_norm(g: ModelGraph) -> bool:
    nodes = g.nodes
    cons = _consumers(nodes)
    for i, n in enumerate(nodes):
        if n.op_type != "SimplifiedLayerNormalization" or len(n.outputs) > 1 and any(n.outputs[1:]):
            continue
        h = n.outputs[0]
        if h in g.outputs or not _norm_consumers_ok(nodes, cons, h):
            continue
        eps = n.attributes.get("epsilon", 1e-5)
        repl = {u: _fused_from(nodes[u], n.inputs[0], gamma=n.inputs[1], epsilon=eps) for u in cons[h]}
        g.nodes = [repl.get(j, m) for j, m in enumerate(nodes) if j != i]
        return True
    return False


def _fuse_skip_norm(g: ModelGraph) -> bool:
    nodes = g.nodes
    cons, prod = _consumers(nodes), _producers(nodes)
    protected = set(g.inputs) | set(g.outputs) | set(g.initializers)
    for i, n in enumerate(nodes):
        if n.op_type != "SkipSimplifiedLayerNormalization":
            continue
        ins = list(n.inputs) + [""] * (5 - len(n.inputs))
        outs = list(n.outputs) + [""] * (4 - len(n.outputs))
        if ins[3] or ins[4] or outs[1] or outs[2]:
            continue
        a, skip, gamma = ins[0], ins[1], ins[2]
        h, s = outs[0], outs[3] or (n.name + ".sum")
        for x, y in ((a, skip), (skip, a)):  # the sum is symmetric: either input may be the product
            p = prod.get(x)
            if p is None or nodes[p].op_type not in _MNB or cons.get(x) != [i] or nodes[p].outputs[0] != x:
                continue
            pn = nodes[p]
            if pn.op_type == "MatMulNBitsFused" and len(pn.inputs) > 5 and pn.inputs[5]:
                continue  # already accumulating
            if y in protected or prod.get(y, p) >= p or any(u > p for u in cons.get(y, []) if u != i):
                continue  # the residual must exist before the in-place add and have no later reader
            if h in g.outputs or not _norm_consumers_ok(nodes, cons, h):
                continue
            eps = n.attributes.get("epsilon", 1e-5)
            repl = {p: _fused_from(pn, pn.inputs[0], residual=y, out=s)}
            for u in cons[h]:
                repl[u] = _fused_from(nodes[u], s, gamma=gamma, epsilon=eps)
            g.nodes = [repl.get(j, m) for j, m in enumerate(nodes) if j != i]
            return True
    return False


def fuse_decode_graph(graph: ModelGraph) -> ModelGraph:
    """A copy of `graph` with the patterns above rewritten (initializers shared, merged gate/up
    weights added)."""
    g = ModelGraph(list(graph.inputs), list(graph.outputs), list(graph.nodes), dict(graph.initializers))
    while _fuse_swiglu(g):
        pass
    while _fuse_skip_norm(g) or _fuse_norm(g):
        pass
    return g
