"""Host logic of the operator API that needs no GPU: registry and engine contract
(KernelRegistry.cs:20-33, ManagedCpuEngine.cs:36-84) and the MatMulNBits node's validation,
which must raise the reference's messages before any device work."""
import numpy as np
import pytest

from modelsharp_b200 import CudaEngine, GraphNode, KernelRegistry, ModelGraph, ModelSharpException
from modelsharp_b200.engine import UnsupportedOperatorException
from modelsharp_b200.kernels import GraphContext


class _Echo:
    op_type = "Identity"

    def execute(self, node, ctx):
        ctx.set(node.outputs[0], ctx.get_tensor(node.inputs[0]))


class _Echo2(_Echo):
    pass


def test_registry_register_replaces_by_op_type():
    r = KernelRegistry().register(_Echo())
    assert r.count == 1
    r.register(_Echo2())
    ok, k = r.try_get("Identity")
    assert ok and isinstance(k, _Echo2) and r.count == 1
    assert r.try_get("Nope") == (False, None)


def test_default_registry_holds_matmulnbits(native_lib):
    ok, k = KernelRegistry.create_default().try_get("MatMulNBits")
    assert ok and k.op_type == "MatMulNBits"


def test_engine_contract(native_lib):
    g = ModelGraph(["x"], ["y"], [GraphNode("Identity", "id", ["x"], ["y"])])
    eng = CudaEngine(g, KernelRegistry().register(_Echo()))
    assert eng.run({"x": 3})["y"] == 3
    with pytest.raises(ModelSharpException, match="Missing feed for required input 'x'."):
        eng.run({})
    g2 = ModelGraph(["x"], ["y"], [GraphNode("Conv", "c0", ["x"], ["y"])])
    with pytest.raises(UnsupportedOperatorException, match="Conv"):
        CudaEngine(g2, KernelRegistry()).run({"x": 1})


def test_context_semantics():
    ctx = GraphContext({"a": np.zeros(2, np.float32)})
    assert ctx.has("a") and not ctx.has("") and not ctx.has("b")
    with pytest.raises(ModelSharpException, match="Tensor 'b' is not available in the execution context."):
        ctx.get_tensor("b")


def _node_graph(attrs, b, scales, zp=None, g_idx=None):
    inputs = ["A", "B", "scales"]
    inits = {"B": b, "scales": scales}
    if zp is not None or g_idx is not None:
        inputs.append("zp" if zp is not None else "")
        if zp is not None:
            inits["zp"] = zp
    if g_idx is not None:
        inputs.append("g_idx")
        inits["g_idx"] = g_idx
    return ModelGraph(["A"], ["Y"], [GraphNode("MatMulNBits", "n", inputs, ["Y"], attrs)], inits)


@pytest.mark.parametrize("attrs,b_len,s_len,msg", [
    ({"N": 2, "K": 4, "block_size": 4}, 3, 2, "MatMulNBits B has 3 elements; expected 4"),
    ({"N": 2, "K": 4, "bits": 2, "block_size": 4}, 4, 2, "MatMulNBits supports bits=4 or bits=8; got 2."),
    ({"N": 2, "K": 4}, 4, 2, "MatMulNBits requires a positive block_size; got 0."),
    ({"K": 4, "block_size": 4}, 4, 2, "MatMulNBits requires positive N and K attributes (got N=0, K=4)."),
    ({"N": 2, "K": 4, "block_size": 4}, 4, 1, "MatMulNBits scales has 1 elements; expected 2"),
])
def test_node_validation_before_device_work(native_lib, attrs, b_len, s_len, msg):
    g = _node_graph(attrs, np.zeros(b_len, np.uint8), np.ones(s_len, np.float32))
    with pytest.raises(ModelSharpException) as ei:
        CudaEngine(g).run({"A": np.zeros((1, 4), np.float32)})
    assert msg in str(ei.value)


def test_node_rejects_non_uint8_b_and_bad_g_idx(native_lib):
    g = _node_graph({"N": 2, "K": 4, "block_size": 4}, np.zeros(4, np.int8), np.ones(2, np.float32))
    with pytest.raises(ModelSharpException, match="Tensor dtype is Int8; expected UInt8."):
        CudaEngine(g).run({"A": np.zeros((1, 4), np.float32)})
    g = _node_graph({"N": 2, "K": 8, "block_size": 4}, np.zeros(8, np.uint8), np.ones(4, np.float32),
                    g_idx=np.array([0, 0, 0, 0, 1, 1, 1, 0], np.int64))
    with pytest.raises(ModelSharpException, match="non-trivial block permutation"):
        CudaEngine(g).run({"A": np.zeros((1, 8), np.float32)})
    g = _node_graph({"N": 2, "K": 8, "block_size": 4}, np.zeros(8, np.uint8), np.ones(4, np.float32))
    with pytest.raises(ModelSharpException, match=r"A inner dimension must equal K=8; got shape \[1,7\]."):
        CudaEngine(g).run({"A": np.zeros((1, 7), np.float32)})
