"""ONNX loading (modelsharp_b200.onnx_loader) against models written by tests/onnx_model.py.

CPU: the parsed graph's nodes, attributes and initializers equal what was written, for inline
raw data, external data (memory-mapped, with offsets), int32_data-packed and bfloat16 tensors,
and the reference loader's errors (no graph, unresolvable external data). GPU: a MatMulNBits
model whose weights live in an external-data file is packed at load (CudaEngine preload) and
its run matches the parity checker at the GEMV bar (rel-L2 <= 1e-5).
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import synth
from modelsharp_b200.errors import ModelSharpException
from modelsharp_b200.onnx_loader import load_model, parse_model
from tests import onnx_model as om


def _case(zp="packed"):
    return synth.make_case(91, 2, 200, 256, 4, 32, zp, scale_dtype="f16")


def test_inline_model_round_trip():
    c = _case()
    g = parse_model(om.matmulnbits_model(c))
    assert g.inputs == ["A"] and g.outputs == ["Y"]  # initializers are not feeds
    (n,) = g.nodes
    assert (n.op_type, n.name, n.inputs, n.outputs) == ("MatMulNBits", "mnb", ["A", "B", "scales", "zp"], ["Y"])
    assert n.attributes == {"K": 256, "N": 200, "bits": 4, "block_size": 32}
    np.testing.assert_array_equal(g.initializers["B"], c["b"])
    assert g.initializers["scales"].dtype == np.float16
    np.testing.assert_array_equal(g.initializers["scales"].reshape(-1), np.asarray(c["scales"]).reshape(-1))
    np.testing.assert_array_equal(g.initializers["zp"], c["zp"])


def test_external_data_is_memory_mapped(tmp_path):
    c = _case("none")
    (tmp_path / "m.onnx").write_bytes(om.matmulnbits_model(c, ext_dir=tmp_path))
    g = load_model(tmp_path / "m.onnx")
    np.testing.assert_array_equal(g.initializers["B"], c["b"])
    np.testing.assert_array_equal(g.initializers["scales"].reshape(-1), np.asarray(c["scales"]).reshape(-1))
    assert not g.initializers["B"].flags.writeable  # a view of the mapping, not a copy
    with pytest.raises(ModelSharpException, match="in-memory byte buffer"):
        parse_model((tmp_path / "m.onnx").read_bytes())
    (tmp_path / "weights.bin").unlink()
    with pytest.raises(ModelSharpException, match="was not found"):
        load_model(tmp_path / "m.onnx")


def test_typed_fields_and_bfloat16():
    i8 = np.arange(-5, 5, dtype=np.int8)
    h = np.asarray([1.5, -2.25, 65504.0], dtype=np.float16)
    bf = np.asarray([1.0, -3.5, 2.0 ** 100], dtype=np.float32)
    bf_bits = (bf.view(np.uint32) >> 16).astype(np.uint16)
    raw_bf = om._vi(1, 3) + om._vi(2, 16) + om._str(8, "bf") + om._ld(9, bf_bits.tobytes())
    floats = om._vi(1, 2) + om._vi(2, 1) + om._str(8, "f") + om._key(4, 5) + np.float32(0.5).tobytes() + \
        om._key(4, 5) + np.float32(-1.0).tobytes()
    m = om.model([om.node("Identity", ["x"], ["y"], attrs=[om.attr_ints("perm", [1, 0]), om.attr_float("alpha", 0.25)])],
                 [om.tensor("i8", i8, as_int32_data=True), om.tensor("h", h, as_int32_data=True), raw_bf, floats],
                 ["x"], ["y"])
    g = parse_model(m)
    np.testing.assert_array_equal(g.initializers["i8"], i8)
    np.testing.assert_array_equal(g.initializers["h"], h)
    np.testing.assert_array_equal(g.initializers["bf"], bf)
    np.testing.assert_array_equal(g.initializers["f"], np.asarray([0.5, -1.0], np.float32))
    assert g.nodes[0].name == "Identity" and g.nodes[0].attributes == {"perm": [1, 0], "alpha": 0.25}


def test_model_without_graph_is_rejected():
    with pytest.raises(ModelSharpException, match=r"no graph \(field 7\)"):
        parse_model(om._vi(1, 8))


def test_declared_size_beyond_data_is_rejected():
    t = om._vi(1, 1 << 20) + om._vi(2, 2) + om._str(8, "big") + om._ld(9, b"\1\2\3")
    with pytest.raises(ModelSharpException, match="declares"):
        parse_model(om.model([], [t], [], []))


@pytest.mark.gpu
def test_external_weights_packed_at_load_and_run(cuda_device, native_lib, tmp_path):
    from modelsharp_b200 import CudaEngine
    from modelsharp_b200 import _native as N
    from oracle import oracle

    c = synth.make_case(92, 3, 1000, 1024, 4, 32, "packed", scale_dtype="f16", scale_lo=0.001, scale_hi=0.01)
    (tmp_path / "m.onnx").write_bytes(om.matmulnbits_model(c, ext_dir=tmp_path))
    g = load_model(tmp_path / "m.onnx")
    eng = CudaEngine(g, device=cuda_device, preload=True)
    assert eng.preloaded == 1
    launches = N.launch_count()
    a = torch.from_numpy(c["a"]).to(cuda_device)
    y = eng.run({"A": a})["Y"]
    y2 = eng.run({"A": a})["Y"]
    torch.cuda.synchronize(cuda_device)
    ok, k = eng.kernels.try_get("MatMulNBits")
    assert len(k._cache) == 1  # packed once, at load; the runs reused it
    assert N.launch_count() > launches
    ref = oracle.managed(dict(c, scales=np.asarray(c["scales"], np.float32)))
    assert oracle.rel_l2(y.cpu().numpy(), ref) <= 1e-5
    assert torch.equal(y, y2)
