"""CUDA MatMulNBits against the parity checker, through the C ABI (needs a B200).

Bars (north_star): rel-L2 <= 1e-5 for the fp32-accumulate kernels (generic, decode GEMV),
<= 5e-3 for the tensor-core GEMM; the reference's KATs within their own 1e-4 absolute.
"""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from modelsharp_b200 import CudaEngine, GraphNode, KernelRegistry, ModelGraph, QuantizedWeights, synth
from modelsharp_b200 import _native as N
from modelsharp_b200.errors import ModelSharpException
from oracle import oracle
from tests.golden import cases
from tests.test_oracle import GOLD, KATS, META, golden_case, kat_case

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5   # rel-L2, fp32-accumulate paths
TOL_TC = 5e-3     # rel-L2, fp16 tensor-core GEMM


def fast_ok(c) -> bool:
    bs = c["block_size"]
    return c["bits"] == 4 and bs >= 32 and (bs & (bs - 1)) == 0


def pack(c, dev, generic_only=False, rows=None):
    return QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], c["bits"], c["block_size"],
                            rows=rows, device=dev, generic_only=generic_only)


def run(c, dev, path=N.PATH_AUTO, generic_only=False, a=None):
    w = pack(c, dev, generic_only)
    a_t = torch.from_numpy(np.ascontiguousarray(c["a"] if a is None else a)).to(dev)
    y = w.matmul(a_t.reshape(-1, c["K"]), path=path)
    torch.cuda.synchronize(dev)
    return y.cpu().numpy()


def test_library_loaded_on_device(cuda_device):
    assert N.available()
    assert N.library_path().exists()


@pytest.mark.parametrize("k", KATS["cases"], ids=[k["name"] for k in KATS["cases"]])
def test_known_answers_through_engine(cuda_device, k):
    """The reference's KATs, one MatMulNBits node run by the engine on the CUDA registry."""
    c = kat_case(k)
    inputs = ["A", "B", "scales"] + (["zp"] if c["zp"] is not None else [])
    inits = {"B": c["b"].reshape(k["b_shape"]), "scales": c["scales"]}
    if c["zp"] is not None:
        inits["zp"] = c["zp"]
    g = ModelGraph(["A"], ["Y"], [GraphNode("MatMulNBits", "n", inputs, ["Y"],
                                            {"N": k["N"], "K": k["K"], "bits": k["bits"],
                                             "block_size": k["block_size"]})], inits)
    a = torch.from_numpy(c["a"]).to(cuda_device)
    y = CudaEngine(g).run({"A": a})["Y"]
    assert list(y.shape) == k["y_shape"]
    assert y.is_cuda
    np.testing.assert_allclose(y.cpu().numpy().reshape(-1), np.array(k["expected"], np.float32), rtol=0,
                               atol=KATS["tolerance_abs"])
    # the same node with a host A goes through the host-buffer entry point
    y_host = CudaEngine(g).run({"A": c["a"]})["Y"]
    np.testing.assert_allclose(y_host.numpy().reshape(-1), np.array(k["expected"], np.float32), rtol=0,
                               atol=KATS["tolerance_abs"])


@pytest.mark.parametrize("e", META["cases"], ids=[e["key"] for e in META["cases"]])
def test_golden_generic(cuda_device, e):
    c = golden_case(e["key"])
    ref = np.load(GOLD / "ref_native.npz")[e["key"]]
    y = run(c, cuda_device, N.PATH_GENERIC, generic_only=True)
    assert N.last_path() == "generic"
    assert oracle.rel_l2(y, ref) <= TOL_FP32
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


@pytest.mark.parametrize("e", [e for e in META["cases"] if fast_ok(e)], ids=lambda e: e["key"])
def test_golden_gemv(cuda_device, e):
    c = golden_case(e["key"])
    ref = np.load(GOLD / "ref_native.npz")[e["key"]]
    y = run(c, cuda_device, N.PATH_GEMV)
    assert N.last_path().startswith("gemv_")
    assert oracle.rel_l2(y, ref) <= TOL_FP32
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 11, 16])
@pytest.mark.parametrize("i", range(len(cases.BASELINE_GEMV)), ids=[b[0] for b in cases.BASELINE_GEMV])
def test_decode_shapes_batched(cuda_device, i, M):
    """Baseline decode shapes (Qwen up-proj, the 7B sweep) at every decode batch size."""
    c = cases.baseline_case(i, M=M)
    y = run(c, cuda_device)
    assert N.last_path().startswith("gemv_")
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


@pytest.mark.parametrize("zp_kind", ["none", "packed", "float"])
@pytest.mark.parametrize("K,bs", [(1000, 32), (4096, 64), (4160, 128), (96, 32), (8192, 256)])
def test_gemv_zero_point_forms_and_ragged_k(cuda_device, zp_kind, K, bs):
    c = synth.make_case(77, 3, 777, K, 4, bs, zp_kind)
    y = run(c, cuda_device, N.PATH_GEMV)
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32
    yg = run(c, cuda_device, N.PATH_GENERIC, generic_only=True)
    assert oracle.rel_l2(yg, oracle.managed(c)) <= TOL_FP32


@pytest.mark.parametrize("a_dtype,s_dtype", [("f16", "f32"), ("f32", "f16"), ("f16", "f16")])
def test_half_inputs_are_widened_exactly(cuda_device, a_dtype, s_dtype):
    c = synth.make_case(5, 4, 1024, 4096, 4, 32, "packed", a_dtype=a_dtype, scale_dtype=s_dtype,
                        scale_lo=0.001, scale_hi=0.01)
    ref = oracle.managed(c)  # the oracle widens fp16 exactly, as GraphContext.Get does
    assert oracle.rel_l2(run(c, cuda_device, N.PATH_GEMV), ref) <= TOL_FP32
    assert oracle.rel_l2(run(c, cuda_device, N.PATH_GENERIC, generic_only=True), ref) <= TOL_FP32


def test_bf16_activations(cuda_device):
    c = synth.make_case(6, 2, 512, 2048, 4, 128, "packed")
    a16 = torch.from_numpy(c["a"]).to(torch.bfloat16)
    c_ref = dict(c, a=a16.float().numpy())
    w = pack(c, cuda_device)
    y = w.matmul(a16.to(cuda_device)).cpu().numpy()
    assert oracle.rel_l2(y, oracle.managed(c_ref)) <= TOL_FP32


def test_row_shard_writes_into_wide_output(cuda_device):
    """A column shard (rows [n0, n1)) writes Y[:, n0:n1] of a wider buffer via ldy, and nothing else."""
    c = synth.make_case(8, 3, 1000, 2048, 4, 128, "packed")
    full = oracle.managed(c)
    y = torch.full((3, 1000 + 16), float("nan"), device=cuda_device)
    a = torch.from_numpy(c["a"]).to(cuda_device)
    for n0, n1 in ((0, 250), (250, 600), (600, 1000)):
        w = pack(c, cuda_device, rows=(n0, n1))
        w.matmul(a, out=y[:, n0:n1], ldy=y.stride(0))
    torch.cuda.synchronize()
    out = y.cpu().numpy()
    assert np.isnan(out[:, 1000:]).all(), "write past the shard"
    assert oracle.rel_l2(out[:, :1000], full) <= TOL_FP32


def test_output_canaries(cuda_device):
    c = synth.make_case(9, 5, 300, 896, 4, 32, "packed")
    w = pack(c, cuda_device)
    buf = torch.full((5 * 300 + 64,), float("nan"), device=cuda_device)
    a = torch.from_numpy(c["a"]).to(cuda_device)
    w.matmul(a, out=buf[:1500].view(5, 300), ldy=300)
    torch.cuda.synchronize()
    assert torch.isnan(buf[1500:]).all()
    assert not torch.isnan(buf[:1500]).any()


def test_host_buffer_async_entry_matches_the_synchronous_one(cuda_device):
    """msq_matmul_host_async enqueues upload, op and download without waiting: three ops on one
    stream, one synchronize, the same bits as msq_matmul_host gives op by op (fp32 and fp16 A,
    the decode GEMV, the tensor-core batched GEMV and the GEMM)."""
    cs = [synth.make_case(12, 1, 640, 1024, 4, 32, "packed"),
          synth.make_case(13, 8, 300, 1024, 4, 128, "packed", a_dtype="f16", scale_dtype="f16"),
          synth.make_case(14, 40, 256, 512, 4, 64, "float")]
    ws = [pack(c, cuda_device) for c in cs]
    want = [w.matmul_host(c["a"]) for w, c in zip(ws, cs)]
    a_h = [torch.from_numpy(np.ascontiguousarray(c["a"])).pin_memory() for c in cs]
    y_h = [torch.full((c["M"], c["N"]), float("nan")).pin_memory() for c in cs]
    st = torch.cuda.Stream(cuda_device)
    for w, a, y in zip(ws, a_h, y_h):
        rc = N.lib().msq_matmul_host_async(None, st.cuda_stream, w.handle, a.data_ptr(),
                                           N.DT_F16 if a.dtype == torch.float16 else N.DT_F32, a.shape[0], y.data_ptr())
        assert rc == N.MSQ_OK, N.last_error()
    st.synchronize()
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK
    for y, yw, c in zip(y_h, want, cs):
        assert np.array_equal(y.numpy(), yw)
    rc = N.lib().msq_matmul_host_async(None, st.cuda_stream, ws[0].handle, None, N.DT_F32, 1, y_h[0].data_ptr())
    assert rc == N.MSQ_E_INVALID and "NULL host pointer" in N.last_error()
    for w in ws:
        w.free()


def test_host_buffer_entry_and_one_shot(cuda_device):
    c = synth.make_case(10, 2, 640, 1024, 4, 32, "packed")
    ref = oracle.managed(c)
    w = pack(c, cuda_device)
    assert oracle.rel_l2(w.matmul_host(c["a"]), ref) <= TOL_FP32
    y = np.empty((2, 640), np.float32)
    a = np.ascontiguousarray(c["a"])
    rc = N.lib().msq_qgemm_nbits(a.ctypes.data, c["b"].ctypes.data, c["scales"].ctypes.data, c["zp"].ctypes.data,
                                 y.ctypes.data, 2, 640, 1024, 4, 32)
    assert rc == N.MSQ_OK
    assert oracle.rel_l2(y, ref) <= TOL_FP32
    c8 = synth.make_case(11, 3, 100, 300, 8, 16, "none")
    y8 = np.empty((3, 100), np.float32)
    rc = N.lib().msq_qgemm_nbits(c8["a"].ctypes.data, c8["b"].ctypes.data, c8["scales"].ctypes.data, None,
                                 y8.ctypes.data, 3, 100, 300, 8, 16)
    assert rc == N.MSQ_OK
    assert oracle.rel_l2(y8, oracle.managed(c8)) <= TOL_FP32


def test_pack_from_device_buffers(cuda_device):
    c = synth.make_case(12, 1, 512, 4096, 4, 128, "packed")
    dev = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(cuda_device) for k in ("b", "scales", "zp")}
    w = QuantizedWeights(dev["b"], dev["scales"], dev["zp"], 512, 4096, 4, 128, device=cuda_device)
    y = w.matmul(torch.from_numpy(c["a"]).to(cuda_device)).cpu().numpy()
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


def test_empty_a_and_errors(cuda_device):
    c = synth.make_case(13, 1, 64, 256, 4, 32, "none")
    w = pack(c, cuda_device)
    y = w.matmul(torch.empty(0, 256, device=cuda_device))
    assert y.shape == (0, 64)
    with pytest.raises(ModelSharpException, match="A inner dimension must equal K=256"):
        w.matmul(torch.zeros(2, 255, device=cuda_device))
    with pytest.raises(ModelSharpException, match="A must be Float32 or Float16"):
        w.matmul(torch.zeros(2, 256, dtype=torch.int32, device=cuda_device))


def test_registry_replaces_by_op_type(cuda_device):
    r = KernelRegistry.create_default()
    ok, k = r.try_get("MatMulNBits")
    assert ok and k.op_type == "MatMulNBits" and r.count == 1


def test_no_kernel_gave_up_a_wait(cuda_device):
    """Every bounded wait in the pipelined kernels completed during the parity runs above."""
    c = cases.baseline_case(1)
    run(c, cuda_device)
    rc = N.lib().msq_device_status(None, None)
    assert rc == N.MSQ_OK, N.last_error()


@pytest.mark.parametrize("N_", [1, 7, 33, 150, 1000, 5000])
def test_stream_row_blocks_any_height(cuda_device, N_):
    """The row-block height adapts to N (1..32 rows per block); partial last blocks and
    single-row handles must produce every row exactly once."""
    c = synth.make_case(14, 1, N_, 2048, 4, 128, "packed")
    y = run(c, cuda_device, N.PATH_GEMV)
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


@pytest.mark.parametrize("N_,K,bs,zp", [(1000, 4160, 128, "packed"), (384, 2048, 32, "float"), (256, 1024, 64, "none"),
                                        (4096, 4096, 128, "packed")])
def test_lazy_gemm_layout_holds_one_copy_and_matches(cuda_device, N_, K, bs, zp):
    """MSQ_PACK_LAZY_GEMM: the handle holds the decode stream only (<= 1.1x the reference's
    bytes), decodes exactly as before, and the GEMM layout it derives from the stream at its
    first GEMM call gives the eagerly packed handle's GEMM output bit for bit."""
    c = synth.make_case(44, 64, N_, K, 4, bs, zp, scale_lo=0.001, scale_hi=0.01)
    lazy = QuantizedWeights(c["b"], c["scales"], c["zp"], N_, K, 4, bs, device=cuda_device, lazy_gemm=True)
    eager = pack(c, cuda_device)
    alg = synth.algorithmic_bytes(N_, K, 4, bs, zp)
    assert lazy.query_device_bytes() <= 1.1 * alg, (lazy.query_device_bytes(), alg)
    assert eager.query_device_bytes() > 1.5 * alg
    a = torch.from_numpy(c["a"]).to(cuda_device)
    y1 = lazy.matmul(a[:1])
    assert N.last_path() == "gemv_imma"
    assert torch.equal(y1, eager.matmul(a[:1]))
    # the no-allocation entry refuses the handle before its GEMM layout exists
    yy = torch.empty(64, N_, device=cuda_device)
    with torch.cuda.device(cuda_device):
        rc = N.lib().msq_matmul_noalloc(None, torch.cuda.current_stream(cuda_device).cuda_stream, lazy.handle,
                                        a.data_ptr(), N.DT_F32, 64, yy.data_ptr(), N_)
    assert rc == N.MSQ_E_UNSUPPORTED and "LAZY_GEMM" in N.last_error()
    if bs == 128:  # the tensor-core batched GEMV reads the derived planes too
        assert torch.equal(lazy.matmul(a[:16], path=N.PATH_GEMV_TC), eager.matmul(a[:16], path=N.PATH_GEMV_TC))
    for path in (N.PATH_GEMM, N.PATH_GEMM_SPLIT):
        assert torch.equal(lazy.matmul(a, path=path), eager.matmul(a, path=path))
    torch.cuda.synchronize()
    assert lazy.query_device_bytes() == eager.query_device_bytes()
    assert oracle.rel_l2(lazy.matmul(a).cpu().numpy(), oracle.managed(c)) <= TOL_TC
    lazy.free()
    eager.free()

