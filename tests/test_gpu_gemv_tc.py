"""The batched decode GEMV on tcgen05 kind::i8 (MSQ_PATH_GEMV_TC), against the checker (needs a B200).

The decode GEMV's exact integer scheme (24-bit fixed-point activations as three int8 digits,
u8 codes, per-block scale and zero-point terms in fp32) with the tensor core doing every
multiply-add and each weight read once for all rows of A: the same bar as the decode GEMV,
rel-L2 <= 1e-5 against the reference's fp32 MatMulNBits (MatMulNBitsKernel.cs:236-261).
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import QuantizedWeights, synth
from modelsharp_b200 import _native as N
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5


def _run(c, dev, a=None):
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, c["block_size"], device=dev)
    a = c["a"] if a is None else a
    at = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))
    y = w.matmul(at.to(dev), path=N.PATH_GEMV_TC)
    torch.cuda.synchronize(dev)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    path = N.last_path()
    w.free()
    return y.float().cpu().numpy(), path


@pytest.mark.parametrize("M", [1, 5, 8, 16, 17, 24, 32])
def test_tc_gemv_rows(cuda_device, M):
    c = synth.make_case(80 + M, M, 700, 4096, 4, 128, "packed", scale_lo=0.001, scale_hi=0.01)
    y, path = _run(c, cuda_device)
    assert path.startswith("gemv_tc_i8")
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


@pytest.mark.parametrize("zp", ["none", "float", "packed"])
def test_tc_gemv_zero_point_forms_and_ragged_k(cuda_device, zp):
    c = synth.make_case(90, 12, 300, 1000, 4, 128, zp, scale_lo=0.001, scale_hi=0.01)
    y, _ = _run(c, cuda_device)
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


def test_tc_gemv_half_activations(cuda_device):
    c = synth.make_case(91, 9, 520, 2048, 4, 128, "packed", a_dtype="f16", scale_dtype="f16",
                        scale_lo=0.001, scale_hi=0.01)
    y, _ = _run(c, cuda_device)
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32
    # bf16 A: the kernel widens each value exactly; the checker sees the same widened values
    ab = torch.from_numpy(c["a"].astype(np.float32)).to(torch.bfloat16)
    cb = dict(c, a=ab.float().numpy())
    y, _ = _run(cb, cuda_device, a=ab)
    assert oracle.rel_l2(y, oracle.managed(cb)) <= TOL_FP32


def test_tc_gemv_k_split(cuda_device):
    """One 256-row tile over a long K: the blocks are split across CTAs and the partial outputs
    summed in split order."""
    c = synth.make_case(92, 32, 256, 28672, 4, 128, "packed", a_dtype="f16", scale_dtype="f16",
                        scale_lo=0.001, scale_hi=0.01)
    y, path = _run(c, cuda_device)
    assert path == "gemv_tc_i8_ksplit"
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32
    y2, _ = _run(c, cuda_device)
    assert np.array_equal(y, y2)  # fixed summation order: the same bits run to run


def test_tc_gemv_nonfinite_activations(cuda_device):
    c = synth.make_case(93, 6, 300, 1024, 4, 128, "packed", scale_lo=0.001, scale_hi=0.01)
    a = c["a"].copy()
    a[0, 5] = np.inf
    a[1, 700] = np.nan
    a[2, 3] = np.inf
    a[2, 1023] = -np.inf
    c = dict(c, a=a)
    y, _ = _run(c, cuda_device)
    ref = oracle.managed(c)
    for f in (np.isnan, np.isposinf, np.isneginf):
        assert np.array_equal(f(y), f(ref)), f.__name__
    fin = np.isfinite(ref)
    assert oracle.rel_l2(y[fin], ref[fin]) <= TOL_FP32


@pytest.mark.parametrize("K", [1024, 28672])  # one CTA per tile, and the k split
def test_tc_gemv_writes_only_its_columns(cuda_device, K):
    """A shard's Y written into a wider row (ldy > N, as the column split does): the columns
    outside [200, 200 + N) keep their contents, on the direct store and the split sum."""
    c = synth.make_case(94, 12, 300, K, 4, 128, "packed", scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, 128, device=cuda_device)
    buf = torch.full((12, 640), float("nan"), device=cuda_device)
    w.matmul(torch.from_numpy(c["a"]).to(cuda_device), out=buf[:, 200:500], ldy=640, path=N.PATH_GEMV_TC)
    torch.cuda.synchronize(cuda_device)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    y = buf.cpu().numpy()
    assert np.isnan(y[:, :200]).all() and np.isnan(y[:, 500:]).all()
    assert oracle.rel_l2(y[:, 200:500], oracle.managed(c)) <= TOL_FP32
    w.free()
