"""Parity at the north_star's own shapes, and A values outside the usual range (needs a B200).

* the 70B-shaped MLP layers (K=8192, N=28672) and (K=28672, N=8192), block_size 128,
  fp16 A and scales, packed zero points, at M = 1 (decode GEMV, rel-L2 <= 1e-5), 32 (the
  tensor-core decode GEMV, rel-L2 <= 1e-5, and the GEMM) and 1024 (tensor-core GEMM, rel-L2 <=
  5e-3; M = 1024 on sampled rows, rows being independent).
* configs[2] at M = 8192 on sampled rows.
* Infinity and NaN in A propagate as in the reference's fp32 sum (MatMulNBitsKernel.cs:236-261):
  an output is NaN, +inf or -inf exactly where the checker's is, on the GEMV and the GEMM;
  the other outputs stay within the path's bar.
* fp32 A beyond fp16's range (|a| up to 1e30) or below its normal range (1e-20) on the GEMM:
  the staging scales each row by a power of two, so nothing overflows or flushes.
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import QuantizedWeights, synth
from modelsharp_b200 import _native as N
from oracle import decoder as od
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5
TOL_TC = 5e-3


def _weights(c, dev):
    return QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, c["block_size"], device=dev)


def _mm(w, a, dev, path=N.PATH_AUTO):
    y = w.matmul(torch.from_numpy(np.ascontiguousarray(a)).to(dev), path=path)
    torch.cuda.synchronize(dev)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    return y.cpu().numpy()


def _sampled(c, y, rows):
    ref = np.concatenate([oracle.managed(c, rows=r) for r in rows], axis=0)
    got = np.concatenate([y[r] for r in rows], axis=0)
    return got, ref


@pytest.mark.parametrize("K,N_", [(8192, 28672), (28672, 8192)], ids=["up", "down"])
def test_70b_layers_at_configs3_row_counts(cuda_device, K, N_):
    c = synth.make_case(70, 1024, N_, K, 4, 128, "packed", a_dtype="f16", scale_dtype="f16",
                        scale_lo=0.001, scale_hi=0.01)
    w = _weights(c, cuda_device)
    a = c["a"]
    # M = 1: decode GEMV
    c1 = dict(c, a=a[:1], M=1)
    y1 = _mm(w, a[:1], cuda_device)
    assert N.last_path() == "gemv_imma"
    assert oracle.rel_l2(y1, oracle.managed(c1)) <= TOL_FP32
    # M = 32: the tensor-core decode GEMV (exact; k split across CTAs at this size), and the
    # fp16 GEMM when asked for it
    c32 = dict(c, a=a[:32], M=32)
    ref32 = oracle.managed(c32)
    y32 = _mm(w, a[:32], cuda_device)
    assert N.last_path().startswith("gemv_tc_i8")
    assert oracle.rel_l2(y32, ref32) <= TOL_FP32
    y32 = _mm(w, a[:32], cuda_device, path=N.PATH_GEMM)
    assert N.last_path().startswith("gemm_tc")
    assert oracle.rel_l2(y32, ref32) <= TOL_TC
    # M = 1024: the GEMM, sampled rows
    y = _mm(w, a, cuda_device)
    assert N.last_path().startswith("gemm_tc")
    got, ref = _sampled(c, y, [slice(0, 16), slice(500, 516), slice(1008, 1024)])
    assert oracle.rel_l2(got, ref) <= TOL_TC
    w.free()


def test_prefill_config_m8192_sampled_rows(cuda_device):
    M = 8192
    c = synth.make_case(3, M, 14336, 4096, 4, 32, "packed", a_dtype="f16", scale_dtype="f16",
                        scale_lo=0.001, scale_hi=0.01)
    w = _weights(c, cuda_device)
    y = _mm(w, c["a"], cuda_device)
    assert N.last_path() == "gemm_tc_m384_n128"  # 2464 three-accumulator tiles: 17 waves (1792 of four: 13)
    got, ref = _sampled(c, y, [slice(0, 16), slice(4090, 4106), slice(M - 16, M)])
    assert oracle.rel_l2(got, ref) <= TOL_TC
    w.free()


@pytest.mark.parametrize("M,N_,K,bs", [(1, 4096, 14336, 128), (3, 4096, 14336, 128), (1, 1000, 8960, 32),
                                        (4, 700, 8960, 64), (6, 300, 8960, 32)])
def test_gemv_tiles_of_fewer_than_32_units(cuda_device, M, N_, K, bs):
    """Stream tiles of 28 k-units (K = 14336 at block_size 128, 8960 at 32 / 64), whose units
    each warp takes by its index along the whole row (w mod 16), so the count per warp differs
    from tile to tile: the plain and fused decode GEMV against the checker."""
    c = synth.make_case(75, M, N_, K, 4, bs, "packed", scale_lo=0.001, scale_hi=0.01)
    w = _weights(c, cuda_device)
    y = _mm(w, c["a"], cuda_device, path=N.PATH_GEMV)
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32
    gamma = np.random.default_rng(5).uniform(0.8, 1.2, K).astype(np.float32)
    yf = torch.zeros(M, N_, device=cuda_device)
    w.matmul_fused(torch.from_numpy(c["a"]).to(cuda_device), yf, rms_gamma=torch.from_numpy(gamma).to(cuda_device),
                   rms_eps=1e-5)
    torch.cuda.synchronize(cuda_device)
    ref = oracle.managed(dict(c, a=od.rms_norm(c["a"], gamma, 1e-5)))
    assert oracle.rel_l2(yf.cpu().numpy(), ref) <= TOL_FP32
    w.free()


def _classes_match(y, ref):
    for f in (np.isnan, np.isposinf, np.isneginf):
        assert np.array_equal(f(y), f(ref)), f.__name__


def _nonfinite_case(M, N_, K, bs, zp, seed):
    c = synth.make_case(seed, M, N_, K, 4, bs, zp, scale_lo=0.001, scale_hi=0.01)
    a = c["a"].copy()
    a[0, 5] = np.inf             # row 0: +inf, outputs +inf / -inf by the weight's sign, NaN where q == zp
    if M > 1:
        a[1, K // 2] = np.nan    # row 1: NaN everywhere
    if M > 2:
        a[2, 3] = np.inf         # row 2: +inf and -inf in two blocks
        a[2, K - 1] = -np.inf
    return dict(c, a=a)


@pytest.mark.parametrize("M,bs,zp", [(1, 128, "packed"), (3, 32, "float"), (4, 64, "none")])
def test_gemv_nonfinite_activations_propagate(cuda_device, M, bs, zp):
    c = _nonfinite_case(M, 300, 1024, bs, zp, 71)
    w = _weights(c, cuda_device)
    y = _mm(w, c["a"], cuda_device, path=N.PATH_GEMV)
    ref = oracle.managed(c)
    _classes_match(y, ref)
    assert np.isinf(ref[0]).any()
    fin = np.isfinite(ref)
    assert oracle.rel_l2(y[fin], ref[fin]) <= TOL_FP32
    # finite rows of the same launch are untouched by the slow path
    clean = dict(c, a=synth.make_case(71, M, 300, 1024, 4, bs, zp)["a"])
    assert oracle.rel_l2(_mm(w, clean["a"], cuda_device, path=N.PATH_GEMV), oracle.managed(clean)) <= TOL_FP32
    w.free()


@pytest.mark.parametrize("M,bs,K", [(1, 32, 8960), (3, 128, 14336)])
def test_gemv_rows_over_several_stream_tiles(cuda_device, M, bs, K):
    """Rows of A that span several stream tiles (K = 8960 at block_size 32 is five k-tiles,
    14336 at 128 four), with magnitudes that differ by 1e6 from one part of the row to the
    next and inf / NaN only in the last tiles: each block's fixed-point exponent is its own,
    and the outputs have the checker's finite values and IEEE classes."""
    c = synth.make_case(77, M, 500, K, 4, bs, "packed", scale_lo=0.001, scale_hi=0.01)
    a = c["a"].copy()
    a[:, : K // 3] *= 1e-3
    a[:, 2 * K // 3:] *= 1e3
    w = _weights(dict(c, a=a), cuda_device)
    y = _mm(w, a, cuda_device, path=N.PATH_GEMV)
    assert oracle.rel_l2(y, oracle.managed(dict(c, a=a))) <= TOL_FP32
    b = a.copy()
    b[0, K - 7] = np.inf
    if M > 1:
        b[1, K - 200] = np.nan
    y = _mm(w, b, cuda_device, path=N.PATH_GEMV)
    ref = oracle.managed(dict(c, a=b))
    _classes_match(y, ref)
    fin = np.isfinite(ref)
    assert oracle.rel_l2(y[fin], ref[fin]) <= TOL_FP32
    w.free()


def test_gemm_nonfinite_activations_propagate(cuda_device):
    c = _nonfinite_case(40, 256, 1024, 32, "packed", 72)
    w = _weights(c, cuda_device)
    y = _mm(w, c["a"], cuda_device, path=N.PATH_GEMM)
    ref = oracle.managed(c)
    _classes_match(y, ref)
    fin = np.isfinite(ref)
    assert oracle.rel_l2(y[fin], ref[fin]) <= TOL_TC
    w.free()


def test_gemm_fp32_activations_beyond_fp16_range(cuda_device):
    c = synth.make_case(73, 48, 384, 2048, 4, 128, "packed", scale_lo=0.001, scale_hi=0.01)
    a = c["a"].astype(np.float64)
    a[:16] *= 1e30    # far above fp16's 65504
    a[16:32] *= 1e-20  # far below fp16's normal range
    a[40, :] *= 1e5   # one row past fp16 next to ordinary rows
    c = dict(c, a=a.astype(np.float32))
    w = _weights(c, cuda_device)
    y = _mm(w, c["a"], cuda_device, path=N.PATH_GEMM)
    ref = oracle.managed(c)
    assert np.isfinite(y).all()
    for rows in (slice(0, 16), slice(16, 32), slice(32, 48)):
        assert oracle.rel_l2(y[rows], ref[rows]) <= TOL_TC
    w.free()


def test_fused_rmsnorm_of_a_nonfinite_row_is_nan(cuda_device):
    """RMSNorm of a row holding inf is NaN everywhere (inf / inf), so the fused GEMV's outputs of
    that row are NaN; the other row of the launch keeps its value."""
    K, N_ = 512, 256
    c = synth.make_case(74, 2, N_, K, 4, 32, "packed", scale_lo=0.001, scale_hi=0.01)
    w = _weights(c, cuda_device)
    x = c["a"].copy()
    x[1, 7] = np.inf
    gamma = np.random.default_rng(3).uniform(0.8, 1.2, K).astype(np.float32)
    y = torch.empty(2, N_, device=cuda_device)
    w.matmul_fused(torch.from_numpy(x).to(cuda_device), y, rms_gamma=torch.from_numpy(gamma).to(cuda_device),
                   rms_eps=1e-5)
    torch.cuda.synchronize(cuda_device)
    out = y.cpu().numpy()
    assert np.isnan(out[1]).all()
    ref = oracle.managed(dict(c, a=od.rms_norm(x[:1], gamma, 1e-5), M=1))
    assert oracle.rel_l2(out[:1], ref) <= TOL_FP32
    w.free()
