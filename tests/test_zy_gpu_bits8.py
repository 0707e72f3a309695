"""bits=8 weights on the decode GEMV's 8-bit form, through the C ABI (needs a B200).

A bits=8 handle keeps only the decode stream, one byte per code in the mma.m16n8k32 fragment
order, and every M takes the exact integer GEMV (M > 4 in passes). Bar: rel-L2 <= 1e-5 against
the parity checker and against the reference's own ms_qgemm_nbits outputs
(tests/golden/ref_native.npz); inf / NaN in A propagate class by class as for 4-bit weights.
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import synth
from modelsharp_b200 import _native as N
from oracle import oracle
from tests.test_gpu_parity import GOLD, META, TOL_FP32, golden_case, pack, run

pytestmark = pytest.mark.gpu

@pytest.mark.parametrize("e", [e for e in META["cases"] if e["bits"] == 8 and e["block_size"] in (32, 64, 128)],
                         ids=lambda e: e["key"])
def test_golden_gemv_bits8(cuda_device, e):
    """bits=8 weights on the decode GEMV's 8-bit form against the reference's own ms_qgemm_nbits."""
    c = golden_case(e["key"])
    ref = np.load(GOLD / "ref_native.npz")[e["key"]]
    y = run(c, cuda_device)  # the default route: every M of a bits=8 handle takes the GEMV
    assert N.last_path().startswith("gemv_imma_b8")
    assert oracle.rel_l2(y, ref) <= TOL_FP32
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32


@pytest.mark.parametrize("M", [1, 3, 4, 7, 16, 40])
@pytest.mark.parametrize("K,bs,zp_kind", [(4096, 128, "packed"), (1000, 32, "none"), (2048, 64, "float"),
                                          (4160, 128, "none"), (896, 32, "packed")])
def test_gemv_bits8(cuda_device, M, K, bs, zp_kind):
    c = synth.make_case(88, M, 700, K, 8, bs, zp_kind, scale_lo=0.0001, scale_hi=0.001)
    w = pack(c, cuda_device)
    assert w.query_device_bytes() <= 1.1 * synth.algorithmic_bytes(700, K, 8, bs, zp_kind)  # one layout
    y = w.matmul(torch.from_numpy(c["a"]).to(cuda_device)).cpu().numpy()
    assert N.last_path().startswith("gemv_imma_b8")
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_FP32
    w.free()


def test_gemv_bits8_half_activations_and_nonfinite(cuda_device):
    c = synth.make_case(89, 3, 512, 2048, 8, 64, "packed", a_dtype="f16", scale_lo=0.0001, scale_hi=0.001)
    assert oracle.rel_l2(run(c, cuda_device), oracle.managed(c)) <= TOL_FP32
    a = np.asarray(c["a"], np.float32).copy()
    a[0, 9] = np.inf
    a[2, 100] = np.nan
    cn = dict(c, a=a)
    y = run(cn, cuda_device)
    ref = oracle.managed(cn)
    for f in (np.isnan, np.isposinf, np.isneginf):
        assert np.array_equal(f(y), f(ref)), f.__name__
    fin = np.isfinite(ref)
    assert oracle.rel_l2(y[fin], ref[fin]) <= TOL_FP32
