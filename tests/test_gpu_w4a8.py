"""msq_matmul_w4a8, the int8-activation decode GEMV, against the reference's ms_qgemm_w4a8
arithmetic (needs a B200).

The activations are quantised per (row, block) with the reference's IEEE steps, so the GPU's
int8 values and integer block dots equal the restatement's; only the fp32 sum over blocks runs
in another order. Bar: rel-L2 <= 1e-6 against the restatement (oracle.w4a8) and against the
reference's own build where it exists. Against the fp32 op the form is approximate, as the
reference's is (about 0.5 %).
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import QuantizedWeights, synth
from modelsharp_b200 import _native as N
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-6


def w4a8(w, a, dev):
    M = a.shape[0]
    y = torch.full((M, w.n_rows), float("nan"), device=dev)
    at = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    with torch.cuda.device(dev):
        rc = N.lib().msq_matmul_w4a8(None, torch.cuda.current_stream(dev).cuda_stream, w.handle, at.data_ptr(),
                                     N.DT_F32 if a.dtype == np.float32 else N.DT_F16, M, y.data_ptr(), w.n_rows)
    N.check(rc, "msq_matmul_w4a8")
    torch.cuda.synchronize(dev)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    return y.cpu().numpy()


@pytest.mark.parametrize("M,N_,K,bs,zp", [
    (1, 4864, 896, 32, "packed"),     # the Qwen up-proj of configs[0]
    (1, 4096, 4096, 128, "packed"),
    (3, 1000, 4160, 128, "none"),     # ragged K, ragged N
    (8, 512, 1024, 64, "packed"),     # a full pass of 8 rows
    (13, 300, 2048, 32, "packed"),    # two passes
    (4, 14336, 4096, 128, "packed"),
    (8, 700, 14336, 128, "packed"),   # 28 k-units per stream tile, 4 tiles
])
def test_w4a8_matches_reference_arithmetic(cuda_device, M, N_, K, bs, zp):
    c = synth.make_case(95, M, N_, K, 4, bs, zp, scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], N_, K, 4, bs, device=cuda_device)
    y = w4a8(w, c["a"], cuda_device)
    assert N.last_path().startswith("gemv_w4a8")
    assert oracle.rel_l2(y, oracle.w4a8(c)) <= TOL
    if oracle.reference_available():
        assert oracle.rel_l2(y, oracle.reference_w4a8(c)) <= TOL
    assert 1e-4 < oracle.rel_l2(y, oracle.managed(c)) < 2e-2  # approximate, like the reference's form
    w.free()


def test_w4a8_rejects_float_zero_points(cuda_device):
    c = synth.make_case(96, 1, 256, 256, 4, 32, "float")
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], 256, 256, 4, 32, device=cuda_device)
    y = torch.empty(1, 256, device=cuda_device)
    a = torch.from_numpy(c["a"]).to(cuda_device)
    rc = N.lib().msq_matmul_w4a8(None, None, w.handle, a.data_ptr(), N.DT_F32, 1, y.data_ptr(), 256)
    assert rc == N.MSQ_E_UNSUPPORTED and "zero points" in N.last_error()
    w.free()
