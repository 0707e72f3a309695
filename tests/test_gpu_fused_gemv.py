"""The decode GEMV with decode-step glue folded in (msq_matmul_fused), through the C ABI.

Each form is compared with the unfused chain on the CPU: the parity checker's MatMulNBits
(oracle.managed) applied to the checker's RMSNorm or SwiGLU of A (oracle/decoder.py), plus
the residual for the accumulating form. Bar: rel-L2 <= 1e-5 (the fused RMSNorm scales the
dot product by 1/rms instead of each element, a difference of fp32 rounding).
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import QuantizedWeights, synth
from modelsharp_b200 import _native as N
from modelsharp_b200.errors import ModelSharpException
from oracle import decoder as od
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-5
SHAPES = [(4096, 4096, 32), (4096, 6144, 32), (1024, 640, 128), (512, 200, 64), (14336, 1024, 32)]


def _case(K, N_, bs, M, seed):
    c = synth.make_case(seed, M, N_, K, 4, bs, "packed", a_dist="normal", scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], N_, K, 4, bs, device="cuda:0")
    return c, w


def _ref(c, a):
    return oracle.managed(dict(c, a=np.ascontiguousarray(a, dtype=np.float32), M=a.shape[0]))


@pytest.mark.parametrize("K,N_,bs", SHAPES)
@pytest.mark.parametrize("M", [1, 3, 6])
def test_rmsnorm_folded(cuda_device, K, N_, bs, M):
    c, w = _case(K, N_, bs, M, K + N_ + M)
    rng = np.random.default_rng(M)
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    gamma = rng.uniform(0.8, 1.2, K).astype(np.float32)
    y = torch.empty(M, N_, device=cuda_device)
    w.matmul_fused(torch.from_numpy(x).to(cuda_device), y, rms_gamma=torch.from_numpy(gamma).to(cuda_device),
                   rms_eps=1e-5)
    ref = _ref(c, od.rms_norm(x, gamma, 1e-5))
    assert oracle.rel_l2(y.cpu().numpy(), ref) <= TOL
    assert N.last_path() == "gemv_imma_fused"
    w.free()


@pytest.mark.parametrize("K,N_,bs", SHAPES)
@pytest.mark.parametrize("M", [1, 4])
def test_swiglu_accumulate_folded(cuda_device, K, N_, bs, M):
    c, w = _case(K, N_, bs, M, 7 * K + N_ + M)
    rng = np.random.default_rng(K + M)
    gu = (rng.standard_normal((M, 2 * K)) * 2).astype(np.float32)
    resid = rng.standard_normal((M, N_)).astype(np.float32)
    y = torch.from_numpy(resid.copy()).to(cuda_device)
    w.matmul_fused(torch.from_numpy(gu).to(cuda_device), y, swiglu=True, accumulate=True)
    g, u = gu[:, :K], gu[:, K:]
    act = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
    ref = resid + _ref(c, act)
    assert oracle.rel_l2(y.cpu().numpy(), ref) <= TOL
    w.free()


def test_accumulate_only_and_plain_form(cuda_device):
    K, N_, bs, M = 4096, 4096, 32, 2
    c, w = _case(K, N_, bs, M, 99)
    a = torch.from_numpy(c["a"].reshape(M, K)).to(cuda_device)
    base = torch.randn(M, N_, device=cuda_device)
    y = base.clone()
    w.matmul_fused(a, y, accumulate=True)
    ref = _ref(c, c["a"].reshape(M, K))
    assert oracle.rel_l2(y.cpu().numpy(), base.cpu().numpy() + ref) <= TOL
    y2 = torch.full((M, N_), 7.0, device=cuda_device)
    w.matmul_fused(a, y2)  # no fusion: the plain GEMV, Y overwritten
    np.testing.assert_array_equal(y2.cpu().numpy(), w.matmul(a, path=N.PATH_GEMV).cpu().numpy())
    w.free()


def test_fused_in_graph_replays_equal_eager(cuda_device):
    K, N_, bs = 4096, 6144, 32
    c, w = _case(K, N_, bs, 1, 5)
    x = torch.randn(1, K, device=cuda_device)
    gamma = torch.rand(K, device=cuda_device) + 0.5
    y_e = torch.empty(1, N_, device=cuda_device)
    w.matmul_fused(x, y_e, rms_gamma=gamma)
    y = torch.empty(1, N_, device=cuda_device)
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            w.matmul_fused(x, y, rms_gamma=gamma)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    g.replay()
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(y, y_e)  # deterministic: fixed reduction order
    del g
    w.free()


def test_rejections(cuda_device):
    K, N_ = 4096, 256
    c, w = _case(K, N_, 32, 1, 3)
    x = torch.randn(1, K + 4, device=cuda_device)
    y = torch.empty(1, N_, device=cuda_device)
    gamma = torch.ones(K, device=cuda_device)
    L = N.lib()
    st = torch.cuda.current_stream(cuda_device).cuda_stream
    both = N.FusionT(gamma.data_ptr(), 1e-5, 1, 0)
    assert L.msq_matmul_fused(None, st, w.handle, x.data_ptr(), 1, y.data_ptr(), N_, N.C.byref(both)) == N.MSQ_E_INVALID
    plain = N.FusionT(None, 0.0, 0, 0)
    # A one float off a 16-byte boundary
    assert L.msq_matmul_fused(None, st, w.handle, x.data_ptr() + 4, 1, y.data_ptr(), N_,
                              N.C.byref(plain)) == N.MSQ_E_UNSUPPORTED
    assert L.msq_matmul_fused(None, st, w.handle, x.data_ptr(), 17, y.data_ptr(), N_,
                              N.C.byref(plain)) == N.MSQ_E_UNSUPPORTED  # M > 16
    assert L.msq_matmul_fused(None, st, w.handle, x.data_ptr(), 1, y.data_ptr(), N_ - 1,
                              N.C.byref(plain)) == N.MSQ_E_INVALID  # ldy < rows
    w.free()
    c16 = synth.make_case(4, 1, 64, 256, 4, 16, "packed")
    w16 = QuantizedWeights(c16["b"], c16["scales"], c16["zp"], 64, 256, 4, 16, device=cuda_device)
    with pytest.raises(ModelSharpException):
        w16.matmul_fused(torch.randn(1, 256, device=cuda_device), torch.empty(1, 64, device=cuda_device))
    w16.free()
