"""msq_matmul_noalloc, the GEMM entry point that allocates nothing, on a B200.

It must give what msq_matmul_ex(..., MSQ_PATH_GEMM) gives on the same inputs (bar: the GEMM
tolerance, rel-L2 <= 5e-3, the weights entering the tensor core as fp16), on consecutive
calls that share its fixed staging array, and refuse inputs whose staging exceeds the array.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from modelsharp_b200 import QuantizedWeights, synth
from modelsharp_b200 import _native as N
from modelsharp_b200.weights import current_stream_ptr, dtype_code
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL_TC = 5e-3


def _run(fn_name, w, a, extra=()):
    M = a.numel() // w.K
    y = torch.full((M, w.n_rows), float("nan"), dtype=torch.float32, device=a.device)
    with torch.cuda.device(a.device):
        rc = getattr(N.lib(), fn_name)(None, current_stream_ptr(a.device), w.handle, a.data_ptr(), dtype_code(a), M,
                                       y.data_ptr(), w.n_rows, *extra)
    N.check(rc, fn_name)
    path = N.last_path()
    torch.cuda.synchronize(a.device)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    return y.cpu().numpy(), path


def _pair(w, a):
    y_ref, _ = _run("msq_matmul_ex", w, a, (N.PATH_GEMM,))
    y, path = _run("msq_matmul_noalloc", w, a)
    assert path.startswith("gemm_tc"), path
    assert np.isfinite(y).all()
    return y, y_ref


def test_noalloc_matches_gemm_entry_on_two_calls(cuda_device, native_lib):
    c = synth.make_case(51, 96, 1000, 4160, 4, 128, "packed", scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, c["block_size"], device=cuda_device)
    a1 = torch.from_numpy(c["a"]).to(cuda_device)
    # second call: other values, fewer rows and another dtype, over the contents the first left
    a2 = (torch.randn(40, c["K"], generator=torch.Generator().manual_seed(7)) * 0.5).to(torch.bfloat16)
    a2 = a2.to(cuda_device)
    y1, r1 = _pair(w, a1)
    y2, r2 = _pair(w, a2)
    assert oracle.rel_l2(y1, r1) <= TOL_TC
    assert oracle.rel_l2(y2, r2) <= TOL_TC
    assert oracle.rel_l2(y1, oracle.managed(c)) <= TOL_TC
    w.free()


def test_noalloc_size_limit_and_unstaged_fp16(cuda_device, native_lib):
    K = 4096
    c = synth.make_case(52, 1, 256, K, 4, 32, "none", scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], K, 4, 32, device=cuda_device)
    M = N.NOALLOC_SCRATCH_BYTES // (2 * K) + 1  # one row past what the fixed array can stage
    g = torch.Generator().manual_seed(9)
    a = torch.randn(M, K, generator=g).to(cuda_device)
    y = torch.empty(M, w.n_rows, dtype=torch.float32, device=cuda_device)
    before = N.launch_count()
    with torch.cuda.device(cuda_device):
        rc = N.lib().msq_matmul_noalloc(None, current_stream_ptr(cuda_device), w.handle, a.data_ptr(), N.DT_F32, M,
                                        y.data_ptr(), w.n_rows)
    assert rc == N.MSQ_E_INVALID
    assert "fixed scratch" in N.last_error()
    assert N.launch_count() == before
    # aligned fp16 A with K % 8 == 0 feeds the tensor core directly: no staging, no limit
    y16, r16 = _pair(w, a.to(torch.float16))
    assert oracle.rel_l2(y16, r16) <= TOL_TC
    w.free()
