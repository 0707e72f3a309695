"""msq_matmul_noalloc, the GEMM entry point that allocates nothing, on a B200.

It must give what msq_matmul_ex(..., MSQ_PATH_GEMM) gives on the same inputs (bar: the GEMM
tolerance, rel-L2 <= 5e-3, the weights entering the tensor core as fp16), on consecutive
calls that share its fixed staging array, take no memory from any allocator once its set-up
has run, and refuse inputs whose staging exceeds the array. Its set-up (the array's address)
is per CUDA context: a context created after another was destroyed gets its own lookup even
when the driver hands back the same CUcontext handle.
"""
import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from modelsharp_b200 import QuantizedWeights, synth
from modelsharp_b200 import _native as N
from modelsharp_b200.weights import current_stream_ptr, dtype_code
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL_TC = 5e-3


def _max_rows(K):
    M = N.NOALLOC_SCRATCH_BYTES // (2 * K)
    while N.noalloc_staging_bytes(M, K) > N.NOALLOC_SCRATCH_BYTES:
        M -= 1
    return M


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
    M = _max_rows(K) + 1  # one row past what the fixed array can stage
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


def test_noalloc_takes_no_memory_and_fills_the_array_exactly(cuda_device, native_lib):
    K = 4096
    c = synth.make_case(53, 1, 512, K, 4, 32, "packed", scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], K, 4, 32, device=cuda_device)
    M = _max_rows(K)  # the largest M the fixed array stages: full to within one row scale
    assert N.NOALLOC_SCRATCH_BYTES - N.noalloc_staging_bytes(M, K) < 2 * K + 4
    g = torch.Generator().manual_seed(11)
    a = torch.randn(M, K, generator=g).to(cuda_device)
    y = torch.empty(M, w.n_rows, dtype=torch.float32, device=cuda_device)

    def call():
        with torch.cuda.device(cuda_device):
            rc = N.lib().msq_matmul_noalloc(None, current_stream_ptr(cuda_device), w.handle, a.data_ptr(),
                                            N.DT_F32, M, y.data_ptr(), w.n_rows)
        N.check(rc, "msq_matmul_noalloc")
        torch.cuda.synchronize(cuda_device)

    call()  # set-up: the array's address in this context
    pool_allocs = N.diag_counter(N.DIAG_POOL_ALLOCS)
    pool_reserved = N.diag_counter(N.DIAG_POOL_RESERVED)
    lookups = N.diag_counter(N.DIAG_NOALLOC_LOOKUPS)
    torch_bytes = torch.cuda.memory_allocated(cuda_device)
    free_before = torch.cuda.mem_get_info(cuda_device)[0]
    for _ in range(3):
        call()
    assert N.diag_counter(N.DIAG_POOL_ALLOCS) == pool_allocs
    assert N.diag_counter(N.DIAG_POOL_RESERVED) == pool_reserved
    assert N.diag_counter(N.DIAG_NOALLOC_LOOKUPS) == lookups
    assert torch.cuda.memory_allocated(cuda_device) == torch_bytes
    assert torch.cuda.mem_get_info(cuda_device)[0] == free_before
    y_na = y.cpu().numpy()
    y_ref, _ = _run("msq_matmul_ex", w, a, (N.PATH_GEMM,))
    assert oracle.rel_l2(y_na, y_ref) <= TOL_TC
    w.free()


def _child_two_contexts() -> None:
    """Runs in a fresh process without torch: two driver contexts, one after the other, each
    packing weights, calling the no-allocation GEMM twice and checking it against the exact
    GEMV path in the same context. Prints the lookup counts it saw."""
    import numpy as np

    from modelsharp_b200 import _native as NN
    from modelsharp_b200 import synth as S

    cu = C.CDLL("libcuda.so.1")
    def ok(r, what):
        if r != 0:
            raise RuntimeError(f"{what} failed ({r})")
    ok(cu.cuInit(0), "cuInit")
    dev = C.c_int()
    ok(cu.cuDeviceGet(C.byref(dev), 0), "cuDeviceGet")
    L = NN.lib()
    c = S.make_case(54, 40, 384, 1024, 4, 32, "packed", scale_lo=0.001, scale_hi=0.01)
    a = np.ascontiguousarray(c["a"], dtype=np.float32)
    M, K, Nn = 40, 1024, 384
    handles, lookups, outs = [], [], []
    for rnd in range(2):
        ctx = C.c_void_p()
        ok(cu.cuCtxCreate_v2(C.byref(ctx), 0, dev), "cuCtxCreate")
        handles.append(ctx.value)
        wh = C.c_void_p()
        zp = c["zp"]
        rc = L.msq_pack_host(ctx, None, c["b"].ctypes.data, c["b"].size, c["scales"].ctypes.data, NN.DT_F32,
                             c["scales"].size, zp.ctypes.data, NN.DT_U8, zp.size, Nn, K, 4, 32, 0, Nn, 0,
                             C.byref(wh))
        NN.check(rc, "msq_pack_host")
        da, dy, dg = C.c_uint64(), C.c_uint64(), C.c_uint64()
        ok(cu.cuMemAlloc_v2(C.byref(da), C.c_size_t(a.nbytes)), "cuMemAlloc")
        ok(cu.cuMemAlloc_v2(C.byref(dy), C.c_size_t(M * Nn * 4)), "cuMemAlloc")
        ok(cu.cuMemAlloc_v2(C.byref(dg), C.c_size_t(M * Nn * 4)), "cuMemAlloc")
        ok(cu.cuMemcpyHtoD_v2(da, a.ctypes.data, C.c_size_t(a.nbytes)), "cuMemcpyHtoD")
        ys = []
        for _ in range(2):
            NN.check(L.msq_matmul_noalloc(ctx, None, wh, da.value, NN.DT_F32, M, dy.value, Nn), "noalloc")
            ok(cu.cuCtxSynchronize(), "cuCtxSynchronize")
            y = np.empty((M, Nn), np.float32)
            ok(cu.cuMemcpyDtoH_v2(y.ctypes.data, dy, C.c_size_t(y.nbytes)), "cuMemcpyDtoH")
            ys.append(y)
        NN.check(L.msq_matmul_ex(ctx, None, wh, da.value, NN.DT_F32, M, dg.value, Nn, NN.PATH_GEMV), "gemv")
        ok(cu.cuCtxSynchronize(), "cuCtxSynchronize")
        yg = np.empty((M, Nn), np.float32)
        ok(cu.cuMemcpyDtoH_v2(yg.ctypes.data, dg, C.c_size_t(yg.nbytes)), "cuMemcpyDtoH")
        NN.check(L.msq_device_status(ctx, None), "device status")
        lookups.append(NN.diag_counter(NN.DIAG_NOALLOC_LOOKUPS))
        err = float(np.linalg.norm(ys[0] - yg) / np.linalg.norm(yg))
        assert np.array_equal(ys[0], ys[1]), "two calls in one context differ"
        assert err <= TOL_TC, err
        outs.append(ys[0])
        NN.check(L.msq_free(wh), "msq_free")
        for d in (da, dy, dg):
            ok(cu.cuMemFree_v2(d), "cuMemFree")
        ok(cu.cuCtxDestroy_v2(ctx), "cuCtxDestroy")
    assert np.array_equal(outs[0], outs[1]), "the two contexts disagree"
    print(f"handles_equal={handles[0] == handles[1]} lookups={lookups}")
    assert lookups == [1, 2], lookups


def test_noalloc_set_up_is_per_context(cuda_device, native_lib):
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = env.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0] or "0"
    r = subprocess.run([sys.executable, "-c", "from tests.test_zz_no_alloc import _child_two_contexts as f; f()"],
                       cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "lookups=[1, 2]" in r.stdout, r.stdout
