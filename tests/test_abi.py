"""The C-ABI library on a host without a GPU: it loads, exports exactly what the header
declares, and its validation reproduces the reference op's errors (MatMulNBitsKernel.cs:87-161).
No compute call is made here."""
import ctypes as C
import re

import numpy as np
import pytest

from modelsharp_b200 import _native as N


def header_functions() -> list[str]:
    text = N.HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(msq_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert header_functions() == sorted(N.SIGNATURES)


def test_library_exports_every_symbol(native_lib):
    for name in header_functions():
        assert hasattr(native_lib, name), name


def test_build_info(native_lib):
    info = native_lib.msq_build_info().decode()
    assert "sm_100a" in info


def check(N_, K, bits, bs, b_len, s_len, zp_dt=N.DT_ABSENT, zp_len=0, g_idx=None, a_dims=(1, 4)):
    M = C.c_int64(-7)
    dims = np.asarray(a_dims, dtype=np.int64)
    gi = None if g_idx is None else np.asarray(g_idx, dtype=np.int64)
    rc = N.lib().msq_check_node(N_, K, bits, bs, b_len, s_len, zp_dt, zp_len,
                                gi.ctypes.data if gi is not None else None, 0 if gi is None else gi.size,
                                dims.ctypes.data if dims.size else None, dims.size, C.byref(M))
    return rc, N.last_error(), M.value


@pytest.mark.parametrize("args,rc,msg", [
    ((0, 4, 4, 4, 4, 2), N.MSQ_E_INVALID, "MatMulNBits requires positive N and K attributes (got N=0, K=4)."),
    ((2, -1, 4, 4, 4, 2), N.MSQ_E_INVALID, "MatMulNBits requires positive N and K attributes (got N=2, K=-1)."),
    ((2, 4, 3, 4, 4, 2), N.MSQ_E_INVALID, "MatMulNBits supports bits=4 or bits=8; got 3."),
    ((2, 4, 4, 0, 4, 2), N.MSQ_E_INVALID, "MatMulNBits requires a positive block_size; got 0."),
    ((2, 4, 4, 4, 5, 2), N.MSQ_E_INVALID,
     "MatMulNBits B has 5 elements; expected 4 (N=2 × n_blocks_per_row=1 × blob_size=2)."),
    ((2, 4, 4, 4, 4, 3), N.MSQ_E_INVALID,
     "MatMulNBits scales has 3 elements; expected 2 (N=2 × n_blocks_per_row=1)."),
])
def test_validation_messages(native_lib, args, rc, msg):
    got_rc, got_msg, _ = check(*args)
    assert got_rc == rc
    assert got_msg == msg


def test_zero_point_validation(native_lib):
    rc, msg, _ = check(2, 4, 4, 4, 4, 2, N.DT_F32, 3)
    assert (rc, msg) == (N.MSQ_E_INVALID, "MatMulNBits float zero_points has 3 elements; expected 2.")
    rc, msg, _ = check(2, 4, 4, 4, 4, 2, N.DT_U8, 3)
    assert (rc, msg) == (N.MSQ_E_INVALID, "MatMulNBits packed zero_points has 3 bytes; expected 2 (N=2 × 1).")
    rc, msg, _ = check(2, 4, 4, 4, 4, 2, N.DT_F16, 2)
    assert (rc, msg) == (N.MSQ_E_INVALID, "MatMulNBits zero_points must be Float32 or UInt8; got Float16.")
    assert check(2, 4, 4, 4, 4, 2, N.DT_U8, 2)[0] == N.MSQ_OK
    assert check(2, 4, 4, 4, 4, 2, N.DT_F32, 2)[0] == N.MSQ_OK


def test_g_idx_and_a_shape(native_lib):
    assert check(2, 8, 4, 4, 8, 4, g_idx=[0, 0, 0, 0, 1, 1, 1, 1], a_dims=(3, 8))[0] == N.MSQ_OK
    rc, msg, _ = check(2, 8, 4, 4, 8, 4, g_idx=[0, 0, 0, 0, 1, 1, 0, 1], a_dims=(3, 8))
    assert (rc, msg) == (N.MSQ_E_UNSUPPORTED,
                         "MatMulNBits g_idx with a non-trivial block permutation is not supported.")
    rc, msg, _ = check(2, 8, 4, 4, 8, 4, a_dims=(2, 3, 7))
    assert (rc, msg) == (N.MSQ_E_INVALID, "MatMulNBits A inner dimension must equal K=8; got shape [2,3,7].")
    rc, msg, _ = check(2, 8, 4, 4, 8, 4, a_dims=())
    assert (rc, msg) == (N.MSQ_E_INVALID, "MatMulNBits A inner dimension must equal K=8; got shape [].")
    rc, _, M = check(2, 8, 4, 4, 8, 4, a_dims=(2, 3, 8))
    assert rc == N.MSQ_OK and M == 6
    rc, _, M = check(2, 8, 4, 4, 8, 4, a_dims=(0, 8))
    assert rc == N.MSQ_OK and M == 0


def test_ragged_k_geometry(native_lib):
    # K=6, bs=4 -> nb=2, blob=2 (MatMulNBitsTests.cs:217-241)
    assert check(1, 6, 4, 4, 4, 2, a_dims=(1, 6))[0] == N.MSQ_OK
    # bits=8, bs=4 -> blob=4
    assert check(2, 4, 8, 4, 8, 2)[0] == N.MSQ_OK


def test_pack_rejects_before_touching_a_device(native_lib):
    h = C.c_void_p()
    rc = native_lib.msq_pack(None, None, None, 5, None, N.DT_F32, 2, None, N.DT_ABSENT, 0, 2, 4, 4, 4, 0, 2, 0,
                             C.byref(h))
    assert rc == N.MSQ_E_INVALID and "B has 5 elements" in N.last_error()
    rc = native_lib.msq_pack(None, None, None, 4, None, N.DT_I32, 2, None, N.DT_ABSENT, 0, 2, 4, 4, 4, 0, 2, 0,
                             C.byref(h))
    assert rc == N.MSQ_E_INVALID and "scales must be Float32 or Float16; got Int32" in N.last_error()
    rc = native_lib.msq_pack(None, None, C.c_void_p(16), 4, C.c_void_p(16), N.DT_F32, 2, None, N.DT_ABSENT, 0,
                             2, 4, 4, 4, 1, 1, 0, C.byref(h))
    assert rc == N.MSQ_E_INVALID and "row range" in N.last_error()
    assert not h.value


def test_noalloc_scratch_size_constant():
    m = re.search(r"#define\s+MSQ_NOALLOC_SCRATCH_BYTES\s+\((\d+)u\s*<<\s*(\d+)\)", N.HEADER.read_text())
    assert m and int(m.group(1)) << int(m.group(2)) == N.NOALLOC_SCRATCH_BYTES
