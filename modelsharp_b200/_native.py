"""ctypes binding of libms_cuda_nbits.so (include/ms_cuda_nbits.h).

Library resolution mirrors the reference's DllImport resolver
(src/ModelSharp/Native/NativeGemm.cs:235-253, NativeCuda.cs:182-200): an explicit path in
MODELSHARP_CUDA_NBITS_LIB first, then the in-tree build next to this file. There is no
fallback: a missing library raises, because this op has no CPU or library path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

from .errors import ModelSharpException

MSQ_OK = 0
MSQ_E_INVALID = -1
MSQ_E_UNSUPPORTED = -2
MSQ_E_CUDA = -3
MSQ_E_NO_DEVICE = -4
MSQ_E_OOM = -5
MSQ_E_TIMEOUT = -6

# ElementType codes (src/ModelSharp/Tensors/ElementType.cs:4-15) plus bf16.
DT_ABSENT, DT_F32, DT_F64, DT_F16, DT_I32, DT_I64, DT_I8, DT_U8, DT_BOOL, DT_BF16 = -1, 1, 2, 3, 4, 5, 6, 7, 8, 16

PATH_AUTO, PATH_GENERIC, PATH_GEMV, PATH_GEMM, PATH_GEMM_SPLIT, PATH_AUTO_SPLIT, PATH_GEMV_TC = 0, 1, 2, 3, 4, 5, 6
NOALLOC_SCRATCH_BYTES = 16 << 20  # MSQ_NOALLOC_SCRATCH_BYTES


def noalloc_staging_bytes(M: int, K: int) -> int:
    """Bytes msq_matmul_noalloc stages for M rows of float32/bfloat16 A: fp16 rows of K rounded
    up to 8, padded to 256 bytes, then one fp32 row scale per row."""
    return (M * ((K + 7) // 8 * 8) * 2 + 255) // 256 * 256 + 4 * M
MAX_RANKS = 8  # MSQ_MAX_RANKS
IPC_HANDLE_BYTES = 64  # MSQ_IPC_HANDLE_BYTES


class GatherT(C.Structure):
    """msq_gather_t: one layer's output exchange seen from one rank."""
    _fields_ = [("nranks", C.c_int), ("rank", C.c_int), ("y", C.c_void_p * MAX_RANKS),
                ("arrivals", C.c_void_p * MAX_RANKS), ("ldy", C.c_int64), ("col0", C.c_int64),
                ("produced", C.c_void_p), ("done", C.c_void_p)]


class WaitT(C.Structure):
    """msq_wait_t: a gathered input to wait for."""
    _fields_ = [("arrivals", C.c_void_p), ("produced", C.c_void_p), ("nranks", C.c_int)]


class FusionT(C.Structure):
    """msq_fusion_t: glue folded into a decode GEMV."""
    _fields_ = [("rms_gamma", C.c_void_p), ("rms_eps", C.c_float), ("swiglu", C.c_int32), ("accumulate", C.c_int32)]


PACK_DEFAULT, PACK_GENERIC_ONLY, PACK_LAZY_GEMM = 0, 1, 2
DIAG_POOL_ALLOCS, DIAG_NOALLOC_LOOKUPS, DIAG_POOL_RESERVED = 1, 2, 3  # MSQ_DIAG_*

LIB_NAME = "libms_cuda_nbits.so"
HEADER = Path(__file__).resolve().parent.parent / "include" / "ms_cuda_nbits.h"

_vp = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int

# name -> (restype, argtypes); every function the header declares.
SIGNATURES: dict[str, tuple] = {
    "msq_build_info": (C.c_char_p, []),
    "msq_available": (_i32, []),
    "msq_last_error": (C.c_char_p, []),
    "msq_launch_count": (_i64, []),
    "msq_last_path": (C.c_char_p, []),
    "msq_diag_counter": (_i64, [_i32]),
    "msq_check_node": (_i32, [_i32, _i32, _i32, _i32, _i64, _i64, _i32, _i64, _vp, _i64, _vp, _i32, _vp]),
    "msq_pack": (_i32, [_vp, _vp, _vp, _i64, _vp, _i32, _i64, _vp, _i32, _i64, _i32, _i32, _i32, _i32,
                        _i32, _i32, _i32, _vp]),
    "msq_pack_host": (_i32, [_vp, _vp, _vp, _i64, _vp, _i32, _i64, _vp, _i32, _i64, _i32, _i32, _i32, _i32,
                             _i32, _i32, _i32, _vp]),
    "msq_weights_query": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "msq_free": (_i32, [_vp]),
    "msq_matmul": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _vp, _i64]),
    "msq_matmul_ex": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _vp, _i64, _i32]),
    "msq_matmul_host": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _vp]),
    "msq_matmul_host_async": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _vp]),
    "msq_matmul_noalloc": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _vp, _i64]),
    "msq_matmul_w4a8": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _vp, _i64]),
    "msq_device_status": (_i32, [_vp, _vp]),
    "msq_set_wait_budget": (_i32, [_vp, _i64]),
    "msq_xbuf_alloc": (_i32, [_vp, _i64, _vp]),
    "msq_xbuf_free": (_i32, [_vp, _vp]),
    "msq_ipc_handle": (_i32, [_vp, _vp, _vp]),
    "msq_ipc_open": (_i32, [_vp, _vp, _vp]),
    "msq_ipc_close": (_i32, [_vp, _vp]),
    "msq_matmul_gather": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _vp, _vp]),
    "msq_wait_gathered": (_i32, [_vp, _vp, _vp]),
    "msq_add_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, C.c_float]),
    "msq_rope_append": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i64]),
    "msq_gqa_decode": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64]),
    "msq_rope_gqa_decode": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64]),
    "msq_swiglu": (_i32, [_vp, _vp, _vp, _vp, _i64]),
    "msq_argmax": (_i32, [_vp, _vp, _vp, _i64, _vp, _vp]),
    "msq_rope_append_rows": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i64]),
    "msq_gqa_prefill": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _i32, _i32, _i32, _i64]),
    "msq_swiglu_rows": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64]),
    "msq_matmul_fused": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, C.POINTER(FusionT)]),
    "msq_qgemm_nbits": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32]),
}

_lib: C.CDLL | None = None


def library_path() -> Path:
    env = os.environ.get("MODELSHARP_CUDA_NBITS_LIB")
    if env:
        return Path(env)
    return Path(__file__).resolve().parent / LIB_NAME


def lib() -> C.CDLL:
    """The loaded library; raises ModelSharpException when it is missing."""
    global _lib
    if _lib is None:
        p = library_path()
        if not p.exists():
            raise ModelSharpException(
                f"{LIB_NAME} not found at {p}; build it with `python -m modelsharp_b200.build` "
                "(MatMulNBits has no CPU fallback on this backend).")
        L = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().msq_last_error() or b"").decode("utf-8", "replace")


def check(rc: int, what: str = "") -> None:
    """Raises ModelSharpException with the library's message for a non-zero status."""
    if rc != MSQ_OK:
        msg = last_error() or f"{what} failed with status {rc}"
        raise ModelSharpException(msg, status=rc)


def launch_count() -> int:
    return int(lib().msq_launch_count())


def diag_counter(which: int) -> int:
    """msq_diag_counter: DIAG_POOL_ALLOCS, DIAG_NOALLOC_LOOKUPS or DIAG_POOL_RESERVED."""
    return int(lib().msq_diag_counter(which))


def last_path() -> str:
    return (lib().msq_last_path() or b"").decode()


def available() -> bool:
    return bool(lib().msq_available())
