"""Parity checker for MatMulNBits -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this
module. The product path (modelsharp_b200) never does.

* managed(case)           C restatement of the reference's managed kernel,
                          MatMulNBitsKernel.cs:216-262 + MatMulNBitsSimd.cs:40-96,141-203
                          (mnb_oracle.c: mnb_ref_managed)
* f64(case)               dequant + double dot, native/test/qgemm_test.cpp:60-89
                          (mnb_oracle.c: mnb_ref_f64)
* reference_native(case)  the reference's own ms_qgemm_nbits (native/src/qgemm.cpp:77-118),
                          compiled from the reference sources into oracle/_ref/ by
                          oracle/Makefile; fp32 scales, packed or absent zero points only.

Inputs follow the op: fp16 A / scales are widened exactly to fp32 first, as
GraphContext.Get does (src/ModelSharp/Cpu/Kernels/GraphContext.cs:106).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libmnb_oracle.so"
REF_SO = HERE / "_ref" / "libms_kernels_ref.so"
REF_TEST = HERE / "_ref" / "test_qgemm"

_oracle = None
_ref = None


def reference_root() -> str | None:
    """The reference checkout whose native sources the _ref build compiles: $MODELSHARP_REFERENCE,
    else a `reference` tree beside this repository; None when neither holds native/src/qgemm.cpp."""
    cands = [os.environ.get("MODELSHARP_REFERENCE"), str(HERE.parent.parent / "reference")]
    for c in cands:
        if c and Path(c, "native", "src", "qgemm.cpp").exists():
            return c
    return None


def build(ref_root: str | None = None) -> None:
    """Compiles the C restatement (and the reference kernel when its sources exist)."""
    env = dict(os.environ)
    if ref_root:
        env["REF"] = ref_root
    args = ["make", "-s", "-C", str(HERE)]
    if ref_root:
        args.append(f"REF={ref_root}")
    subprocess.run(args, check=True, env=env)


def _lib():
    global _oracle
    if _oracle is None:
        if not ORACLE_SO.exists():
            build()
        L = C.CDLL(str(ORACLE_SO))
        for name in ("mnb_ref_managed", "mnb_ref_f64", "mnb_ref_w4a8"):
            f = getattr(L, name)
            f.restype = C.c_int
            f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                          C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.mnb_dequant.restype = C.c_int
        L.mnb_dequant.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                  C.c_int, C.c_int, C.c_int]
        _oracle = L
    return _oracle


def reference_available() -> bool:
    return REF_SO.exists()


def _ref_lib():
    global _ref
    if _ref is None:
        L = C.CDLL(str(REF_SO))
        L.ms_qgemm_nbits.restype = None
        L.ms_qgemm_nbits.argtypes = [C.c_void_p] * 5 + [C.c_int] * 5
        L.ms_qgemm_w4a8.restype = None
        L.ms_qgemm_w4a8.argtypes = [C.c_void_p] * 5 + [C.c_int] * 5
        L.ms_build_info.restype = C.c_char_p
        _ref = L
    return _ref


def _inputs(case: dict, rows: slice | None = None):
    a = np.ascontiguousarray(np.asarray(case["a"], dtype=np.float32).reshape(-1, case["K"]))
    if rows is not None:
        a = np.ascontiguousarray(a[rows])
    b = np.ascontiguousarray(case["b"], dtype=np.uint8)
    s = np.ascontiguousarray(np.asarray(case["scales"]).astype(np.float32).reshape(-1))
    zk = case["zp_kind"]
    kind = {"none": 0, "packed": 1, "float": 2}[zk]
    z = None if case["zp"] is None else np.ascontiguousarray(case["zp"])
    if kind == 2:
        z = np.ascontiguousarray(z.astype(np.float32))
    return a, b, s, kind, z


def _run(fn_name: str, case: dict, threads: int = 0, rows: slice | None = None) -> np.ndarray:
    a, b, s, kind, z = _inputs(case, rows)
    M = a.shape[0]
    y = np.empty((M, case["N"]), dtype=np.float32)
    rc = getattr(_lib(), fn_name)(a.ctypes.data, b.ctypes.data, s.ctypes.data, kind,
                                  z.ctypes.data if z is not None else None, y.ctypes.data,
                                  M, case["N"], case["K"], case["bits"], case["block_size"], threads)
    if rc != 0:
        raise ValueError(f"{fn_name} rejected the case")
    return y


def managed(case: dict, threads: int = 0, rows: slice | None = None) -> np.ndarray:
    return _run("mnb_ref_managed", case, threads, rows)


def w4a8(case: dict, threads: int = 0, rows: slice | None = None) -> np.ndarray:
    """The C restatement of ms_qgemm_w4a8 (int8 activations per row and block; approximate)."""
    return _run("mnb_ref_w4a8", case, threads, rows)


def reference_w4a8(case: dict, rows: slice | None = None) -> np.ndarray:
    """The reference's own ms_qgemm_w4a8 (oracle/_ref, built from native/src/qgemm_w4a8.cpp)."""
    if case["zp_kind"] == "float":
        raise ValueError("ms_qgemm_w4a8 takes packed or absent zero points only")
    a, b, s, kind, z = _inputs(case, rows)
    M = a.shape[0]
    y = np.empty((M, case["N"]), dtype=np.float32)
    _ref_lib().ms_qgemm_w4a8(a.ctypes.data, b.ctypes.data, s.ctypes.data, z.ctypes.data if z is not None else None,
                             y.ctypes.data, M, case["N"], case["K"], case["bits"], case["block_size"])
    return y


def dequant(case: dict, threads: int = 0) -> np.ndarray:
    """The fp32 weight matrix W[N, K] = (q - zp) * scale (mnb_dequant)."""
    _, b, s, kind, z = _inputs(dict(case, a=np.zeros((1, case["K"]), np.float32)))
    out = np.empty((case["N"], case["K"]), dtype=np.float32)
    rc = _lib().mnb_dequant(b.ctypes.data, s.ctypes.data, kind, z.ctypes.data if z is not None else None,
                            out.ctypes.data, case["N"], case["K"], case["bits"], case["block_size"], threads)
    if rc != 0:
        raise ValueError("mnb_dequant rejected the case")
    return out


def f64(case: dict, threads: int = 0, rows: slice | None = None) -> np.ndarray:
    return _run("mnb_ref_f64", case, threads, rows)


def reference_native(case: dict, rows: slice | None = None) -> np.ndarray:
    """The reference's ms_qgemm_nbits on the case (packed / absent zero points only)."""
    if case["zp_kind"] == "float":
        raise ValueError("ms_qgemm_nbits takes packed or absent zero points only")
    a, b, s, kind, z = _inputs(case, rows)
    M = a.shape[0]
    y = np.empty((M, case["N"]), dtype=np.float32)
    _ref_lib().ms_qgemm_nbits(a.ctypes.data, b.ctypes.data, s.ctypes.data,
                              z.ctypes.data if z is not None else None, y.ctypes.data,
                              M, case["N"], case["K"], case["bits"], case["block_size"])
    return y


def rel_l2(y: np.ndarray, ref: np.ndarray) -> float:
    y = np.asarray(y, dtype=np.float64).reshape(-1)
    r = np.asarray(ref, dtype=np.float64).reshape(-1)
    den = np.linalg.norm(r)
    return float(np.linalg.norm(y - r) / (den if den > 0 else 1.0))
