"""Writes ONNX ModelProto bytes for the loader tests (test infrastructure; there is no onnx
package here). Field numbers are ONNX's (onnx.proto): ModelProto ir_version 1, graph 7,
opset_import 8; GraphProto node 1, name 2, initializer 5, input 11, output 12; NodeProto input 1,
output 2, name 3, op_type 4, attribute 5, domain 7; AttributeProto name 1, f 2, i 3, s 4,
floats 7, ints 8, type 20; TensorProto dims 1, data_type 2, float_data 4, int32_data 5, name 8,
raw_data 9, external_data 13, data_location 14.
"""
from __future__ import annotations

import struct

import numpy as np

DT = {np.dtype(np.float32): 1, np.dtype(np.uint8): 2, np.dtype(np.int8): 3, np.dtype(np.int32): 6,
      np.dtype(np.int64): 7, np.dtype(np.bool_): 9, np.dtype(np.float16): 10}


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _ld(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _vi(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v)


def _str(field: int, s: str) -> bytes:
    return _ld(field, s.encode())


def tensor(name: str, arr: np.ndarray, external: tuple[str, int, int] | None = None, as_int32_data: bool = False,
           bf16: bool = False) -> bytes:
    """TensorProto: raw_data inline, or external (location, offset, length), or int32_data."""
    arr = np.asarray(arr)
    out = b"".join(_vi(1, d) for d in arr.shape)
    out += _vi(2, 16 if bf16 else DT[arr.dtype]) + _str(8, name)
    if external is not None:
        loc, off, length = external
        for k, v in (("location", loc), ("offset", str(off)), ("length", str(length))):
            out += _ld(13, _str(1, k) + _str(2, v))
        out += _vi(14, 1)
    elif as_int32_data:
        vals = arr.view(np.uint16) if arr.dtype == np.float16 else arr
        out += b"".join(_vi(5, int(v)) for v in vals.reshape(-1))
    else:
        out += _ld(9, np.ascontiguousarray(arr).astype(arr.dtype.newbyteorder("<")).tobytes())
    return out


def attr_int(name: str, v: int) -> bytes:
    return _str(1, name) + _vi(3, v) + _vi(20, 2)


def attr_float(name: str, v: float) -> bytes:
    return _str(1, name) + _key(2, 5) + struct.pack("<f", v) + _vi(20, 1)


def attr_ints(name: str, vs: list[int]) -> bytes:
    return _str(1, name) + b"".join(_vi(8, v) for v in vs) + _vi(20, 7)


def node(op: str, inputs: list[str], outputs: list[str], name: str = "", attrs: list[bytes] = (),
         domain: str = "") -> bytes:
    out = b"".join(_str(1, i) for i in inputs) + b"".join(_str(2, o) for o in outputs)
    if name:
        out += _str(3, name)
    out += _str(4, op) + b"".join(_ld(5, a) for a in attrs)
    if domain:
        out += _str(7, domain)
    return out


def model(nodes: list[bytes], initializers: list[bytes], inputs: list[str], outputs: list[str]) -> bytes:
    g = b"".join(_ld(1, n) for n in nodes) + _str(2, "g") + b"".join(_ld(5, t) for t in initializers)
    g += b"".join(_ld(11, _str(1, i)) for i in inputs) + b"".join(_ld(12, _str(1, o)) for o in outputs)
    opset = _str(1, "") + _vi(2, 17)
    return _vi(1, 8) + _ld(7, g) + _ld(8, opset)


def matmulnbits_model(case: dict, ext_dir=None, ext_file: str = "weights.bin") -> bytes:
    """One com.microsoft MatMulNBits node Y = MatMulNBits(A, B, scales[, zp]) with its weights as
    initializers; with ext_dir, B and the scales go to one external-data file (B after a 64-byte
    pad so the offsets are non-zero)."""
    b = np.ascontiguousarray(case["b"])
    s = np.ascontiguousarray(np.asarray(case["scales"]).reshape(case["N"], -1))
    inits = []
    if ext_dir is not None:
        pad = b"\0" * 64
        blob = pad + b.tobytes() + s.tobytes()
        (ext_dir / ext_file).write_bytes(blob)
        inits.append(tensor("B", b, external=(ext_file, 64, b.nbytes)))
        inits.append(tensor("scales", s, external=(ext_file, 64 + b.nbytes, s.nbytes)))
    else:
        inits += [tensor("B", b), tensor("scales", s)]
    ins = ["A", "B", "scales"]
    if case["zp"] is not None:
        inits.append(tensor("zp", np.ascontiguousarray(case["zp"])))
        ins.append("zp")
    attrs = [attr_int("K", case["K"]), attr_int("N", case["N"]), attr_int("bits", case["bits"]),
             attr_int("block_size", case["block_size"])]
    return model([node("MatMulNBits", ins, ["Y"], "mnb", attrs, domain="com.microsoft")], inits,
                 ["A", "B", "scales"], ["Y"])
