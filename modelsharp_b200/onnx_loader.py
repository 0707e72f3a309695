"""ONNX model loading for the CUDA backend: a protobuf reader of its own (no onnx package),
and load-time residency of MatMulNBits weights.

`load_model(path)` / `parse_model(bytes)` read a ModelProto into a ModelGraph with the fields
and rules of the reference's loader (src/ModelSharp/Onnx/OnnxModelLoader.cs):

* ModelProto.graph (field 7); GraphProto node (1), initializer (5), input (11), output (12);
  graph inputs that are initializers are not feeds (:77-121).
* NodeProto input (1), output (2), name (3, the op type when empty), op_type (4),
  attribute (5); AttributeProto name (1), f (2), i (3), s (4), floats (7), ints (8), type (20)
  (:142-231).
* TensorProto dims (1), data_type (2), float_data (4), int32_data (5), int64_data (7),
  name (8), raw_data (9), external_data (13), data_location (14) (:236-360); element types
  FLOAT, UINT8, INT8, INT32, INT64, BOOL, FLOAT16 (kept as float16: the kernels widen it
  exactly) and BFLOAT16 (widened to float32 as the reference does) (:364-436).
* External data (data_location = 1): the `location` file relative to the model's directory,
  `offset` and `length` (to the end of the file when absent) (:23-27, 439-520). The file is
  memory-mapped and each initializer is a view of its byte range, so a packed weight goes from
  the mapping straight to the device without another host copy.

`preload_matmulnbits(graph, kernel, device)` packs the weights of every MatMulNBits node whose
B, scales and zero points are initializers, once, at load: the residency role of
IlgpuEngine.ResidentOrTempInt (src/ModelSharp.Gpu/IlgpuEngine.cs:3392-3429), keyed by the
initializer names; CudaEngine(graph, preload=True) calls it.
"""
from __future__ import annotations

import mmap
import os
import struct
from pathlib import Path

import numpy as np

from .errors import ModelSharpException
from .kernels import GraphNode, ModelGraph

DT_FLOAT, DT_UINT8, DT_INT8, DT_INT32, DT_INT64, DT_BOOL, DT_FLOAT16, DT_BFLOAT16 = 1, 2, 3, 6, 7, 9, 10, 16
_NP = {DT_FLOAT: np.float32, DT_UINT8: np.uint8, DT_INT8: np.int8, DT_INT32: np.int32, DT_INT64: np.int64,
       DT_BOOL: np.bool_, DT_FLOAT16: np.float16, DT_BFLOAT16: np.uint16}


class _Reader:
    """Protobuf wire-format reader over a buffer (varint, 64-bit, length-delimited, 32-bit)."""

    def __init__(self, buf, start: int = 0, end: int | None = None):
        self.b = buf
        self.p = start
        self.end = len(buf) if end is None else end

    def more(self) -> bool:
        return self.p < self.end

    def varint(self) -> int:
        v, shift = 0, 0
        while True:
            if self.p >= self.end:
                raise ModelSharpException("Truncated varint in ONNX protobuf.")
            c = self.b[self.p]
            self.p += 1
            v |= (c & 0x7F) << shift
            if c < 0x80:
                return v
            shift += 7
            if shift > 63:
                raise ModelSharpException("Malformed varint in ONNX protobuf.")

    def tag(self) -> tuple[int, int]:
        t = self.varint()
        return t >> 3, t & 7

    def int64(self) -> int:
        v = self.varint()
        return v - (1 << 64) if v >= 1 << 63 else v

    def span(self) -> tuple[int, int]:
        n = self.varint()
        if self.p + n > self.end:
            raise ModelSharpException("Length-delimited field runs past the end of the ONNX protobuf.")
        s = self.p
        self.p += n
        return s, s + n

    def fixed32(self) -> bytes:
        v = bytes(self.b[self.p:self.p + 4])
        self.p += 4
        return v

    def skip(self, wire: int) -> None:
        if wire == 0:
            self.varint()
        elif wire == 1:
            self.p += 8
        elif wire == 2:
            self.span()
        elif wire == 5:
            self.p += 4
        else:
            raise ModelSharpException(f"Unsupported protobuf wire type {wire} in ONNX model.")


def _string(buf, s: int, e: int) -> str:
    return bytes(buf[s:e]).decode("utf-8")


def _packed_varints(buf, s: int, e: int, signed: bool = True) -> list[int]:
    r = _Reader(buf, s, e)
    return [r.int64() if signed else r.varint() for _ in iter(r.more, False)]


class _External:
    """Memory maps of the external-data files of one load, each opened once."""

    def __init__(self, base_dir: str | None):
        self.base_dir = base_dir
        self.maps: dict[str, mmap.mmap] = {}

    def read(self, location: str, offset: int, length: int, name: str) -> memoryview:
        if self.base_dir is None:
            raise ModelSharpException(
                f"Initializer '{name}' references external data file '{location}', but the model was parsed from an "
                "in-memory byte buffer with no base directory; load it from a file path (load_model) so external "
                "data can be resolved.")
        path = os.path.normpath(os.path.join(self.base_dir, location))
        m = self.maps.get(path)
        if m is None:
            if not os.path.isfile(path):
                raise ModelSharpException(f"External data file '{location}' for initializer '{name}' was not found.")
            with open(path, "rb") as f:
                m = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) if os.path.getsize(path) else b""
            self.maps[path] = m
        end = len(m) if length < 0 else offset + length
        if offset < 0 or end > len(m):
            raise ModelSharpException(
                f"External data range [{offset}, {end}) of initializer '{name}' is outside '{location}' "
                f"({len(m)} bytes).")
        return memoryview(m)[offset:end]


def _tensor(buf, s: int, e: int, ext: _External) -> tuple[str, np.ndarray]:
    dims: list[int] = []
    dt = 0
    name = ""
    raw = None
    floats: list[float] = []
    i32: list[int] = []
    i64: list[int] = []
    loc, off, length, data_location = None, 0, -1, 0
    r = _Reader(buf, s, e)
    while r.more():
        f, w = r.tag()
        if f == 1 and w == 0:
            dims.append(r.int64())
        elif f == 1 and w == 2:
            dims.extend(_packed_varints(buf, *r.span()))
        elif f == 2 and w == 0:
            dt = r.int64()
        elif f == 4 and w == 5:
            floats.append(struct.unpack("<f", r.fixed32())[0])
        elif f == 4 and w == 2:
            a, b = r.span()
            floats.extend(np.frombuffer(bytes(buf[a:b]), dtype="<f4").tolist())
        elif f == 5 and w == 0:
            i32.append(r.int64())
        elif f == 5 and w == 2:
            i32.extend(_packed_varints(buf, *r.span()))
        elif f == 7 and w == 0:
            i64.append(r.int64())
        elif f == 7 and w == 2:
            i64.extend(_packed_varints(buf, *r.span()))
        elif f == 8 and w == 2:
            name = _string(buf, *r.span())
        elif f == 9 and w == 2:
            a, b = r.span()
            raw = memoryview(buf)[a:b]
        elif f == 13 and w == 2:  # StringStringEntryProto: key 1, value 2
            ka, kb = r.span()
            er = _Reader(buf, ka, kb)
            key = val = ""
            while er.more():
                ff, ww = er.tag()
                if ff in (1, 2) and ww == 2:
                    txt = _string(buf, *er.span())
                    key, val = (txt, val) if ff == 1 else (key, txt)
                else:
                    er.skip(ww)
            if key == "location":
                loc = val
            elif key == "offset":
                off = int(val)
            elif key == "length":
                length = int(val)
        elif f == 14 and w == 0:
            data_location = r.int64()
        else:
            r.skip(w)
    if data_location == 1:
        if loc is None:
            raise ModelSharpException(f"Initializer '{name}' is EXTERNAL but has no 'location' in external_data.")
        raw = ext.read(loc, off, length, name)
    if dt == 0:
        dt = DT_INT64 if i64 else DT_INT32 if i32 else DT_FLOAT
    if dt not in _NP:
        raise ModelSharpException(f"Initializer '{name}' has unsupported ONNX data type {dt}.")
    count = int(np.prod(dims, dtype=np.int64)) if dims else 1
    npdt = np.dtype(_NP[dt])
    if raw is not None:
        if len(raw) < count * npdt.itemsize:
            raise ModelSharpException(
                f"Initializer '{name}' declares {count} elements but holds {len(raw)} bytes of data.")
        arr = np.frombuffer(raw, dtype=npdt.newbyteorder("<"), count=count)
    elif dt == DT_FLOAT:
        arr = np.asarray(floats[:count], dtype=np.float32)
    elif dt == DT_INT64:
        arr = np.asarray(i64[:count], dtype=np.int64)
    else:  # int32_data carries uint8 / int8 / int32 / bool / 16-bit float bit patterns
        arr = np.asarray(i32[:count], dtype=np.int64).astype(np.uint16 if dt in (DT_FLOAT16, DT_BFLOAT16) else npdt)
        if dt == DT_FLOAT16:
            arr = arr.view(np.float16)
    if arr.size != count:
        raise ModelSharpException(f"Initializer '{name}' declares {count} elements but holds {arr.size}.")
    if dt == DT_BFLOAT16:
        arr = (arr.astype(np.uint32) << 16).view(np.float32)
    return name, arr.reshape(dims) if dims else arr.reshape(())


def _attribute(buf, s: int, e: int, ext: _External):
    name, typ = "", 0
    f_val = i_val = s_val = t_val = None
    ints: list[int] | None = None
    floats: list[float] | None = None
    r = _Reader(buf, s, e)
    while r.more():
        f, w = r.tag()
        if f == 1 and w == 2:
            name = _string(buf, *r.span())
        elif f == 20 and w == 0:
            typ = r.int64()
        elif f == 2 and w == 5:
            f_val = struct.unpack("<f", r.fixed32())[0]
        elif f == 3 and w == 0:
            i_val = r.int64()
        elif f == 4 and w == 2:
            s_val = _string(buf, *r.span())
        elif f == 5 and w == 2:
            t_val = _tensor(buf, *r.span(), ext)[1]
        elif f == 7 and w == 5:
            (floats := floats or []).append(struct.unpack("<f", r.fixed32())[0])
        elif f == 7 and w == 2:
            a, b = r.span()
            floats = (floats or []) + np.frombuffer(bytes(buf[a:b]), dtype="<f4").tolist()
        elif f == 8 and w == 0:
            (ints := ints or []).append(r.int64())
        elif f == 8 and w == 2:
            ints = (ints or []) + _packed_varints(buf, *r.span())
        else:
            r.skip(w)
    by_type = {1: f_val, 2: i_val, 3: s_val, 4: t_val, 6: floats, 7: ints}
    if typ in by_type:
        return name, by_type[typ]
    for v in (ints, floats, i_val, f_val, s_val, t_val):  # type unset: whichever field was present
        if v is not None:
            return name, v
    return name, None


def _node(buf, s: int, e: int, ext: _External) -> GraphNode:
    inputs, outputs, name, op, attrs = [], [], "", "", {}
    r = _Reader(buf, s, e)
    while r.more():
        f, w = r.tag()
        if f == 1 and w == 2:
            inputs.append(_string(buf, *r.span()))
        elif f == 2 and w == 2:
            outputs.append(_string(buf, *r.span()))
        elif f == 3 and w == 2:
            name = _string(buf, *r.span())
        elif f == 4 and w == 2:
            op = _string(buf, *r.span())
        elif f == 5 and w == 2:
            an, av = _attribute(buf, *r.span(), ext)
            if av is not None:
                attrs[an] = av
        else:
            r.skip(w)
    return GraphNode(op, name or op, inputs, outputs, attrs)


def _value_info_name(buf, s: int, e: int) -> str:
    r = _Reader(buf, s, e)
    while r.more():
        f, w = r.tag()
        if f == 1 and w == 2:
            return _string(buf, *r.span())
        r.skip(w)
    return ""


def _graph(buf, s: int, e: int, ext: _External) -> ModelGraph:
    nodes, inits, ins, outs = [], {}, [], []
    r = _Reader(buf, s, e)
    while r.more():
        f, w = r.tag()
        if f == 1 and w == 2:
            nodes.append(_node(buf, *r.span(), ext))
        elif f == 5 and w == 2:
            n, t = _tensor(buf, *r.span(), ext)
            inits[n] = t
        elif f == 11 and w == 2:
            ins.append(_value_info_name(buf, *r.span()))
        elif f == 12 and w == 2:
            outs.append(_value_info_name(buf, *r.span()))
        else:
            r.skip(w)
    return ModelGraph([n for n in ins if n not in inits], outs, nodes, inits)


def parse_model(data, base_dir: str | None = None) -> ModelGraph:
    """A ModelProto from bytes; external data resolves against `base_dir` (None: an error)."""
    buf = memoryview(data).cast("B") if not isinstance(data, (bytes, bytearray)) else data
    ext = _External(base_dir)
    r = _Reader(buf)
    span = None
    while r.more():
        f, w = r.tag()
        if f == 7 and w == 2:
            span = r.span()
        else:
            r.skip(w)
    if span is None:
        raise ModelSharpException("ONNX model contains no graph (field 7).")
    g = _graph(buf, *span, ext)
    g._external = ext  # keeps the memory maps the initializers view alive with the graph
    return g


def load_model(path: str | os.PathLike) -> ModelGraph:
    """An ONNX file, with external-data initializers resolved next to it."""
    p = Path(path)
    return parse_model(p.read_bytes(), base_dir=str(p.resolve().parent))


def preload_matmulnbits(graph: ModelGraph, kernel, device) -> int:
    """Packs the device weights of every MatMulNBits node whose B / scales / zero points are
    initializers (once per initializer-name triple and device); returns how many were packed."""
    n = 0
    for node in graph.nodes:
        if node.op_type != "MatMulNBits":
            continue
        names = node.inputs[1:4]
        if len(names) < 2 or not all(x in graph.initializers for x in names if x):
            continue
        n += kernel.preload(node, graph.initializers, device)
    return n
