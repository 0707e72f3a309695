"""Operator plugin API mirror and the CUDA MatMulNBits kernel behind it.

The names and behaviour follow the reference's plugin seam so a graph dispatches the
node unchanged:

* IKernel        { op_type; execute(node, ctx) }        Cpu/Kernels/IKernel.cs:10-17
* KernelRegistry register (replaces by op type), try_get, create_default
                                                         Cpu/Kernels/KernelRegistry.cs:20-33,158
* GraphContext   get / get_tensor / has / set            Cpu/Kernels/GraphContext.cs:106-122
* GraphNode      (op_type, name, inputs, outputs, attrs)  Graph/GraphNode.cs:29-41
* CudaMatMulNBitsKernel  op type "MatMulNBits", the reference op's validation and output
                 shape (MatMulNBitsKernel.cs:77-169), executed by libms_cuda_nbits.so.

Values are torch tensors (numpy arrays are accepted and wrapped). A CUDA-resident A gives
a CUDA-resident Y on the same device; a host A runs through the host-buffer entry point.
"""
from __future__ import annotations

import ctypes as C
import threading
from dataclasses import dataclass, field
from typing import Any, Protocol

import numpy as np
import torch

from . import _native as N
from .errors import ModelSharpException
from .weights import QuantizedWeights, as_torch, dtype_code


@dataclass
class GraphNode:
    op_type: str
    name: str
    inputs: list[str]
    outputs: list[str]
    attributes: dict[str, Any] = field(default_factory=dict)


@dataclass
class ModelGraph:
    inputs: list[str]
    outputs: list[str]
    nodes: list[GraphNode]
    initializers: dict[str, Any] = field(default_factory=dict)


class GraphContext:
    """Named tensor environment of one graph run."""

    def __init__(self, values: dict[str, Any] | None = None):
        self.values: dict[str, Any] = dict(values or {})

    def get_tensor(self, name: str):
        if name not in self.values:
            raise ModelSharpException(f"Tensor '{name}' is not available in the execution context.")
        return self.values[name]

    def get(self, name: str):
        """Float view (fp16 / bf16 stay compact: the kernels widen them exactly, as
        GraphContext.Get does on the host, GraphContext.cs:106)."""
        t = as_torch(self.get_tensor(name))
        if t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ModelSharpException(f"Tensor '{name}' has dtype {t.dtype}; expected a float tensor.")
        return t

    def has(self, name: str) -> bool:
        return len(name) != 0 and name in self.values

    def set(self, name: str, value) -> None:
        self.values[name] = value


class IKernel(Protocol):
    op_type: str

    def preload(self, node: GraphNode, initializers: dict, device=None) -> int:
        """Load-time residency: validates the node and packs its B / scales / zero-point
        initializers on `device` now, so runs only move A and Y (IlgpuEngine.cs:3392-3429 keeps
        quantized initializers resident by name the same way). Returns 1 when it packed, 0 when
        that initializer triple was already resident."""
        names = node.inputs[1:4]
        b_raw, s_raw = initializers[names[0]], initializers[names[1]]
        zp_raw = initializers[names[2]] if len(names) > 2 and names[2] else None
        b = as_torch(b_raw)
        if b.dtype != torch.uint8:
            raise ModelSharpException(f"Tensor dtype is {_et_name(b)}; expected UInt8.")
        N_, K = _attr_int(node, "N", 0), _attr_int(node, "K", 0)
        bits, bs = _attr_int(node, "bits", 4), _attr_int(node, "block_size", 0)
        s_t, z_t = as_torch(s_raw), as_torch(zp_raw) if zp_raw is not None else None
        rc = N.lib().msq_check_node(N_, K, bits, bs, b.numel(), s_t.numel(),
                                    dtype_code(z_t) if z_t is not None else N.DT_ABSENT,
                                    z_t.numel() if z_t is not None else 0, None, 0,
                                    np.asarray([K], np.int64).ctypes.data, 1, None)
        N.check(rc, "MatMulNBits validation")
        dev = torch.device(device) if device is not None else (
            self.device or torch.device("cuda", torch.cuda.current_device()))
        key = (id(b_raw), id(s_raw), id(zp_raw) if zp_raw is not None else None, N_, K, bits, bs, str(dev))
        with self._lock:
            if key in self._cache:
                return 0
        self._weights(b_raw, s_raw, zp_raw, N_, K, bits, bs, dev)
        self.preloaded[tuple(names) + (str(dev),)] = key
        return 1

    def execute(self, node: GraphNode, ctx: GraphContext) -> None: ...


class KernelRegistry:
    def __init__(self):
        self._kernels: dict[str, IKernel] = {}

    def register(self, kernel: IKernel) -> "KernelRegistry":
        self._kernels[kernel.op_type] = kernel
        return self

    def try_get(self, op_type: str) -> tuple[bool, IKernel | None]:
        k = self._kernels.get(op_type)
        return k is not None, k

    @property
    def count(self) -> int:
        return len(self._kernels)

    @staticmethod
    def create_default(device: torch.device | int | str | None = None) -> "KernelRegistry":
        """The CUDA backend's registry (this backend implements MatMulNBits only)."""
        return KernelRegistry().register(CudaMatMulNBitsKernel(device))


def _attr_int(node: GraphNode, name: str, default: int) -> int:
    v = node.attributes.get(name, default)
    return int(np.int64(v).astype(np.int32))  # (int)Attr.Int(...) truncates to 32 bits


class CudaMatMulNBitsKernel:
    """com.microsoft.MatMulNBits on sm_100a.

    Weight initializers (B, scales, zero_points) are packed once per (tensor, device) and
    kept resident; later runs only move A and Y.
    """

    op_type = "MatMulNBits"

    def __init__(self, device: torch.device | int | str | None = None, path: int = N.PATH_AUTO):
        self.device = torch.device(device) if device is not None else None
        self.path = path
        self._cache: dict[tuple, QuantizedWeights] = {}
        self._lock = threading.Lock()
        self.calls = 0  # diagnostics, like NativeCuda.CtxCalls (NativeCuda.cs:147)
        self.preloaded: dict[tuple, tuple] = {}  # (B, scales, zp initializer names, device) -> cache key

    def _weights(self, b, scales, zp, N_, K, bits, bs, dev) -> QuantizedWeights:
        key = (id(b), id(scales), id(zp) if zp is not None else None, N_, K, bits, bs, str(dev))
        with self._lock:
            w = self._cache.get(key)
            if w is None:
                w = QuantizedWeights(b, scales, zp, N_, K, bits, bs, device=dev)
                # keep the source objects alive so their ids stay unique while cached
                w._sources = (b, scales, zp)
                self._cache[key] = w
            return w

    def preload(self, node: GraphNode, initializers: dict, device=None) -> int:
        """Load-time residency: validates the node and packs its B / scales / zero-point
        initializers on `device` now, so runs only move A and Y (IlgpuEngine.cs:3392-3429 keeps
        quantized initializers resident by name the same way). Returns 1 when it packed, 0 when
        that initializer triple was already resident."""
        names = node.inputs[1:4]
        b_raw, s_raw = initializers[names[0]], initializers[names[1]]
        zp_raw = initializers[names[2]] if len(names) > 2 and names[2] else None
        b = as_torch(b_raw)
        if b.dtype != torch.uint8:
            raise ModelSharpException(f"Tensor dtype is {_et_name(b)}; expected UInt8.")
        N_, K = _attr_int(node, "N", 0), _attr_int(node, "K", 0)
        bits, bs = _attr_int(node, "bits", 4), _attr_int(node, "block_size", 0)
        s_t, z_t = as_torch(s_raw), as_torch(zp_raw) if zp_raw is not None else None
        rc = N.lib().msq_check_node(N_, K, bits, bs, b.numel(), s_t.numel(),
                                    dtype_code(z_t) if z_t is not None else N.DT_ABSENT,
                                    z_t.numel() if z_t is not None else 0, None, 0,
                                    np.asarray([K], np.int64).ctypes.data, 1, None)
        N.check(rc, "MatMulNBits validation")
        dev = torch.device(device) if device is not None else (
            self.device or torch.device("cuda", torch.cuda.current_device()))
        key = (id(b_raw), id(s_raw), id(zp_raw) if zp_raw is not None else None, N_, K, bits, bs, str(dev))
        with self._lock:
            if key in self._cache:
                return 0
        self._weights(b_raw, s_raw, zp_raw, N_, K, bits, bs, dev)
        self.preloaded[tuple(names) + (str(dev),)] = key
        return 1

    def execute(self, node: GraphNode, ctx: GraphContext) -> None:
        a = ctx.get(node.inputs[0])
        b_raw = ctx.get_tensor(node.inputs[1])
        b = as_torch(b_raw)
        if b.dtype != torch.uint8:
            raise ModelSharpException(f"Tensor dtype is {_et_name(b)}; expected UInt8.")
        N_ = _attr_int(node, "N", 0)
        K = _attr_int(node, "K", 0)
        bits = _attr_int(node, "bits", 4)
        bs = _attr_int(node, "block_size", 0)
        scales_raw = ctx.get_tensor(node.inputs[2])
        scales = as_torch(scales_raw)
        zp_raw = None
        if len(node.inputs) > 3 and ctx.has(node.inputs[3]):
            zp_raw = ctx.get_tensor(node.inputs[3])
        zp = as_torch(zp_raw) if zp_raw is not None else None
        g_idx = None
        if len(node.inputs) > 4 and ctx.has(node.inputs[4]):
            g_idx = as_torch(ctx.get_tensor(node.inputs[4])).to(torch.int64).contiguous().cpu()
        dims = np.asarray(list(a.shape), dtype=np.int64)
        M = C.c_int64()
        lib = N.lib()
        rc = lib.msq_check_node(N_, K, bits, bs, b.numel(), scales.numel(),
                                dtype_code(zp) if zp is not None else N.DT_ABSENT,
                                zp.numel() if zp is not None else 0,
                                g_idx.data_ptr() if g_idx is not None else None,
                                g_idx.numel() if g_idx is not None else 0,
                                dims.ctypes.data if dims.size else None, int(dims.size), C.byref(M))
        N.check(rc, "MatMulNBits validation")
        dev = a.device if a.is_cuda else (self.device or torch.device("cuda", torch.cuda.current_device()))
        w = self._weights(b_raw, scales_raw, zp_raw, N_, K, bits, bs, dev)
        self.calls += 1
        if a.is_cuda:
            y = torch.empty(*a.shape[:-1], N_, dtype=torch.float32, device=a.device)
            w.matmul(a, out=y.view(-1, N_) if y.numel() else y, path=self.path, ldy=N_)
        else:
            y = torch.from_numpy(w.matmul_host(a))
        ctx.set(node.outputs[0], y)


def _et_name(t: torch.Tensor) -> str:
    return {torch.float32: "Float32", torch.float16: "Float16", torch.int64: "Int64", torch.int32: "Int32",
            torch.int8: "Int8", torch.float64: "Float64", torch.bool: "Boolean"}.get(t.dtype, str(t.dtype))
