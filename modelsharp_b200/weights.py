"""Device-resident MatMulNBits weights: a Python owner of one msq_weights_t handle.

Packing is the load-time repack of the reference layout (B uint8 [N, nb, blob], scales,
optional zero points) into the kernel layout; it happens once per initializer and device,
like IlgpuEngine's residency cache (src/ModelSharp.Gpu/IlgpuEngine.cs:2218-2229).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native as N
from .errors import ModelSharpException

_TORCH_DT = {
    torch.float32: N.DT_F32, torch.float64: N.DT_F64, torch.float16: N.DT_F16, torch.int32: N.DT_I32,
    torch.int64: N.DT_I64, torch.int8: N.DT_I8, torch.uint8: N.DT_U8, torch.bool: N.DT_BOOL,
    torch.bfloat16: N.DT_BF16,
}


def dtype_code(t) -> int:
    """C-ABI element-type code of a torch tensor / numpy array."""
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t))
    try:
        return _TORCH_DT[t.dtype]
    except KeyError:
        raise ModelSharpException(f"unsupported tensor dtype {t.dtype}") from None


def as_torch(x) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x
    return torch.from_numpy(np.ascontiguousarray(x))


def current_stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class QuantizedWeights:
    """Rows [n_begin, n_end) of one MatMulNBits weight, packed on a CUDA device."""

    def __init__(self, b, scales, zero_points, N_: int, K: int, bits: int = 4, block_size: int = 32,
                 rows: tuple[int, int] | None = None, device: torch.device | int | str | None = None,
                 generic_only: bool = False, lazy_gemm: bool = False):
        lib = N.lib()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            raise ModelSharpException(f"QuantizedWeights needs a CUDA device, got {dev}")
        n0, n1 = rows if rows is not None else (0, N_)
        b_t, s_t = as_torch(b), as_torch(scales)
        z_t = as_torch(zero_points) if zero_points is not None else None
        flags = (N.PACK_GENERIC_ONLY if generic_only else N.PACK_DEFAULT) | (N.PACK_LAZY_GEMM if lazy_gemm else 0)
        h = C.c_void_p()
        with torch.cuda.device(dev):
            on_dev = b_t.is_cuda
            if on_dev:
                b_t, s_t = b_t.contiguous(), s_t.contiguous()
                z_t = z_t.contiguous() if z_t is not None else None
                rc = lib.msq_pack(None, current_stream_ptr(dev), b_t.data_ptr(), b_t.numel(), s_t.data_ptr(),
                                  dtype_code(s_t), s_t.numel(), z_t.data_ptr() if z_t is not None else None,
                                  dtype_code(z_t) if z_t is not None else N.DT_ABSENT,
                                  z_t.numel() if z_t is not None else 0, N_, K, bits, block_size, n0, n1, flags,
                                  C.byref(h))
            else:
                b_t, s_t = b_t.contiguous(), s_t.contiguous()
                z_t = z_t.contiguous() if z_t is not None else None
                rc = lib.msq_pack_host(None, current_stream_ptr(dev), b_t.data_ptr(), b_t.numel(), s_t.data_ptr(),
                                       dtype_code(s_t), s_t.numel(), z_t.data_ptr() if z_t is not None else None,
                                       dtype_code(z_t) if z_t is not None else N.DT_ABSENT,
                                       z_t.numel() if z_t is not None else 0, N_, K, bits, block_size, n0, n1,
                                       flags, C.byref(h))
        N.check(rc, "msq_pack")
        self._h = h
        self.device = dev
        self.N_total, self.K, self.bits, self.block_size = N_, K, bits, block_size
        self.n_begin, self.n_end = n0, n1
        self.n_rows = n1 - n0
        nb_ = C.c_int64()
        lib.msq_weights_query(h, None, None, None, None, C.byref(nb_))
        self.device_bytes = nb_.value

    def query_device_bytes(self) -> int:
        """Device bytes the handle holds now (a lazy handle grows at its first GEMM call)."""
        nb_ = C.c_int64()
        N.check(N.lib().msq_weights_query(self.handle, None, None, None, None, C.byref(nb_)), "msq_weights_query")
        return nb_.value

    @property
    def handle(self) -> C.c_void_p:
        if self._h is None:
            raise ModelSharpException("QuantizedWeights used after free()")
        return self._h

    def matmul(self, a: torch.Tensor, out: torch.Tensor | None = None, path: int = N.PATH_AUTO,
               ldy: int | None = None, stream: int | None = None) -> torch.Tensor:
        """Y[..., j] = A[..., :] . W[n_begin + j, :] on A's device (enqueued, not synchronized)."""
        if not a.is_cuda:
            raise ModelSharpException("matmul expects a CUDA tensor; use matmul_host for host buffers")
        if a.shape[-1] != self.K:
            raise ModelSharpException(
                f"MatMulNBits A inner dimension must equal K={self.K}; got shape [{','.join(map(str, a.shape))}].")
        a = a.contiguous()
        M = a.numel() // self.K if self.K else 0
        if out is None:
            out = torch.empty(*a.shape[:-1], self.n_rows, dtype=torch.float32, device=a.device)
            ldy = self.n_rows
        elif ldy is None:
            ldy = out.stride(-2) if out.dim() >= 2 else self.n_rows
        with torch.cuda.device(a.device):
            st = current_stream_ptr(a.device) if stream is None else stream
            rc = N.lib().msq_matmul_ex(None, st, self.handle, a.data_ptr(), dtype_code(a), M, out.data_ptr(), ldy,
                                       path)
        N.check(rc, "msq_matmul")
        return out

    def matmul_fused(self, a: torch.Tensor, out: torch.Tensor, rms_gamma: torch.Tensor | None = None,
                     rms_eps: float = 1e-5, swiglu: bool = False, accumulate: bool = False,
                     stream: int | None = None) -> torch.Tensor:
        """The decode GEMV with glue folded in (msq_matmul_fused): A rows normalised by RMSNorm
        with `rms_gamma`, or A rows [gate | up] of 2K through SwiGLU; `accumulate` adds the
        product into `out`. fp32, M <= 16; enqueued, not synchronized."""
        kin = 2 * self.K if swiglu else self.K
        if a.dtype != torch.float32 or not a.is_cuda or a.shape[-1] != kin:
            raise ModelSharpException(f"matmul_fused expects a CUDA float32 A with rows of {kin}")
        a = a.contiguous()
        f = N.FusionT(rms_gamma.data_ptr() if rms_gamma is not None else None, rms_eps, int(swiglu), int(accumulate))
        with torch.cuda.device(a.device):
            st = current_stream_ptr(a.device) if stream is None else stream
            rc = N.lib().msq_matmul_fused(None, st, self.handle, a.data_ptr(), a.numel() // kin, out.data_ptr(),
                                          out.stride(-2) if out.dim() >= 2 else self.n_rows, C.byref(f))
        N.check(rc, "msq_matmul_fused")
        return out

    def matmul_host(self, a: np.ndarray | torch.Tensor) -> np.ndarray:
        """Host buffers in and out (copies inside the call), synchronous."""
        at = as_torch(a).contiguous()
        if at.shape[-1] != self.K:
            raise ModelSharpException(
                f"MatMulNBits A inner dimension must equal K={self.K}; got shape [{','.join(map(str, at.shape))}].")
        M = at.numel() // self.K
        y = np.empty((*at.shape[:-1], self.n_rows), dtype=np.float32)
        with torch.cuda.device(self.device):
            rc = N.lib().msq_matmul_host(None, current_stream_ptr(self.device), self.handle, at.data_ptr(),
                                         dtype_code(at), M, y.ctypes.data)
        N.check(rc, "msq_matmul_host")
        return y

    def free(self) -> None:
        if self._h is not None:
            N.lib().msq_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
