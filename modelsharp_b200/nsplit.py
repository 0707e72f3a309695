"""Column split of one MatMulNBits weight across GPUs, one process per GPU.

Output columns of MatMulNBits are independent: Y[..., n] reads only row n of B, scales and
zero points (src/ModelSharp/Cpu/Kernels/Quantize/MatMulNBitsKernel.cs:211-215). Rank p of a
process group of P ranks packs rows [n0, n1) of the weight on its own GPU, computes
Y[:, n0:n1] with the local kernel, and an all-gather of the shards assembles the full Y on
every rank, ready to be the next layer's replicated input.

Shards are contiguous, `align` rows (a multiple of the 16-row record block) per rank except
at the end: with chunk = align * ceil(N / (P * align)), rank p owns rows
[min(N, p * chunk), min(N, (p + 1) * chunk)).

Two ways to assemble Y:

* "p2p" (decode, M <= 4, one CUDA device per rank): the shard's decode GEMV stores its
  outputs straight into every rank's full-Y buffer over NVLink and signals every rank
  (msq_matmul_gather); a later call that reads the gathered Y waits on the device, bounded,
  for all ranks' shards (pass `wait=producer.out_wait`; host readers call `wait_gathered`).
  The buffers are shared between the rank processes with CUDA IPC.
* "nccl" (any M, any backend): every rank computes into a zero-padded [M, chunk] buffer and
  an all-gather makes [P, M, chunk], moved to [M, P * chunk] and cut at N.
"""
from __future__ import annotations

from typing import Callable

import ctypes as C

import torch
import torch.distributed as dist

from . import _native as NAT
from .errors import ModelSharpException
from .weights import QuantizedWeights, current_stream_ptr, dtype_code

LocalCompute = Callable[[torch.Tensor, int, int], torch.Tensor]


def shard_bounds(n: int, parts: int, align: int = 128) -> tuple[list[tuple[int, int]], int]:
    """Row ranges of `parts` contiguous shards of `n` rows, `align`-row granular, and the chunk size."""
    if n <= 0 or parts <= 0 or align <= 0:
        raise ModelSharpException(f"shard_bounds needs positive sizes (n={n}, parts={parts}, align={align})")
    chunk = -(-n // (parts * align)) * align
    return [(min(n, p * chunk), min(n, (p + 1) * chunk)) for p in range(parts)], chunk


class _DeviceView:
    """A raw device buffer as a torch tensor (CUDA array interface, no copy)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


class _Exchange:
    """Full-Y buffers (two, used alternately) and counters of one layer on this rank, with
    every other rank's mapped in through CUDA IPC."""

    CTRL_BYTES = 64  # arrivals u64 @0, produced u64 @8, done u32 @16

    def __init__(self, n: int, col0: int, rank: int, world: int, group, device: torch.device, max_m: int = 4):
        lib = NAT.lib()
        self.n, self.max_m, self.device = n, max_m, device
        self.own: list[int] = []
        self.opened: list[int] = []
        with torch.cuda.device(device):
            for nbytes in (max_m * n * 4, max_m * n * 4, self.CTRL_BYTES):
                ptr = C.c_void_p()
                NAT.check(lib.msq_xbuf_alloc(None, nbytes, C.byref(ptr)), "msq_xbuf_alloc")
                self.own.append(ptr.value)
            mine = []
            for ptr in self.own:
                h = (C.c_ubyte * NAT.IPC_HANDLE_BYTES)()
                NAT.check(lib.msq_ipc_handle(None, C.c_void_p(ptr), h), "msq_ipc_handle")
                mine.append(bytes(h))
            everyone = [None] * world
            if world > 1:
                dist.all_gather_object(everyone, mine, group=group)
            else:
                everyone = [mine]
            ptrs = []  # [rank][y0, y1, ctrl]
            for r in range(world):
                if r == rank:
                    ptrs.append(list(self.own))
                    continue
                row = []
                for hb in everyone[r]:
                    out = C.c_void_p()
                    h = (C.c_ubyte * NAT.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                    NAT.check(lib.msq_ipc_open(None, h, C.byref(out)), "msq_ipc_open")
                    row.append(out.value)
                    self.opened.append(out.value)
                ptrs.append(row)
        ctrl = self.own[2]
        self.gathers = []
        for parity in (0, 1):
            g = NAT.GatherT()
            g.nranks, g.rank, g.ldy, g.col0 = world, rank, n, col0
            for r in range(world):
                g.y[r] = ptrs[r][parity]
                g.arrivals[r] = ptrs[r][2]
            g.produced, g.done = ctrl + 8, ctrl + 16
            self.gathers.append(g)
        self.wait = NAT.WaitT()
        self.wait.arrivals, self.wait.produced, self.wait.nranks = ctrl, ctrl + 8, world
        self.parity = 0
        if world > 1:
            dist.barrier(group=group)  # every rank's counters are zero before anyone signals

    def output(self, parity: int, m: int) -> torch.Tensor:
        return torch.as_tensor(_DeviceView(self.own[parity], (self.max_m, self.n)), device=self.device)[:m]

    def close(self) -> None:
        lib = NAT.lib()
        with torch.cuda.device(self.device):
            for ptr in self.opened:
                lib.msq_ipc_close(None, C.c_void_p(ptr))
            for ptr in self.own:
                lib.msq_xbuf_free(None, C.c_void_p(ptr))
        self.opened, self.own = [], []


class ShardedMatMulNBits:
    """One MatMulNBits weight split by output rows over the ranks of `group`.

    `b`, `scales`, `zero_points` are the whole weight in the reference layouts (host or device
    tensors; every rank passes the same values). Without an initialised process group the
    split has one part. `local` replaces the CUDA kernel for the shard (signature
    `local(a2d, n0, n1) -> [M, n1 - n0]`), which lets the host logic run on CPU ranks.
    """

    def __init__(self, b, scales, zero_points, N: int, K: int, bits: int = 4, block_size: int = 32,
                 group: dist.ProcessGroup | None = None, device: torch.device | str | int | None = None,
                 align: int = 128, local: LocalCompute | None = None, gather: str = "nccl"):
        if dist.is_available() and dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        self.group = group
        self.N, self.K = N, K
        self.bounds, self.chunk = shard_bounds(N, self.world, align)
        self.n0, self.n1 = self.bounds[self.rank]
        self._local = local
        self.weights: QuantizedWeights | None = None
        if local is None:
            dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
            self.device = dev
            if self.n1 > self.n0:
                self.weights = QuantizedWeights(b, scales, zero_points, N, K, bits, block_size,
                                                rows=(self.n0, self.n1), device=dev)
        else:
            self.device = torch.device("cpu") if device is None else torch.device(device)
        if gather not in ("nccl", "p2p"):
            raise ModelSharpException(f"gather must be 'nccl' or 'p2p', got {gather!r}")
        self.exchange: _Exchange | None = None
        self.out_wait: NAT.WaitT | None = None
        if gather == "p2p":
            if local is not None or self.weights is None:
                raise ModelSharpException("the p2p gather needs a CUDA shard with at least one row on every rank")
            self.exchange = _Exchange(N, self.n0, self.rank, self.world, group, self.device)

    def local_shard(self, a2: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's columns, zero-padded to [M, chunk]."""
        M = a2.shape[0]
        y = torch.zeros(M, self.chunk, dtype=torch.float32, device=a2.device) if out is None else out
        rows = self.n1 - self.n0
        if rows > 0:
            if self._local is not None:
                y[:, :rows] = self._local(a2, self.n0, self.n1)
            else:
                self.weights.matmul(a2, out=y, ldy=self.chunk)
        return y

    def gather(self, y_local: torch.Tensor) -> torch.Tensor:
        """All-gather of the [M, chunk] shards into Y [M, N] on every rank."""
        M = y_local.shape[0]
        if self.world == 1:
            full = y_local.view(1, M, self.chunk)
        elif dist.get_backend(self.group) == "nccl":
            full = torch.empty(self.world * M * self.chunk, dtype=y_local.dtype, device=y_local.device)
            dist.all_gather_into_tensor(full, y_local.reshape(-1), group=self.group)
            full = full.view(self.world, M, self.chunk)
        else:
            parts = [torch.empty_like(y_local) for _ in range(self.world)]
            dist.all_gather(parts, y_local.contiguous(), group=self.group)
            full = torch.stack(parts)
        if M == 1:
            return full.reshape(1, self.world * self.chunk)[:, :self.N]
        return full.permute(1, 0, 2).reshape(M, self.world * self.chunk)[:, :self.N]

    def __call__(self, a: torch.Tensor, wait: NAT.WaitT | None = None) -> torch.Tensor:
        """Y = A . W^T assembled on every rank. With the p2p gather and M <= 4 the result is a
        view of this rank's full-Y buffer that stays valid until the call after next; `wait` is
        the `out_wait` of the sharded op that produced A when A is such a view."""
        if a.shape[-1] != self.K:
            raise ModelSharpException(
                f"MatMulNBits A inner dimension must equal K={self.K}; got shape [{','.join(map(str, a.shape))}].")
        a2 = a.reshape(-1, self.K)
        M = a2.shape[0]
        if self.exchange is not None and 1 <= M <= self.exchange.max_m and a2.is_cuda:
            a2 = a2.contiguous()
            ex = self.exchange
            par = ex.parity
            ex.parity ^= 1
            with torch.cuda.device(self.device):
                rc = NAT.lib().msq_matmul_gather(None, current_stream_ptr(self.device), self.weights.handle,
                                               a2.data_ptr(), dtype_code(a2), M,
                                               C.byref(wait) if wait is not None else None, C.byref(ex.gathers[par]))
            NAT.check(rc, "msq_matmul_gather")
            self.out_wait = ex.wait
            y = ex.output(par, M)
        else:
            if wait is not None:
                self._wait(wait)
            y = self.gather(self.local_shard(a2))
            self.out_wait = None
        return y.reshape(*a.shape[:-1], self.N)

    def _wait(self, wait: NAT.WaitT) -> None:
        with torch.cuda.device(self.device):
            NAT.check(NAT.lib().msq_wait_gathered(None, current_stream_ptr(self.device), C.byref(wait)),
                    "msq_wait_gathered")

    def wait_gathered(self) -> None:
        """Orders the current stream after the latest p2p-gathered output (for host copies and
        other readers outside this library)."""
        if self.out_wait is not None:
            self._wait(self.out_wait)

    def free(self) -> None:
        if self.exchange is not None:
            if self.world > 1:
                torch.cuda.synchronize(self.device)
                dist.barrier(group=self.group)  # no rank still writes into the buffers
            self.exchange.close()
            self.exchange = None
        if self.weights is not None:
            self.weights.free()
            self.weights = None
