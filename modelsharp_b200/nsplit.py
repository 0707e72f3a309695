"""Column split of one MatMulNBits weight across GPUs, one process per GPU.

Output columns of MatMulNBits are independent: Y[..., n] reads only row n of B, scales and
zero points (src/ModelSharp/Cpu/Kernels/Quantize/MatMulNBitsKernel.cs:211-215). Rank p of a
process group of P ranks packs rows [n0, n1) of the weight on its own GPU, computes
Y[:, n0:n1] with the local kernel, and an all-gather of the shards assembles the full Y on
every rank, ready to be the next layer's replicated input.

Shards are contiguous, `align` rows (a multiple of the 16-row record block) per rank except
at the end: with chunk = align * ceil(N / (P * align)), rank p owns rows
[min(N, p * chunk), min(N, (p + 1) * chunk)). Every rank computes into a zero-padded
[M, chunk] buffer so the gathered [P, M, chunk] tensor, moved to [M, P * chunk] and cut at N,
is Y.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .errors import ModelSharpException
from .weights import QuantizedWeights

LocalCompute = Callable[[torch.Tensor, int, int], torch.Tensor]


def shard_bounds(n: int, parts: int, align: int = 128) -> tuple[list[tuple[int, int]], int]:
    """Row ranges of `parts` contiguous shards of `n` rows, `align`-row granular, and the chunk size."""
    if n <= 0 or parts <= 0 or align <= 0:
        raise ModelSharpException(f"shard_bounds needs positive sizes (n={n}, parts={parts}, align={align})")
    chunk = -(-n // (parts * align)) * align
    return [(min(n, p * chunk), min(n, (p + 1) * chunk)) for p in range(parts)], chunk


class ShardedMatMulNBits:
    """One MatMulNBits weight split by output rows over the ranks of `group`.

    `b`, `scales`, `zero_points` are the whole weight in the reference layouts (host or device
    tensors; every rank passes the same values). Without an initialised process group the
    split has one part. `local` replaces the CUDA kernel for the shard (signature
    `local(a2d, n0, n1) -> [M, n1 - n0]`), which lets the host logic run on CPU ranks.
    """

    def __init__(self, b, scales, zero_points, N: int, K: int, bits: int = 4, block_size: int = 32,
                 group: dist.ProcessGroup | None = None, device: torch.device | str | int | None = None,
                 align: int = 128, local: LocalCompute | None = None):
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

    def __call__(self, a: torch.Tensor) -> torch.Tensor:
        if a.shape[-1] != self.K:
            raise ModelSharpException(
                f"MatMulNBits A inner dimension must equal K={self.K}; got shape [{','.join(map(str, a.shape))}].")
        a2 = a.reshape(-1, self.K)
        y = self.gather(self.local_shard(a2))
        return y.reshape(*a.shape[:-1], self.N)

    def free(self) -> None:
        if self.weights is not None:
            self.weights.free()
            self.weights = None
