"""Deterministic synthetic inputs for MatMulNBits in the reference's layouts.

Every value is a pure function of (seed, tag, index) through splitmix64, so the same
inputs can be regenerated bit-for-bit on any host (the tests' fixtures store seeds,
not megabytes of weights). Layouts follow the reference op:

* A      float [M, K]                        (MatMulNBitsKernel.cs:157-164)
* B      uint8 [N, n_blocks, blob]           blob = ceil(bs*bits/8), low nibble = even k
                                             (MatMulNBitsKernel.cs:26-30, 95-104)
* scales float [N * n_blocks]                (MatMulNBitsKernel.cs:106-112)
* zp     uint8 [N, ceil(n_blocks*bits/8)]    packed like B, or float [N * n_blocks]
                                             (MatMulNBitsKernel.cs:114-145)

Bytes of B past K in a ragged last block, and the unused high nibble of an odd packed
zero-point row, are filled with random codes on purpose: the op must ignore them.
"""
from __future__ import annotations

import zlib

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _C1
        z = (z ^ (z >> np.uint64(27))) * _C2
        return z ^ (z >> np.uint64(31))


def _key(seed: int, tag: str) -> np.uint64:
    mix = (int(seed) * 0x100000001B3 ^ zlib.crc32(tag.encode())) & ((1 << 64) - 1)
    return _splitmix64(np.array([mix], dtype=np.uint64))[0]


def random_u64(seed: int, tag: str, n: int) -> np.ndarray:
    """n pseudo-random uint64 words of stream (seed, tag)."""
    base = _key(seed, tag)
    with np.errstate(over="ignore"):
        idx = np.arange(n, dtype=np.uint64) + base
    return _splitmix64(idx)


def random_bytes(seed: int, tag: str, n: int) -> np.ndarray:
    words = random_u64(seed, tag, (n + 7) // 8)
    return words.view(np.uint8)[:n].copy()


def uniform(seed: int, tag: str, n: int, lo: float, hi: float) -> np.ndarray:
    """float32 uniform on [lo, hi) from 24-bit grid points."""
    u = (random_u64(seed, tag, n) >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))
    return (lo + (hi - lo) * u).astype(np.float32)


def normal(seed: int, tag: str, n: int) -> np.ndarray:
    """float32 N(0, 1) by Box-Muller over two independent streams."""
    u1 = ((random_u64(seed, tag + "/u1", n) >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0**-53
    u2 = (random_u64(seed, tag + "/u2", n) >> np.uint64(11)).astype(np.float64) * 2.0**-53
    return (np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)).astype(np.float32)


def geometry(K: int, bits: int, block_size: int) -> tuple[int, int, int]:
    """(n_blocks_per_row, blob_size, zp_row_bytes) as MatMulNBitsKernel.cs:95-96,118."""
    nb = (K + block_size - 1) // block_size
    blob = (block_size * bits + 7) // 8
    zp_row = (nb * bits + 7) // 8
    return nb, blob, zp_row


def make_case(seed: int, M: int, N: int, K: int, bits: int = 4, block_size: int = 32,
              zp_kind: str = "packed", a_dist: str = "normal",
              scale_lo: float = 0.002, scale_hi: float = 0.02,
              a_dtype: str = "f32", scale_dtype: str = "f32") -> dict:
    """One MatMulNBits problem in the reference layouts.

    zp_kind: "none" (symmetric default), "packed" (uint8 n-bit), "float" (float32,
    2^(bits-1) + U{-2..2} as the reference's GPU parity tests draw them,
    GpuQuantizedLlmOpsTests.cs:172-176). a_dist: "normal" (N(0,1)) or "uniform" (U(-1,1)).
    a_dtype / scale_dtype: "f32" or "f16" (fp16 values are what the op sees; the
    reference widens them exactly, GraphContext.cs:106).
    """
    nb, blob, zp_row = geometry(K, bits, block_size)
    if a_dist == "normal":
        a = normal(seed, "A", M * K)
    else:
        a = uniform(seed, "A", M * K, -1.0, 1.0)
    a = a.reshape(M, K)
    b = random_bytes(seed, "B", N * nb * blob).reshape(N, nb, blob)
    if bits == 8:
        pass  # one code per byte, all 0..255
    scales = uniform(seed, "scales", N * nb, scale_lo, scale_hi)
    if a_dtype == "f16":
        a = a.astype(np.float16)
    if scale_dtype == "f16":
        scales = scales.astype(np.float16)
    zp = None
    if zp_kind == "packed":
        zp = random_bytes(seed, "zp", N * zp_row).reshape(N, zp_row)
    elif zp_kind == "float":
        centre = float(1 << (bits - 1))
        off = (random_u64(seed, "zpf", N * nb) % np.uint64(5)).astype(np.float32) - 2.0
        zp = (centre + off).astype(np.float32)
    elif zp_kind != "none":
        raise ValueError(zp_kind)
    return dict(a=a, b=b, scales=scales, zp=zp, zp_kind=zp_kind, M=M, N=N, K=K,
                bits=bits, block_size=block_size)


def algorithmic_bytes(N: int, K: int, bits: int, block_size: int, zp_kind: str,
                      scale_bytes: int = 4) -> int:
    """Weight + scale + zero-point bytes of one op as the reference stores them."""
    nb, blob, zp_row = geometry(K, bits, block_size)
    zb = {"none": 0, "packed": N * zp_row, "float": N * nb * 4}[zp_kind]
    return N * nb * blob + N * nb * scale_bytes + zb
