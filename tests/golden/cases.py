"""Seeded MatMulNBits cases shared by the golden-fixture generator and the tests.

Shapes and modes come from the reference's own tests and the baseline configurations;
values come from modelsharp_b200.synth (seeded splitmix64), since the reference's C#
System.Random / std::mt19937 streams are not reproduced here.
"""
from __future__ import annotations

from modelsharp_b200 import synth

# native/test/qgemm_test.cpp:259-276 -- M x N x K x bs grid over b4-sym, b4-asym, b8-sym,
# plus the extra 8-bit asymmetric case; A ~ U(-1,1), scales ~ U[0.005, 0.05).
QGEMM_GRID = [
    (M, N, K, bits, bs, zp)
    for bits, zp in ((4, "none"), (4, "packed"), (8, "none"))
    for M in (1, 8) for N in (64, 512) for K in (128, 4096) for bs in (32, 128)
] + [(8, 512, 4096, 8, 128, "packed")]

# The 4-bit cases of QGEMM_GRID, for the reference's ms_qgemm_w4a8 (native/test/qgemm_w4a8_test.cpp
# runs its own grid of the same kind).
W4A8_CASES = [i for i, g in enumerate(QGEMM_GRID) if g[3] == 4]

# GpuQuantizedLlmOpsTests.cs:326-339 -- (M, K, N, bits, block_size, zp form, seed);
# A ~ U(-1,1), scales 0.01 + 0.05 U, zero points 2^(bits-1) + U{-2..2} for the float form.
GPU_PARITY_GRID = [
    (1, 8, 4, 4, 8, "none", 1), (3, 16, 5, 4, 8, "none", 2), (4, 32, 6, 4, 16, "float", 3),
    (2, 24, 4, 4, 8, "packed", 4), (3, 16, 4, 8, 16, "none", 5), (4, 40, 5, 8, 16, "float", 6),
    (2, 32, 6, 8, 8, "packed", 7), (8, 64, 8, 4, 32, "none", 8), (1, 12, 3, 4, 4, "none", 9),
    (5, 20, 7, 4, 16, "float", 10),
]

# Baseline configurations at decode size (M = 1): the Qwen2.5-0.5B up-proj and the 7B sweep.
BASELINE_GEMV = [
    ("qwen_up", 1, 4864, 896, 32, 0.002, 0.02),
    ("7b_q", 1, 4096, 4096, 128, 0.001, 0.01),
    ("7b_kv", 1, 1024, 4096, 128, 0.001, 0.01),
    ("7b_up", 1, 14336, 4096, 128, 0.001, 0.01),
    ("7b_down", 1, 4096, 14336, 128, 0.001, 0.01),
    ("7b_lm_head", 1, 32000, 4096, 128, 0.001, 0.01),
]


def qgemm_case(i: int) -> dict:
    M, N, K, bits, bs, zp = QGEMM_GRID[i]
    return synth.make_case(1000 + i, M, N, K, bits, bs, zp, a_dist="uniform", scale_lo=0.005, scale_hi=0.05)


def gpu_parity_case(i: int) -> dict:
    M, K, N, bits, bs, zp, seed = GPU_PARITY_GRID[i]
    return synth.make_case(seed, M, N, K, bits, bs, zp, a_dist="uniform", scale_lo=0.01, scale_hi=0.06)


def baseline_case(i: int, M: int | None = None) -> dict:
    name, M0, N, K, bs, lo, hi = BASELINE_GEMV[i]
    return synth.make_case(i, M if M is not None else M0, N, K, 4, bs, "packed", a_dist="normal",
                           scale_lo=lo, scale_hi=hi)
