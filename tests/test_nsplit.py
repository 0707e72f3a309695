"""Column split across ranks (host logic): shard bounds, gather and re-assembly of Y.

Two `gloo` ranks on CPU stand in for two GPUs; each rank's shard is computed by the parity
checker on its rows, so the assembled Y must equal the checker's result on the whole weight
bit for bit (each output column is computed from its own row alone). The CUDA shard runs in
the GPU test below at one rank.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from modelsharp_b200 import synth
from modelsharp_b200.nsplit import ShardedMatMulNBits, shard_bounds


@pytest.mark.parametrize("n,parts,align", [(4096, 2, 128), (28672, 8, 128), (8192, 8, 128), (1000, 2, 16),
                                           (1000, 4, 128), (100, 8, 16), (1, 2, 16)])
def test_shard_bounds_cover_rows(n, parts, align):
    bounds, chunk = shard_bounds(n, parts, align)
    assert chunk % align == 0 and chunk * parts >= n
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
        assert a1 == b0 and a0 <= a1
    for p, (n0, n1) in enumerate(bounds):
        assert n1 - n0 <= chunk and (n0 == n or n0 == p * chunk)


def test_shard_bounds_rejects_nonpositive():
    from modelsharp_b200 import ModelSharpException
    with pytest.raises(ModelSharpException):
        shard_bounds(0, 2)


def _slice_case(c: dict, n0: int, n1: int, a: np.ndarray) -> dict:
    s = dict(c)
    rows = lambda x: np.asarray(x).reshape(c["N"], -1)[n0:n1]  # noqa: E731 (scales may be flat)
    s["b"], s["scales"] = c["b"][n0:n1], rows(c["scales"])
    s["zp"] = rows(c["zp"]) if c["zp"] is not None else None
    s["N"], s["a"], s["M"] = n1 - n0, a, a.shape[0]
    return s


def _worker(rank: int, world: int, port: int, cases: list):
    from oracle import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for c, align in cases:
            def local(a2, n0, n1, c=c):
                return torch.from_numpy(oracle.managed(_slice_case(c, n0, n1, a2.numpy())))
            sh = ShardedMatMulNBits(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, c["block_size"],
                                    align=align, local=local)
            a = torch.from_numpy(c["a"]).reshape(*([2, c["M"] // 2] if c["M"] % 2 == 0 else [c["M"]]), c["K"])
            y = sh(a)
            assert tuple(y.shape) == tuple(a.shape[:-1]) + (c["N"],)
            ref = oracle.managed(c)
            np.testing.assert_array_equal(y.reshape(c["M"], c["N"]).numpy(), ref)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_nsplit_two_ranks_gloo():
    cases = [
        (synth.make_case(61, 1, 1000, 256, 4, 32, "packed"), 16),   # ragged last shard
        (synth.make_case(62, 3, 520, 128, 4, 128, "none"), 128),    # M > 1: permute of the gather
        (synth.make_case(63, 4, 100, 64, 4, 32, "float"), 128),     # rank 1 owns no rows
    ]
    mp.start_processes(_worker, args=(2, _free_port(), cases), nprocs=2, join=True, start_method="spawn")


@pytest.mark.gpu
def test_nsplit_one_rank_cuda_matches_unsplit(cuda_device):
    from modelsharp_b200 import QuantizedWeights
    c = synth.make_case(64, 3, 1000, 4096, 4, 128, "packed", scale_lo=0.001, scale_hi=0.01)
    a = torch.from_numpy(c["a"]).to(cuda_device)
    sh = ShardedMatMulNBits(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, 128, device=cuda_device)
    full = QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, 128, device=cuda_device)
    y = sh(a)
    ref = full.matmul(a)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(y, ref)
    sh.free()
    full.free()
