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


def _p2p_chain_check(dev, rank=0, world=1):
    """Up-proj then down-proj through the p2p gather, eager and as CUDA-graph replays with new
    inputs, against the unsplit kernel on the same device (bit-exact: same kernel per row)."""
    from modelsharp_b200 import QuantizedWeights
    up_c = synth.make_case(71, 2, 1024, 512, 4, 128, "packed", scale_lo=0.001, scale_hi=0.01)
    dn_c = synth.make_case(72, 2, 640, 1024, 4, 32, "none", scale_lo=0.001, scale_hi=0.01)
    up = ShardedMatMulNBits(up_c["b"], up_c["scales"], up_c["zp"], 1024, 512, 4, 128, device=dev, gather="p2p")
    dn = ShardedMatMulNBits(dn_c["b"], dn_c["scales"], dn_c["zp"], 640, 1024, 4, 32, device=dev, gather="p2p")
    up_full = QuantizedWeights(up_c["b"], up_c["scales"], up_c["zp"], 1024, 512, 4, 128, device=dev)
    dn_full = QuantizedWeights(dn_c["b"], dn_c["scales"], dn_c["zp"], 640, 1024, 4, 32, device=dev)
    gen = torch.Generator().manual_seed(5)
    a = torch.randn(2, 512, generator=gen).to(dev)

    def chain():
        return dn(up(a), wait=up.out_wait)

    def reference():
        return dn_full.matmul(up_full.matmul(a))

    for _ in range(3):  # eager, both buffer parities
        y = chain()
        dn.wait_gathered()
        assert torch.equal(y, reference())
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            y_g = chain()
    torch.cuda.current_stream(dev).wait_stream(s)
    for _ in range(4):  # replays: the device counters keep every rank in step
        a.copy_(torch.randn(2, 512, generator=gen).to(dev))
        g.replay()
        dn.wait_gathered()
        assert torch.equal(y_g, reference())
    torch.cuda.synchronize(dev)
    from modelsharp_b200 import _native as NAT
    assert NAT.lib().msq_device_status(None, None) == NAT.MSQ_OK, NAT.last_error()
    del g
    for x in (up, dn, up_full, dn_full):
        x.free()


@pytest.mark.gpu
def test_nsplit_p2p_one_rank(cuda_device):
    _p2p_chain_check(cuda_device)


def _p2p_worker(rank: int, world: int, port: int):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        _p2p_chain_check(torch.device("cuda", rank), rank, world)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nsplit_p2p_two_ranks(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_p2p_worker, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")
