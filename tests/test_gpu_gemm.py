"""tcgen05 prefill GEMM against the parity checker (needs a B200).

Bar: rel-L2 <= 5e-3 against the fp32 reference (the weights enter the tensor core as fp16
(q - zp) * s). Large M is checked on sampled rows of A (rows are independent).
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import QuantizedWeights, synth
from modelsharp_b200 import _native as N
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL_TC = 5e-3


def gemm(c, dev, a=None, path=N.PATH_GEMM):
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, c["block_size"], device=dev)
    a_t = torch.from_numpy(np.ascontiguousarray(c["a"] if a is None else a)).to(dev)
    y = w.matmul(a_t, path=path)
    torch.cuda.synchronize(dev)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    return y.cpu().numpy()


def sampled_ref(c, rows):
    return np.concatenate([oracle.managed(c, rows=r) for r in rows], axis=0)


@pytest.mark.parametrize("M,N_,K,bs,zp", [
    (17, 256, 256, 32, "packed"),      # smallest GEMM M, one partial row tile
    (64, 1000, 4160, 128, "packed"),   # ragged N tile and ragged last k-stage
    (128, 512, 1024, 32, "none"),
    (200, 384, 2048, 64, "float"),
    (300, 4096, 4096, 128, "packed"),  # 256-row tiles (two accumulators)
    (600, 640, 1024, 32, "float"),     # 512-row tiles (four accumulators), ragged last M tile
])
def test_gemm_parity_fp32_activations(cuda_device, M, N_, K, bs, zp):
    c = synth.make_case(31, M, N_, K, 4, bs, zp, scale_lo=0.001, scale_hi=0.01)
    y = gemm(c, cuda_device)
    assert N.last_path().startswith("gemm_tc")
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_TC


@pytest.mark.parametrize("M", [512, 2048])
def test_gemm_prefill_config_fp16(cuda_device, M):
    """K=4096, N=14336, bs=32, zero points, fp16 A and fp16 scales."""
    c = synth.make_case(3, M, 14336, 4096, 4, 32, "packed", a_dtype="f16", scale_dtype="f16",
                        scale_lo=0.001, scale_hi=0.01)
    y = gemm(c, cuda_device)
    rows = [slice(0, 48), slice(M // 2, M // 2 + 16), slice(M - 64, M)]
    ref = sampled_ref(c, rows)
    got = np.concatenate([y[r] for r in rows], axis=0)
    assert oracle.rel_l2(got, ref) <= TOL_TC


@pytest.mark.parametrize("M,N_,K,bs", [
    (32, 2048, 28672, 128),   # a 4-GPU shard of the 70B down-projection: 16 tiles, K split 9 ways
    (32, 256, 8192, 32),      # 2 tiles
    (100, 640, 1000, 64),     # ragged K: the last split is short
])
def test_gemm_split_k(cuda_device, M, N_, K, bs):
    """Tiles that leave SMs idle split K across CTAs; partial tiles are summed in a fixed order,
    so two runs agree bit for bit."""
    c = synth.make_case(35, M, N_, K, 4, bs, "packed", scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], N_, K, 4, bs, device=cuda_device)
    a_t = torch.from_numpy(c["a"]).to(cuda_device).reshape(M, K)
    y1 = w.matmul(a_t, path=N.PATH_GEMM)
    assert N.last_path().endswith("_splitk")
    y2 = w.matmul(a_t, path=N.PATH_GEMM)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert oracle.rel_l2(y1.cpu().numpy(), oracle.managed(c)) <= TOL_TC
    w.free()


def test_gemm_full_grid_does_not_split(cuda_device):
    c = synth.make_case(36, 2048, 14336, 256, 4, 32, "packed", a_dtype="f16", scale_dtype="f16")
    gemm(c, cuda_device)
    assert N.last_path() in ("gemm_tc_m384_n128", "gemm_tc_m512_n128")  # a full grid: no k split


@pytest.mark.parametrize("M,N_,K,bs,zp,a_dtype", [
    (17, 300, 256, 32, "packed", "f32"),     # ragged N, K-split (3 weight tiles), staged A
    (24, 1000, 4160, 128, "none", "f16"),    # ragged last k-stage
    (32, 8192, 2048, 64, "float", "f32"),
    (33, 4096, 4096, 128, "packed", "f16"),
    (48, 256, 8192, 32, "packed", "f16"),    # two weight tiles, many K-splits
    (64, 2000, 1024, 128, "packed", "f32"),
])
def test_gemm_small_m(cuda_device, M, N_, K, bs, zp, a_dtype):
    """17 <= M <= 64 (one 128-row activation tile, K split across CTAs where the weight tiles
    leave SMs idle; staged fp32 rows scaled by a power of two), against the checker at the
    GEMM's bar."""
    c = synth.make_case(37, M, N_, K, 4, bs, zp, a_dtype=a_dtype, scale_lo=0.001, scale_hi=0.01)
    y = gemm(c, cuda_device)
    assert N.last_path().startswith("gemm_tc_m128_n128"), N.last_path()
    assert oracle.rel_l2(y, oracle.managed(c)) <= TOL_TC


def test_gemm_small_m_writes_only_its_shard(cuda_device):
    c = synth.make_case(39, 20, 600, 1024, 4, 64, "packed", scale_lo=0.001, scale_hi=0.01)
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], 600, 1024, 4, 64, rows=(200, 600), device=cuda_device)
    y = torch.full((20, 640), float("nan"), device=cuda_device)
    w.matmul(torch.from_numpy(c["a"]).to(cuda_device), out=y[:, 200:600], ldy=640, path=N.PATH_GEMM)
    torch.cuda.synchronize()
    assert N.last_path().startswith("gemm_tc_m128_n128")
    out = y.cpu().numpy()
    assert np.isnan(out[:, :200]).all() and np.isnan(out[:, 600:]).all()
    ref = oracle.managed(c)[:, 200:600]
    assert oracle.rel_l2(out[:, 200:600], ref) <= TOL_TC
    w.free()


def test_gemm_auto_routes_prefill(cuda_device):
    c = synth.make_case(32, 40, 640, 1024, 4, 128, "packed")
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], 640, 1024, 4, 128, device=cuda_device)
    y = w.matmul(torch.from_numpy(c["a"]).to(cuda_device))
    torch.cuda.synchronize()
    assert N.last_path().startswith("gemm_tc")
    assert oracle.rel_l2(y.cpu().numpy(), oracle.managed(c)) <= TOL_TC


def test_gemm_writes_only_its_shard(cuda_device):
    c = synth.make_case(33, 130, 300, 512, 4, 32, "packed")
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], 300, 512, 4, 32, rows=(100, 300), device=cuda_device)
    y = torch.full((130, 320), float("nan"), device=cuda_device)
    w.matmul(torch.from_numpy(c["a"]).to(cuda_device), out=y[:, 100:300], ldy=320, path=N.PATH_GEMM)
    torch.cuda.synchronize()
    out = y.cpu().numpy()
    assert np.isnan(out[:, :100]).all() and np.isnan(out[:, 300:]).all()
    assert oracle.rel_l2(out[:, 100:300], oracle.managed(c)[:, 100:300]) <= TOL_TC


def test_gemm_bf16_and_unaligned_half(cuda_device):
    c = synth.make_case(34, 70, 256, 1000, 4, 32, "packed")  # K % 8 != 0 -> scratch copy
    a16 = torch.from_numpy(c["a"]).to(torch.float16)
    ref = oracle.managed(dict(c, a=a16.float().numpy()))
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], 256, 1000, 4, 32, device=cuda_device)
    y = w.matmul(a16.to(cuda_device), path=N.PATH_GEMM).cpu().numpy()
    assert oracle.rel_l2(y, ref) <= TOL_TC
    ab = torch.from_numpy(c["a"]).to(torch.bfloat16)
    refb = oracle.managed(dict(c, a=ab.float().numpy()))
    yb = w.matmul(ab.to(cuda_device), path=N.PATH_GEMM).cpu().numpy()
    assert oracle.rel_l2(yb, refb) <= TOL_TC


TOL_SPLIT = 1e-5  # the split-operand GEMM: ~2^-22 products, the fp32-accumulate bar


@pytest.mark.parametrize("M,N_,K,bs,zp,adt", [
    (17, 256, 256, 32, "packed", "f32"),
    (64, 1000, 4160, 128, "packed", "f32"),   # ragged N tile and last k-stage
    (130, 512, 1024, 32, "none", "f32"),      # 256-row tiles, ragged M
    (200, 384, 2048, 64, "float", "f32"),
    (300, 4096, 4096, 32, "packed", "f16"),   # fp16 A: no lo part (exact), 2 MMAs per step
    (40, 640, 1000, 32, "packed", "bf16"),    # K % 8 != 0: staged
    (512, 6144, 4096, 32, "packed", "f32"),   # the 7B prompt's q/k/v shape
])
def test_gemm_split_operands_parity(cuda_device, M, N_, K, bs, zp, adt):
    c = synth.make_case(37, M, N_, K, 4, bs, zp, scale_lo=0.001, scale_hi=0.01)
    a = c["a"]
    if adt == "f16":
        a = a.astype(np.float16)
    elif adt == "bf16":
        a = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    ref = oracle.managed(dict(c, a=np.asarray(a, np.float32)))
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], N_, K, 4, bs, device=cuda_device)
    at = torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    if adt == "bf16":
        at = at.to(torch.bfloat16)
    y = w.matmul(at, path=N.PATH_GEMM_SPLIT)
    torch.cuda.synchronize()
    assert N.last_path().startswith("gemm_tc_x3")
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    err = oracle.rel_l2(y.cpu().numpy(), ref)
    assert err <= TOL_SPLIT, err
    # the fast GEMM on the same inputs is the fp16 one (a bar 500x wider)
    assert oracle.rel_l2(w.matmul(at, path=N.PATH_GEMM).cpu().numpy(), ref) <= TOL_TC
    y2 = w.matmul(at, path=N.PATH_AUTO_SPLIT)
    assert torch.equal(y, y2)
    w.free()


@pytest.mark.parametrize("M,want", [(512, "gemm_tc_m512_n128"), (2048, "gemm_tc_m384_n128"), (2000, "gemm_tc_m384_n128")])
def test_gemm_three_or_four_accumulators(cuda_device, M, want):
    """M >= 512 takes three or four accumulators per weight tile by whole waves of tiles (N = 14336:
    M = 512 one wave of four against two of three; M = 2048 and 2000, whose last 384-row tile
    holds 80 rows, five waves of three against four of four); both forms meet the GEMM bar."""
    c = synth.make_case(38, M, 14336, 256, 4, 32, "packed", a_dtype="f16", scale_dtype="f16",
                        scale_lo=0.001, scale_hi=0.01)
    y = gemm(c, cuda_device)
    if want:
        assert N.last_path() == want
    rows = [slice(0, 16), slice(M - 40, M)]
    ref = sampled_ref(c, rows)
    assert oracle.rel_l2(np.concatenate([y[r] for r in rows]), ref) <= TOL_TC
