"""The prompt forms of the decoder glue, through the C ABI, against the CPU decoder's glue.

msq_rope_append_rows (rotary of S tokens at positions pos0.. with k and v appended to the cache,
qkv unchanged), msq_gqa_prefill (causal grouped-query attention of S queries over the cache)
and msq_swiglu_rows, against oracle/decoder.py's rope, attention / causal_attention and the
SwiGLU formula. Float results agree to 1e-5 relative L2; copies are bit-exact. Edge cases: the
7B shape (32 / 8 heads of 128, a 512-token prompt), a continuation chunk (pos0 > 0, the queries
also attend to the earlier cache rows), 1, 3, 7 and 8 query heads per kv head, a prompt that
fills the cache, a prompt shorter than one 16-token query tile, and cache rows past the prompt
filled with NaN (never read).
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import _native as N
from oracle import decoder as od
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-5


class _Cfg:
    def __init__(self, heads, kv_heads, head_dim, max_seq, rope_theta=1e4):
        self.heads, self.kv_heads, self.head_dim, self.max_seq, self.rope_theta = heads, kv_heads, head_dim, max_seq, rope_theta


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _ok(rc):
    assert rc == N.MSQ_OK, N.last_error()


def _t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("heads,kv,d,max_seq,S,pos0", [(32, 8, 128, 640, 512, 0), (4, 2, 64, 64, 17, 5),
                                                       (6, 6, 32, 40, 40, 0), (3, 1, 16, 20, 3, 17)])
def test_rope_append_rows(cuda_device, heads, kv, d, max_seq, S, pos0):
    cfg = _Cfg(heads, kv, d, max_seq)
    cos, sin = od.rope_tables(cfg)
    rng = np.random.default_rng(S + d + pos0)
    nq, nk = heads * d, kv * d
    qkv = rng.standard_normal((S, nq + 2 * nk)).astype(np.float32)
    kc0 = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc0 = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    # every device buffer stays referenced until the kernel has run (a temporary's block would go
    # back to the caching allocator and be reused by the next upload)
    dqkv, dkc, dvc = _t(qkv, cuda_device), _t(kc0, cuda_device), _t(vc0, cuda_device)
    dcos, dsin = _t(cos, cuda_device), _t(sin, cuda_device)
    dq = torch.full((S, nq), float("nan"), device=cuda_device)
    _ok(N.lib().msq_rope_append_rows(None, _stream(cuda_device), dqkv.data_ptr(), S, pos0, heads, kv, d,
                                     dcos.data_ptr(), dsin.data_ptr(), dq.data_ptr(), dkc.data_ptr(), dvc.data_ptr(),
                                     max_seq))
    torch.cuda.synchronize(cuda_device)
    p = np.arange(pos0, pos0 + S)
    q = od.rope(qkv[:, :nq], heads, d, p, cos, sin)
    k = od.rope(qkv[:, nq:nq + nk], kv, d, p, cos, sin)
    assert oracle.rel_l2(dq.cpu().numpy(), q) <= TOL
    np.testing.assert_array_equal(dqkv.cpu().numpy(), qkv)  # the input is left unchanged
    kc, vc = kc0.copy(), vc0.copy()
    kc[:, pos0:pos0 + S] = k.reshape(S, kv, d).transpose(1, 0, 2)
    vc[:, pos0:pos0 + S] = qkv[:, nq + nk:].reshape(S, kv, d).transpose(1, 0, 2)
    got_k = dkc.cpu().numpy()
    assert oracle.rel_l2(got_k[:, pos0:pos0 + S], kc[:, pos0:pos0 + S]) <= TOL
    outside = np.ones(max_seq, dtype=bool)
    outside[pos0:pos0 + S] = False
    np.testing.assert_array_equal(got_k[:, outside], kc0[:, outside])  # other rows untouched
    np.testing.assert_array_equal(dvc.cpu().numpy(), vc)  # v: copies, bit-exact


@pytest.mark.parametrize("heads,kv,d,S,pos0,max_seq", [
    (32, 8, 128, 512, 0, 640),   # the 7B prompt
    (4, 2, 64, 33, 7, 64),       # a continuation chunk
    (8, 1, 128, 40, 100, 200),   # 8 query heads per kv head
    (3, 3, 64, 17, 0, 17),       # one head per kv head, the prompt fills the cache
    (12, 4, 64, 70, 5, 128),     # 3 per kv head
    (14, 2, 128, 5, 0, 16),      # 7 per kv head, shorter than one query tile
])
def test_gqa_prefill(cuda_device, heads, kv, d, S, pos0, max_seq):
    cfg = _Cfg(heads, kv, d, max_seq)
    rng = np.random.default_rng(heads * 31 + S + pos0)
    q = rng.standard_normal((S, heads * d)).astype(np.float32)
    kc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    kc[:, pos0 + S:] = np.nan  # rows past the prompt hold garbage and must not be read
    vc[:, pos0 + S:] = np.nan
    dq, dkc, dvc = _t(q, cuda_device), _t(kc, cuda_device), _t(vc, cuda_device)
    out = torch.full((S, heads * d), float("nan"), device=cuda_device)
    _ok(N.lib().msq_gqa_prefill(None, _stream(cuda_device), dq.data_ptr(), dkc.data_ptr(), dvc.data_ptr(), S, pos0,
                                out.data_ptr(), heads, kv, d, max_seq))
    torch.cuda.synchronize(cuda_device)
    got = out.cpu().numpy()
    if pos0 == 0:
        k = kc[:, :S].transpose(1, 0, 2).reshape(S, kv * d)
        v = vc[:, :S].transpose(1, 0, 2).reshape(S, kv * d)
        ref = od.causal_attention(q, k, v, cfg)
    else:
        ref = od.attention(q, kc[:, :pos0 + S], vc[:, :pos0 + S], pos0, cfg)
    assert np.isfinite(got).all()
    assert oracle.rel_l2(got, ref) <= TOL


def test_gqa_prefill_limits(cuda_device):
    dev = cuda_device
    buf = torch.zeros(64 * 1024, device=dev)
    p = buf.data_ptr()
    lib, st = N.lib(), _stream(dev)
    assert lib.msq_gqa_prefill(None, st, p, p, p, 4, 0, p, 4, 2, 32, 16) == N.MSQ_E_UNSUPPORTED  # d 32
    assert lib.msq_gqa_prefill(None, st, p, p, p, 4, 0, p, 16, 1, 64, 16) == N.MSQ_E_UNSUPPORTED  # 16 per kv head
    assert lib.msq_gqa_prefill(None, st, p + 4, p, p, 4, 0, p, 4, 2, 64, 16) == N.MSQ_E_UNSUPPORTED  # unaligned q
    assert lib.msq_gqa_prefill(None, st, p, p, p, 10, 8, p, 4, 2, 64, 16) == N.MSQ_E_INVALID  # past the cache
    assert lib.msq_gqa_prefill(None, st, p, p, p, 4, 0, p, 5, 2, 64, 16) == N.MSQ_E_INVALID  # heads % kv
    assert lib.msq_rope_append_rows(None, st, p, 8, 10, 4, 2, 64, p, p, p, p, p, 16) == N.MSQ_E_INVALID
    assert lib.msq_swiglu_rows(None, st, p, p, 0, 8) == N.MSQ_E_INVALID


@pytest.mark.parametrize("rows,n", [(512, 14336), (3, 1000), (1, 1)])
def test_swiglu_rows(cuda_device, rows, n):
    rng = np.random.default_rng(rows + n)
    gu = (3 * rng.standard_normal((rows, 2 * n))).astype(np.float32)
    dgu = _t(gu, cuda_device)
    out = torch.full((rows, n), float("nan"), device=cuda_device)
    _ok(N.lib().msq_swiglu_rows(None, _stream(cuda_device), dgu.data_ptr(), out.data_ptr(), rows, n))
    g, u = gu[:, :n], gu[:, n:]
    ref = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
    assert oracle.rel_l2(out.cpu().numpy(), ref) <= TOL
