"""The library's decoder glue kernels, through the C ABI, against the CPU decoder's glue.

Each kernel runs on seeded inputs and is compared with oracle/decoder.py (float32 restatement
of the reference's CPU kernels): add + RMSNorm, rotary + KV-cache append at a device-side
position, grouped-query decode attention, SwiGLU and argmax. Float results agree to 1e-5
relative L2 (a different summation order than the checker's); index results are exact.
The fused rotary + append + attention entry is compared with the checker's rope followed by
attention. Edge cases: the first position (one key, most of the split-K slices empty), the
last cache row, 1 to 8 query heads per kv head, head sizes 16 to 256, a 40 000-row cache,
ties in argmax (the first index wins), a position past the cache (no write, all keys read).
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


@pytest.mark.parametrize("rows,n,with_delta", [(1, 4096, True), (3, 256, False), (2, 1000, True)])
def test_add_rmsnorm(cuda_device, rows, n, with_delta):
    rng = np.random.default_rng(rows * 7 + n)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    delta = rng.standard_normal((rows, n)).astype(np.float32)
    gamma = rng.uniform(0.8, 1.2, n).astype(np.float32)
    dx, dd, dg = (torch.from_numpy(v).to(cuda_device) for v in (x, delta, gamma))
    dy = torch.empty_like(dx)
    _ok(N.lib().msq_add_rmsnorm(None, _stream(cuda_device), dx.data_ptr(), dd.data_ptr() if with_delta else None,
                                dg.data_ptr(), dy.data_ptr(), rows, n, 1e-5))
    xs = x + delta if with_delta else x
    assert oracle.rel_l2(dx.cpu().numpy(), xs) <= 1e-7
    assert oracle.rel_l2(dy.cpu().numpy(), od.rms_norm(xs, gamma, 1e-5)) <= TOL


@pytest.mark.parametrize("heads,kv,d,max_seq,pos", [(32, 8, 128, 640, 0), (32, 8, 128, 640, 639), (4, 2, 64, 64, 17),
                                                    (6, 6, 32, 10, 3)])
def test_rope_append(cuda_device, heads, kv, d, max_seq, pos):
    cfg = _Cfg(heads, kv, d, max_seq)
    cos, sin = od.rope_tables(cfg)
    rng = np.random.default_rng(pos + d)
    qkv = rng.standard_normal((1, (heads + 2 * kv) * d)).astype(np.float32)
    kc0 = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc0 = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    dq, dkc, dvc = (torch.from_numpy(v.copy()).to(cuda_device) for v in (qkv, kc0, vc0))
    dcos, dsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    dpos = torch.tensor([pos], dtype=torch.int64, device=cuda_device)
    _ok(N.lib().msq_rope_append(None, _stream(cuda_device), dq.data_ptr(), heads, kv, d, dcos.data_ptr(),
                                dsin.data_ptr(), dpos.data_ptr(), dkc.data_ptr(), dvc.data_ptr(), max_seq))
    p = np.asarray([pos])
    nq, nk = heads * d, kv * d
    q = od.rope(qkv[:, :nq], heads, d, p, cos, sin)
    k = od.rope(qkv[:, nq:nq + nk], kv, d, p, cos, sin)
    got = dq.cpu().numpy()
    assert oracle.rel_l2(got[:, :nq], q) <= TOL
    assert oracle.rel_l2(got[:, nq:nq + nk], k) <= TOL
    np.testing.assert_array_equal(got[:, nq + nk:], qkv[:, nq + nk:])  # v untouched
    kc, vc = kc0.copy(), vc0.copy()
    kc[:, pos] = k.reshape(kv, d)
    vc[:, pos] = qkv[0, nq + nk:].reshape(kv, d)
    assert oracle.rel_l2(dkc.cpu().numpy(), kc) <= TOL
    np.testing.assert_array_equal(dvc.cpu().numpy(), vc)  # a copy: bit-exact


def test_rope_append_position_past_cache_writes_nothing(cuda_device):
    heads, kv, d, max_seq = 4, 2, 64, 16
    cfg = _Cfg(heads, kv, d, max_seq)
    cos, sin = od.rope_tables(cfg)
    qkv = torch.randn(1, (heads + 2 * kv) * d, device=cuda_device)
    before = qkv.clone()
    kc = torch.zeros(kv, max_seq, d, device=cuda_device)
    vc = torch.zeros_like(kc)
    dpos = torch.tensor([max_seq], dtype=torch.int64, device=cuda_device)
    dcos, dsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    _ok(N.lib().msq_rope_append(None, _stream(cuda_device), qkv.data_ptr(), heads, kv, d, dcos.data_ptr(),
                                dsin.data_ptr(), dpos.data_ptr(), kc.data_ptr(), vc.data_ptr(), max_seq))
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(qkv, before) and not kc.any() and not vc.any()


@pytest.mark.parametrize("heads,kv,d,max_seq,pos", [(32, 8, 128, 640, 0), (32, 8, 128, 640, 512), (4, 2, 64, 64, 63),
                                                    (6, 3, 32, 100, 41), (8, 8, 128, 2048, 1999), (6, 2, 64, 50, 20),
                                                    (16, 2, 256, 300, 299), (32, 8, 128, 640, 5)])
def test_gqa_decode(cuda_device, heads, kv, d, max_seq, pos):
    cfg = _Cfg(heads, kv, d, max_seq)
    rng = np.random.default_rng(pos * 3 + heads)
    q = rng.standard_normal((1, heads * d)).astype(np.float32)
    kc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    dq, dkc, dvc = (torch.from_numpy(v).to(cuda_device) for v in (q, kc, vc))
    out = torch.empty(1, heads * d, device=cuda_device)
    dpos = torch.tensor([pos], dtype=torch.int64, device=cuda_device)
    _ok(N.lib().msq_gqa_decode(None, _stream(cuda_device), dq.data_ptr(), dkc.data_ptr(), dvc.data_ptr(),
                               dpos.data_ptr(), out.data_ptr(), heads, kv, d, max_seq))
    ref = od.attention(q, kc, vc, pos, cfg)
    assert oracle.rel_l2(out.cpu().numpy(), ref) <= TOL


def test_gqa_decode_position_past_cache_reads_all_keys(cuda_device):
    heads, kv, d, max_seq = 4, 2, 64, 32
    cfg = _Cfg(heads, kv, d, max_seq)
    rng = np.random.default_rng(5)
    q = rng.standard_normal((1, heads * d)).astype(np.float32)
    kc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    dq, dkc, dvc = (torch.from_numpy(v).to(cuda_device) for v in (q, kc, vc))
    out = torch.empty(1, heads * d, device=cuda_device)
    dpos = torch.tensor([max_seq + 5], dtype=torch.int64, device=cuda_device)
    _ok(N.lib().msq_gqa_decode(None, _stream(cuda_device), dq.data_ptr(), dkc.data_ptr(), dvc.data_ptr(),
                               dpos.data_ptr(), out.data_ptr(), heads, kv, d, max_seq))
    assert oracle.rel_l2(out.cpu().numpy(), od.attention(q, kc, vc, max_seq - 1, cfg)) <= TOL


def test_gqa_decode_limits(cuda_device):
    t = torch.zeros(8, device=cuda_device)
    dpos = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    L, st = N.lib(), _stream(cuda_device)
    # 16 query heads per kv head, and d = 512: outside the compiled plans
    assert L.msq_gqa_decode(None, st, t.data_ptr(), t.data_ptr(), t.data_ptr(), dpos.data_ptr(), t.data_ptr(),
                            16, 1, 128, 64) == N.MSQ_E_UNSUPPORTED
    assert L.msq_gqa_decode(None, st, t.data_ptr(), t.data_ptr(), t.data_ptr(), dpos.data_ptr(), t.data_ptr(),
                            2, 1, 512, 64) == N.MSQ_E_UNSUPPORTED
    # a long cache is fine: shared memory does not grow with max_seq
    heads, kv, d, max_seq, pos = 8, 2, 128, 40000, 39000
    cfg = _Cfg(heads, kv, d, max_seq)
    rng = np.random.default_rng(40000)
    q = rng.standard_normal((1, heads * d)).astype(np.float32)
    kc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    dq, dkc, dvc = (torch.from_numpy(v).to(cuda_device) for v in (q, kc, vc))
    out = torch.empty(1, heads * d, device=cuda_device)
    dpos.fill_(pos)
    _ok(L.msq_gqa_decode(None, st, dq.data_ptr(), dkc.data_ptr(), dvc.data_ptr(), dpos.data_ptr(), out.data_ptr(),
                         heads, kv, d, max_seq))
    assert oracle.rel_l2(out.cpu().numpy(), od.attention(q, kc, vc, pos, cfg)) <= TOL


@pytest.mark.parametrize("heads,kv,d,max_seq,pos", [(32, 8, 128, 640, 0), (32, 8, 128, 640, 600), (4, 2, 64, 64, 63),
                                                    (6, 3, 32, 100, 41), (16, 2, 256, 300, 77), (8, 8, 128, 2048, 9),
                                                    (8, 1, 16, 24, 23)])
def test_rope_gqa_decode_matches_rope_then_attention(cuda_device, heads, kv, d, max_seq, pos):
    """The fused entry against the checker's rope then attention, and the cache rows it writes."""
    cfg = _Cfg(heads, kv, d, max_seq)
    cos, sin = od.rope_tables(cfg)
    rng = np.random.default_rng(pos * 7 + d)
    qkv = rng.standard_normal((1, (heads + 2 * kv) * d)).astype(np.float32)
    kc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    dqkv, dkc, dvc = (torch.from_numpy(v.copy()).to(cuda_device) for v in (qkv, kc, vc))
    dcos, dsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    dpos = torch.tensor([pos], dtype=torch.int64, device=cuda_device)
    out = torch.empty(1, heads * d, device=cuda_device)
    _ok(N.lib().msq_rope_gqa_decode(None, _stream(cuda_device), dqkv.data_ptr(), heads, kv, d, dcos.data_ptr(),
                                    dsin.data_ptr(), dpos.data_ptr(), dkc.data_ptr(), dvc.data_ptr(), out.data_ptr(),
                                    max_seq))
    p = np.asarray([pos])
    nq, nk = heads * d, kv * d
    q = od.rope(qkv[:, :nq], heads, d, p, cos, sin)
    k = od.rope(qkv[:, nq:nq + nk], kv, d, p, cos, sin)
    kc[:, pos] = k.reshape(kv, d)
    vc[:, pos] = qkv[0, nq + nk:].reshape(kv, d)
    assert oracle.rel_l2(out.cpu().numpy(), od.attention(q, kc, vc, pos, cfg)) <= TOL
    got_k = dkc.cpu().numpy()
    assert oracle.rel_l2(got_k[:, pos], kc[:, pos]) <= TOL
    np.testing.assert_array_equal(np.delete(got_k, pos, axis=1), np.delete(kc, pos, axis=1))  # other rows untouched
    np.testing.assert_array_equal(dvc.cpu().numpy(), vc)
    np.testing.assert_array_equal(dqkv.cpu().numpy(), qkv)  # the input stays unrotated


def test_rope_gqa_decode_position_past_cache(cuda_device):
    heads, kv, d, max_seq = 4, 2, 64, 32
    cfg = _Cfg(heads, kv, d, max_seq)
    cos, sin = od.rope_tables(cfg)
    rng = np.random.default_rng(6)
    qkv = rng.standard_normal((1, (heads + 2 * kv) * d)).astype(np.float32)
    kc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    vc = rng.standard_normal((kv, max_seq, d)).astype(np.float32)
    dqkv, dkc, dvc = (torch.from_numpy(v.copy()).to(cuda_device) for v in (qkv, kc, vc))
    dpos = torch.tensor([max_seq + 3], dtype=torch.int64, device=cuda_device)
    out = torch.empty(1, heads * d, device=cuda_device)
    dcos, dsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    _ok(N.lib().msq_rope_gqa_decode(None, _stream(cuda_device), dqkv.data_ptr(), heads, kv, d, dcos.data_ptr(),
                                    dsin.data_ptr(), dpos.data_ptr(), dkc.data_ptr(), dvc.data_ptr(), out.data_ptr(),
                                    max_seq))
    ref = od.attention(qkv[:, :heads * d], kc, vc, max_seq - 1, cfg)
    assert oracle.rel_l2(out.cpu().numpy(), ref) <= TOL
    np.testing.assert_array_equal(dkc.cpu().numpy(), kc)
    np.testing.assert_array_equal(dvc.cpu().numpy(), vc)


@pytest.mark.parametrize("n", [14336, 1, 1000])
def test_swiglu(cuda_device, n):
    rng = np.random.default_rng(n)
    gu = (rng.standard_normal((1, 2 * n)) * 4).astype(np.float32)
    dgu = torch.from_numpy(gu).to(cuda_device)
    out = torch.empty(1, n, device=cuda_device)
    _ok(N.lib().msq_swiglu(None, _stream(cuda_device), dgu.data_ptr(), out.data_ptr(), n))
    g, u = gu[:, :n], gu[:, n:]
    ref = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
    assert oracle.rel_l2(out.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("n,tie", [(32000, False), (32000, True), (1, False), (1025, True)])
def test_argmax_advances_position(cuda_device, n, tie):
    rng = np.random.default_rng(n + tie)
    x = rng.standard_normal(n).astype(np.float32)
    if tie and n > 3:
        x[n // 3] = x[n - 1] = np.float32(9.0)  # equal maxima: the first index wins
    dx = torch.from_numpy(x).to(cuda_device)
    idx = torch.full((1,), -1, dtype=torch.int64, device=cuda_device)
    pos = torch.tensor([41], dtype=torch.int64, device=cuda_device)
    _ok(N.lib().msq_argmax(None, _stream(cuda_device), dx.data_ptr(), n, idx.data_ptr(), pos.data_ptr()))
    assert int(idx) == int(np.argmax(x))
    assert int(pos) == 42
    _ok(N.lib().msq_argmax(None, _stream(cuda_device), dx.data_ptr(), n, idx.data_ptr(), None))
    assert int(pos) == 42


def test_argmax_all_negative_infinity_is_index_zero(cuda_device):
    x = torch.full((300,), float("-inf"), device=cuda_device)
    idx = torch.full((1,), -1, dtype=torch.int64, device=cuda_device)
    _ok(N.lib().msq_argmax(None, _stream(cuda_device), x.data_ptr(), 300, idx.data_ptr(), None))
    assert int(idx) == 0


def test_glue_rejects_bad_arguments(cuda_device):
    t = torch.zeros(8, device=cuda_device)
    st = _stream(cuda_device)
    L = N.lib()
    assert L.msq_add_rmsnorm(None, st, None, None, t.data_ptr(), t.data_ptr(), 1, 8, 1e-5) == N.MSQ_E_INVALID
    assert L.msq_rope_append(None, st, t.data_ptr(), 3, 2, 64, t.data_ptr(), t.data_ptr(), t.data_ptr(),
                             t.data_ptr(), t.data_ptr(), 8) == N.MSQ_E_INVALID  # 3 heads over 2 kv heads
    assert L.msq_rope_append(None, st, t.data_ptr(), 2, 2, 63, t.data_ptr(), t.data_ptr(), t.data_ptr(),
                             t.data_ptr(), t.data_ptr(), 8) == N.MSQ_E_INVALID  # odd head dim
    assert L.msq_swiglu(None, st, t.data_ptr(), t.data_ptr(), 0) == N.MSQ_E_INVALID
    assert L.msq_argmax(None, st, t.data_ptr(), 0, t.data_ptr(), None) == N.MSQ_E_INVALID
