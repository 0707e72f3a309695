"""The decoder checker's glue (oracle/decoder.py) pinned to the reference's own hand-computed
cases, within the reference tests' 1e-4 absolute tolerance.

* RMSNorm: tests/ModelSharp.Tests/FusedLlmNormTests.cs:46-82 (x / sqrt(mean(x^2) + eps) * scale)
* SkipSimplifiedLayerNormalization (the residual sum, then RMSNorm): FusedLlmNormTests.cs:86-108
* half-split (NeoX) rotary at positions 0 and 1: FusedLlmNormTests.cs:136-174
* causal grouped-query attention, two query heads sharing one kv head: GqaGenaiTests.cs:356-373
* one decode token over past keys and values: GqaGenaiTests.cs:279-334 (its expectation is the
  test's own softmax-attention formula, restated below)

The GPU glue kernels are checked against these same restatements in test_gpu_decoder_glue.py,
so the kernels are pinned to the reference's cases through them.
"""
import math
from types import SimpleNamespace

import numpy as np

from oracle import decoder as od

TOL = 1e-4  # the reference tests' Close() tolerance


def _close(want, got):
    np.testing.assert_allclose(np.asarray(got, np.float64).reshape(-1), np.asarray(want, np.float64).reshape(-1),
                               rtol=0, atol=TOL)


def test_rmsnorm_last_axis_hand_computed():
    x = np.array([[1, 2, 3, 4]], np.float32)
    inv = 1 / math.sqrt(7.5)
    _close([1 * inv, 2 * inv, 3 * inv, 4 * inv], od.rms_norm(x, np.ones(4, np.float32), 0.0))


def test_rmsnorm_scale_two_rows():
    eps = 1e-5
    x = np.array([[3, 4], [1, 1]], np.float32)
    inv0, inv1 = 1 / math.sqrt((9 + 16) / 2 + eps), 1 / math.sqrt((1 + 1) / 2 + eps)
    _close([3 * inv0 * 2, 4 * inv0 * 0.5, 1 * inv1 * 2, 1 * inv1 * 0.5],
           od.rms_norm(x, np.array([2, 0.5], np.float32), eps))


def test_skip_rmsnorm_sum_then_norm():
    inp = np.array([[1, 2, 3, 4]], np.float32)
    skip = np.array([[1, 2, 0, 0]], np.float32)
    s = inp + skip  # the residual sum the decoder carries forward (the kernel's output 3)
    _close([2, 4, 3, 4], s)
    inv = 1 / math.sqrt(11.25)
    _close([2 * inv, 4 * inv, 3 * inv, 4 * inv], od.rms_norm(s, np.ones(4, np.float32), 0.0))


def test_rope_half_split_hand_computed():
    t0, t1 = 0.5, 1.1
    cos = np.array([[1, 1], [math.cos(t0), math.cos(t1)]], np.float32)
    sin = np.array([[0, 0], [math.sin(t0), math.sin(t1)]], np.float32)
    x = np.array([[1, 2, 3, 4], [5, 6, 7, 8]], np.float32)  # two tokens, one head of 4
    c0, s0, c1, s1 = cos[1, 0], sin[1, 0], cos[1, 1], sin[1, 1]
    want = [1, 2, 3, 4,
            5 * c0 - 7 * s0, 6 * c1 - 8 * s1,
            7 * c0 + 5 * s0, 8 * c1 + 6 * s1]
    _close(want, od.rope(x, 1, 4, np.array([0, 1]), cos, sin))


def test_causal_gqa_two_heads_one_kv_head():
    cfg = SimpleNamespace(heads=2, kv_heads=1, head_dim=1)
    q = np.ones((2, 2), np.float32)                    # [S=2, heads*d]
    kc = np.array([[[0.5], [0.5]]], np.float32)        # [kv, T, d]
    vc = np.array([[[3.0], [9.0]]], np.float32)
    # position 0 sees key 0 only (V=3); position 1 sees both with equal scores (6)
    _close([3, 3, 6, 6], od.attention(q, kc, vc, 0, cfg))


def test_decode_token_over_past_keys():
    cfg = SimpleNamespace(heads=2, kv_heads=1, head_dim=2)
    q = np.array([[1, 0, 0, 1]], np.float32)
    k_all = np.array([[1, 0], [0, 1], [1, 1]], np.float32)  # past key 0, past key 1, the new key
    v_all = np.array([[2, 0], [0, 4], [9, 9]], np.float32)
    kc, vc = k_all[None], v_all[None]
    got = od.attention(q, kc, vc, 2, cfg)  # the new token sits at position 2 and sees all three
    scale = 1 / math.sqrt(2)
    want = []
    for h in range(2):
        sc = k_all @ q[0, 2 * h:2 * h + 2] * scale
        e = np.exp(sc - sc.max())
        want.extend((e / e.sum()) @ v_all)
    _close(want, got)
