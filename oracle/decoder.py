"""CPU restatement of a Llama-shaped INT4 decoder -- TEST INFRASTRUCTURE ONLY.

The parity checker for modelsharp_b200.decoder (tests/, bench.py's CPU-baseline leg).
Every projection is MatMulNBits through the C restatement of the reference's managed kernel
(oracle.managed); the glue restates the reference's CPU kernels:

* rms_norm      y = x / sqrt(mean(x^2) + eps) * gamma
                (src/ModelSharp/Cpu/Kernels/Llm/SimplifiedLayerNormalizationKernel.cs:48-54;
                SkipSimplifiedLayerNormalizationKernel.cs:64-67 adds the residual first)
* rope          half-split pairs (x[j], x[j + d/2]) rotated by cos/sin of the absolute
                position (RotaryEmbeddingKernel.cs:96-114, interleaved = 0)
* attention     causal grouped-query attention, query head h reads kv head h / (H / Hkv),
                scores scaled by 1/sqrt(d), max-subtracted exp, sum, weighted sum of V
                (GroupQueryAttentionKernel.cs:194-195, 275-312)
* swiglu        silu(gate) * up with silu(x) = x / (1 + exp(-x))

Arithmetic is float32 throughout, in a plain order (the reference's SIMD reduction order is
not reproduced, so agreement is to float32 rounding, not bit-exact).
"""
from __future__ import annotations

import numpy as np

from . import oracle

PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def proj_shapes(cfg) -> dict[str, tuple[int, int]]:
    """(N, K) of every projection of a layer."""
    h, kv, i = cfg.hidden, cfg.kv_heads * cfg.head_dim, cfg.inter
    return {"q": (cfg.heads * cfg.head_dim, h), "k": (kv, h), "v": (kv, h), "o": (h, cfg.heads * cfg.head_dim),
            "gate": (i, h), "up": (i, h), "down": (h, i)}


def rope_tables(cfg) -> tuple[np.ndarray, np.ndarray]:
    """cos / sin [max_seq, head_dim/2]: angle = pos * theta^(-2j/d), computed in float64."""
    half = cfg.head_dim // 2
    inv = cfg.rope_theta ** (-np.arange(half, dtype=np.float64) * 2.0 / cfg.head_dim)
    ang = np.arange(cfg.max_seq, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rms_norm(x: np.ndarray, gamma: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(ms + np.float32(eps))
    return (x * inv * gamma).astype(np.float32)


def rope(x: np.ndarray, heads: int, d: int, pos: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x [S, heads*d] rotated at absolute positions pos [S]."""
    s = x.shape[0]
    v = x.reshape(s, heads, d).copy()
    h = d // 2
    c, sn = cos[pos][:, None, :], sin[pos][:, None, :]
    a, b = v[..., :h].copy(), v[..., h:].copy()
    v[..., :h] = a * c - b * sn
    v[..., h:] = b * c + a * sn
    return v.reshape(s, heads * d)


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, pos0: int, cfg) -> np.ndarray:
    """q [S, H*d]; kc / vc [Hkv, T, d] holding positions 0..pos0+S-1; causal."""
    s, d, hq, hkv = q.shape[0], cfg.head_dim, cfg.heads, cfg.kv_heads
    group = hq // hkv
    scale = np.float32(1.0 / np.sqrt(d))
    out = np.zeros((s, hq, d), dtype=np.float32)
    qv = q.reshape(s, hq, d)
    for h in range(hq):
        g = h // group
        for i in range(s):
            n = pos0 + i + 1
            sc = (kc[g, :n] @ qv[i, h]) * scale
            e = np.exp(sc - sc.max())
            out[i, h] = (e / e.sum()) @ vc[g, :n]
    return out.reshape(s, hq * d)


def matmul(x: np.ndarray, w: dict, n: int, k: int, cfg) -> np.ndarray:
    case = dict(a=np.ascontiguousarray(x, dtype=np.float32), b=w["b"], scales=w["scales"], zp=w["zp"],
                zp_kind="packed", M=x.shape[0], N=n, K=k, bits=4, block_size=cfg.block_size)
    return oracle.managed(case)


def forward(weights: dict, cfg, tokens: np.ndarray, pos0: int, cache: dict) -> np.ndarray:
    """Logits [S, vocab] of tokens at positions pos0.. ; appends their K/V to `cache`."""
    shapes = proj_shapes(cfg)
    cos, sin = cache["rope"]
    pos = np.arange(pos0, pos0 + len(tokens))
    x = weights["embed"][tokens].astype(np.float32)
    d = cfg.head_dim
    for li in range(cfg.layers):
        lw = weights["layers"][li]
        h = rms_norm(x, lw["norm_attn"], cfg.eps)
        q = rope(matmul(h, lw["q"], *shapes["q"], cfg), cfg.heads, d, pos, cos, sin)
        kk = rope(matmul(h, lw["k"], *shapes["k"], cfg), cfg.kv_heads, d, pos, cos, sin)
        vv = matmul(h, lw["v"], *shapes["v"], cfg)
        kc, vc = cache["k"][li], cache["v"][li]
        kc[:, pos0:pos0 + len(tokens)] = kk.reshape(len(tokens), cfg.kv_heads, d).transpose(1, 0, 2)
        vc[:, pos0:pos0 + len(tokens)] = vv.reshape(len(tokens), cfg.kv_heads, d).transpose(1, 0, 2)
        x = x + matmul(attention(q, kc, vc, pos0, cfg), lw["o"], *shapes["o"], cfg)
        h = rms_norm(x, lw["norm_mlp"], cfg.eps)
        gate = matmul(h, lw["gate"], *shapes["gate"], cfg)
        up = matmul(h, lw["up"], *shapes["up"], cfg)
        act = (gate / (np.float32(1.0) + np.exp(-gate)) * up).astype(np.float32)
        x = x + matmul(act, lw["down"], *shapes["down"], cfg)
    h = rms_norm(x, weights["norm_final"], cfg.eps)
    return matmul(h, weights["lm_head"], cfg.vocab, cfg.hidden, cfg)


def generate(weights: dict, cfg, prompt: np.ndarray, n_new: int) -> tuple[np.ndarray, list[np.ndarray]]:
    """Greedy decoding: the prompt in one pass, then one token per step. Returns the new
    tokens and the logits that chose each of them."""
    cache = {"k": np.zeros((cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim), np.float32),
             "v": np.zeros((cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim), np.float32),
             "rope": rope_tables(cfg)}
    logits = forward(weights, cfg, np.asarray(prompt), 0, cache)[-1]
    out, all_logits = [], [logits]
    pos = len(prompt)
    for _ in range(n_new):
        tok = int(np.argmax(logits))
        out.append(tok)
        if len(out) == n_new:
            break
        logits = forward(weights, cfg, np.asarray([tok]), pos, cache)[-1]
        all_logits.append(logits)
        pos += 1
    return np.asarray(out), all_logits


def _dense(w: dict, n: int, k: int, cfg) -> np.ndarray:
    """W [n, k] in fp32, (q - zp) * scale (oracle.dequant)."""
    return oracle.dequant(dict(b=w["b"], scales=w["scales"], zp=w["zp"], zp_kind="packed", N=n, K=k, bits=4,
                               block_size=cfg.block_size))


def causal_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, cfg) -> np.ndarray:
    """attention() over a whole sequence from position 0 at once: q [S, H*d], k / v [S, Hkv*d];
    row i attends to positions 0..i with the same scale, max-subtracted exp and normalisation."""
    s, d, hq, hkv = q.shape[0], cfg.head_dim, cfg.heads, cfg.kv_heads
    group = hq // hkv
    scale = np.float32(1.0 / np.sqrt(d))
    qv, kv, vv = q.reshape(s, hq, d), k.reshape(s, hkv, d), v.reshape(s, hkv, d)
    future = np.triu(np.ones((s, s), dtype=bool), 1)
    out = np.empty((s, hq, d), dtype=np.float32)
    for h in range(hq):
        g = h // group
        sc = (qv[:, h] @ kv[:, g].T) * scale
        sc[future] = -np.inf
        e = np.exp(sc - sc.max(axis=1, keepdims=True))
        out[:, h] = (e / e.sum(axis=1, keepdims=True)) @ vv[:, g]
    return out.reshape(s, hq * d)


def teacher_forced_logits(weights: dict, cfg, tokens: np.ndarray, score_from: int) -> np.ndarray:
    """Logits [len(tokens) - score_from, vocab] of positions score_from.. of one pass over the
    whole sequence (the ops of forward(), every projection a dense fp32 product with the
    dequantised weight; agreement with forward() is to fp32 rounding).

    Greedy decoding that produced `tokens` from the prompt tokens[:score_from + 1] is what
    this checker would itself have generated exactly when argmax(logits[i]) ==
    tokens[score_from + 1 + i] for every i: each step's context is then the checker's own."""
    shapes = proj_shapes(cfg)
    cos, sin = rope_tables(cfg)
    tokens = np.asarray(tokens)
    pos = np.arange(len(tokens))
    x = weights["embed"][tokens].astype(np.float32)
    d = cfg.head_dim
    for li in range(cfg.layers):
        lw = weights["layers"][li]
        h = rms_norm(x, lw["norm_attn"], cfg.eps)
        q = rope(h @ _dense(lw["q"], *shapes["q"], cfg).T, cfg.heads, d, pos, cos, sin)
        kk = rope(h @ _dense(lw["k"], *shapes["k"], cfg).T, cfg.kv_heads, d, pos, cos, sin)
        vv = h @ _dense(lw["v"], *shapes["v"], cfg).T
        x = x + causal_attention(q, kk, vv, cfg) @ _dense(lw["o"], *shapes["o"], cfg).T
        h = rms_norm(x, lw["norm_mlp"], cfg.eps)
        gate = h @ _dense(lw["gate"], *shapes["gate"], cfg).T
        up = h @ _dense(lw["up"], *shapes["up"], cfg).T
        act = (gate / (np.float32(1.0) + np.exp(-gate)) * up).astype(np.float32)
        x = x + act @ _dense(lw["down"], *shapes["down"], cfg).T
    h = rms_norm(x[score_from:], weights["norm_final"], cfg.eps)
    return h @ _dense(weights["lm_head"], cfg.vocab, cfg.hidden, cfg).T


def greedy_check(weights: dict, cfg, prompt: np.ndarray, generated: np.ndarray, return_logits: bool = False) -> dict:
    """Checks `generated` (greedy tokens after `prompt`) with one teacher-forced pass.

    Returns matches (tokens equal to the checker's argmax), first_mismatch (step or None), and
    per step the checker's top-2 logit margin (top1 - top2), the smallest margin and the step
    it falls on (and the checker's logits [steps, vocab] under "logits" when asked)."""
    seq = np.concatenate([np.asarray(prompt), np.asarray(generated)[:-1]])
    logits = teacher_forced_logits(weights, cfg, seq, len(prompt) - 1)
    want = logits.argmax(axis=1)
    top2 = np.sort(logits, axis=1)[:, -2:]
    margins = (top2[:, 1] - top2[:, 0]).astype(float)
    eq = want == np.asarray(generated)
    bad = np.flatnonzero(~eq)
    return {"matches": int(eq.sum()), "steps": int(len(eq)),
            "first_mismatch": int(bad[0]) if len(bad) else None,
            "margins": margins.tolist(), "min_margin": float(margins.min()),
            "min_margin_step": int(margins.argmin()), "checker_tokens": want.tolist(),
            **({"logits": logits} if return_logits else {})}
