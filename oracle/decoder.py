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
