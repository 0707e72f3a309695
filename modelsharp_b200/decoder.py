"""A Llama-shaped INT4 decoder whose every projection is MatMulNBits on this backend.

The end-to-end workload of the op (synthetic 7B shape: 32 layers, hidden 4096, 32 query /
8 key-value heads of 128, SwiGLU 14336, vocabulary 32000, every projection bits=4 with
block_size 32 and zero points): the packed q/k/v, o, packed gate/up and down projections and
the LM head run on libms_cuda_nbits (the tensor-core GEMM for a prompt, the decode GEMV per
token). The glue between them (RMSNorm, rotary embedding, causal grouped-query attention over
a KV cache, SwiGLU, residual adds, greedy argmax) is float32: torch for the prompt pass, the
library's fused glue kernels for a decode step. Its semantics follow the reference's CPU
kernels: SimplifiedLayerNormalizationKernel.cs:48-54 (RMSNorm), RotaryEmbeddingKernel.cs:96-114
(half-split rotary), GroupQueryAttentionKernel.cs:194-195, 275-312 (causal GQA, 1/sqrt(d) scale).

Weights are drawn on the device from a seeded torch generator (uniform codes and zero
points, scales uniform in [scale_lo, scale_hi], an N(0, 1) embedding table).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from .errors import ModelSharpException
from .weights import QuantizedWeights

PROJ = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass(frozen=True)
class DecoderConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 14336
    vocab: int = 32000
    block_size: int = 32
    rope_theta: float = 1e4
    eps: float = 1e-5
    max_seq: int = 640
    scale_lo: float = 0.001
    scale_hi: float = 0.01


def proj_shapes(cfg: DecoderConfig) -> dict[str, tuple[int, int]]:
    """(N, K) of every projection of a layer."""
    h, kv, i = cfg.hidden, cfg.kv_heads * cfg.head_dim, cfg.inter
    return {"q": (cfg.heads * cfg.head_dim, h), "k": (kv, h), "v": (kv, h), "o": (h, cfg.heads * cfg.head_dim),
            "gate": (i, h), "up": (i, h), "down": (h, i)}


def weight_bytes_per_token(cfg: DecoderConfig) -> int:
    """Algorithmic MatMulNBits bytes one decode step reads: codes, fp32 scales, packed zp."""
    from .synth import algorithmic_bytes
    per_layer = sum(algorithmic_bytes(n, k, 4, cfg.block_size, "packed") for n, k in proj_shapes(cfg).values())
    return cfg.layers * per_layer + algorithmic_bytes(cfg.vocab, cfg.hidden, 4, cfg.block_size, "packed")


def _quant(n: int, k: int, cfg: DecoderConfig, g: torch.Generator, dev: torch.device) -> dict:
    nb = -(-k // cfg.block_size)
    return {"b": torch.randint(0, 256, (n, nb, cfg.block_size // 2), dtype=torch.uint8, device=dev, generator=g),
            "scales": torch.empty(n * nb, device=dev).uniform_(cfg.scale_lo, cfg.scale_hi, generator=g),
            "zp": torch.randint(0, 256, (n, -(-nb // 2)), dtype=torch.uint8, device=dev, generator=g)}


def make_weights(cfg: DecoderConfig, seed: int, device: torch.device | str) -> dict:
    """Every weight of the decoder in the op's reference layouts, on `device`."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    shapes = proj_shapes(cfg)
    layers = []
    for _ in range(cfg.layers):
        lw = {name: _quant(*shapes[name], cfg, g, dev) for name in PROJ}
        lw["norm_attn"] = torch.empty(cfg.hidden, device=dev).uniform_(0.8, 1.2, generator=g)
        lw["norm_mlp"] = torch.empty(cfg.hidden, device=dev).uniform_(0.8, 1.2, generator=g)
        layers.append(lw)
    return {"layers": layers,
            "embed": torch.randn(cfg.vocab, cfg.hidden, device=dev, generator=g),
            "norm_final": torch.empty(cfg.hidden, device=dev).uniform_(0.8, 1.2, generator=g),
            "lm_head": _quant(cfg.vocab, cfg.hidden, cfg, g, dev)}


def weights_to_host(w: dict) -> dict:
    """numpy copy (for the parity checker)."""
    if isinstance(w, dict):
        return {k: weights_to_host(v) for k, v in w.items()}
    if isinstance(w, list):
        return [weights_to_host(v) for v in w]
    return w.cpu().numpy()


def _cat(ws: list[dict]) -> dict:
    """Weights stacked along N (the output rows): one projection computing several at once."""
    return {"b": torch.cat([w["b"] for w in ws]), "scales": torch.cat([w["scales"].reshape(-1) for w in ws]),
            "zp": torch.cat([w["zp"] for w in ws])}


class CudaDecoder:
    """Greedy decoding with the projections on libms_cuda_nbits.

    q/k/v are packed into one weight (N = (H + 2 Hkv) d) and gate/up into another (N = 2 I), as
    packed-QKV exports do, so a layer runs four MatMulNBits. The prompt pass uses the library's
    row forms of the glue (causal prompt attention included; torch only gathers embedding rows);
    a decode step folds RMSNorm, SwiGLU and the residual adds into its GEMVs and uses the
    library's fused rotary + KV append + GQA decode and argmax kernels, every launch chained
    with programmatic dependent launch."""

    def __init__(self, cfg: DecoderConfig, weights: dict, device: torch.device | str):
        self.cfg = cfg
        self.device = dev = torch.device(device)
        shapes = proj_shapes(cfg)
        self.n_q, self.n_kv = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim

        def pack(w, n, k):
            return QuantizedWeights(w["b"], w["scales"], w["zp"], n, k, 4, cfg.block_size, device=dev)

        self.layers = []
        for lw in weights["layers"]:
            self.layers.append({
                "qkv": pack(_cat([lw["q"], lw["k"], lw["v"]]), self.n_q + 2 * self.n_kv, cfg.hidden),
                "o": pack(lw["o"], *shapes["o"]),
                "gate_up": pack(_cat([lw["gate"], lw["up"]]), 2 * cfg.inter, cfg.hidden),
                "down": pack(lw["down"], *shapes["down"]),
                "norm_attn": lw["norm_attn"], "norm_mlp": lw["norm_mlp"]})
        self.lm_head = pack(weights["lm_head"], cfg.vocab, cfg.hidden)
        self.embed = weights["embed"]
        self.norm_final = weights["norm_final"]
        half = cfg.head_dim // 2
        inv = cfg.rope_theta ** (-np.arange(half, dtype=np.float64) * 2.0 / cfg.head_dim)
        ang = np.arange(cfg.max_seq, dtype=np.float64)[:, None] * inv[None, :]
        self.cos = torch.from_numpy(np.cos(ang).astype(np.float32)).to(dev)
        self.sin = torch.from_numpy(np.sin(ang).astype(np.float32)).to(dev)
        shape = (cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim)
        self.kc = torch.zeros(shape, device=dev)
        self.vc = torch.zeros(shape, device=dev)
        # decode-step buffers (fixed addresses, so a captured step can be replayed)
        f = dict(device=dev, dtype=torch.float32)
        self.bx = torch.empty(1, cfg.hidden, **f)
        self.bqkv = torch.empty(1, self.n_q + 2 * self.n_kv, **f)
        self.battn = torch.empty(1, self.n_q, **f)
        self.bgu, self.blogits = torch.empty(1, 2 * cfg.inter, **f), torch.empty(1, cfg.vocab, **f)

    # ---- prompt pass
    def prefill(self, tokens: torch.Tensor, path: int = N.PATH_AUTO_SPLIT) -> torch.Tensor:
        """Runs the prompt from position 0; returns the last position's logits [vocab]. The
        default route puts the prompt's projections on the split-operand tcgen05 GEMM (products
        good to ~2^-22): the greedy tokens that follow must be the fp32 reference's, and this
        decoder amplifies a projection's error about a hundredfold through its 32 layers, which
        the fp16 GEMM's 2^-11 operands (PATH_AUTO) do not survive.

        Every step is a library launch: add + RMSNorm (the residual add of the previous block
        folded in), the projections, rotary of the S tokens with k and v appended to the cache
        (msq_rope_append_rows), causal attention over the cache (msq_gqa_prefill) and SwiGLU
        (msq_swiglu_rows); torch only gathers the embedding rows."""
        cfg, lib = self.cfg, N.lib()
        st = torch.cuda.current_stream(self.device).cuda_stream
        s = tokens.shape[0]
        if s < 1 or s > cfg.max_seq:
            raise ModelSharpException(f"prompt of {s} tokens does not fit max_seq {cfg.max_seq}")

        def ok(rc, what):
            if rc:
                N.check(rc, what)

        f = dict(device=self.device, dtype=torch.float32)
        x = torch.index_select(self.embed, 0, tokens).contiguous()  # [S, hidden]: the residual stream
        h = torch.empty_like(x)
        q = torch.empty(s, self.n_q, **f)
        attn = torch.empty(s, self.n_q, **f)
        act = torch.empty(s, cfg.inter, **f)

        def add_norm(delta, gamma):  # x += delta (if any); h = RMSNorm(x) * gamma
            ok(lib.msq_add_rmsnorm(None, st, x.data_ptr(), None if delta is None else delta.data_ptr(),
                                   gamma.data_ptr(), h.data_ptr(), s, cfg.hidden, cfg.eps), "msq_add_rmsnorm")

        delta = None
        for li, lw in enumerate(self.layers):
            add_norm(delta, lw["norm_attn"])
            qkv = lw["qkv"].matmul(h, path=path)
            ok(lib.msq_rope_append_rows(None, st, qkv.data_ptr(), s, 0, cfg.heads, cfg.kv_heads, cfg.head_dim,
                                        self.cos.data_ptr(), self.sin.data_ptr(), q.data_ptr(), self.kc[li].data_ptr(),
                                        self.vc[li].data_ptr(), cfg.max_seq), "msq_rope_append_rows")
            ok(lib.msq_gqa_prefill(None, st, q.data_ptr(), self.kc[li].data_ptr(), self.vc[li].data_ptr(), s, 0,
                                   attn.data_ptr(), cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.max_seq),
               "msq_gqa_prefill")
            add_norm(lw["o"].matmul(attn, path=path), lw["norm_mlp"])
            gu = lw["gate_up"].matmul(h, path=path)
            ok(lib.msq_swiglu_rows(None, st, gu.data_ptr(), act.data_ptr(), s, cfg.inter), "msq_swiglu_rows")
            delta = lw["down"].matmul(act, path=path)
        add_norm(delta, self.norm_final)
        return self.lm_head.matmul(h[-1:], path=path)[0]

    # ---- fused decode step
    def decode_step(self, tok: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """One token: tok [1] (int64) at position pos [1] (int64), both on the device; writes
        the argmax into tok, advances pos and returns the logits [vocab]. Only device memory
        changes, so the step can be captured in a CUDA graph and replayed.

        Per layer five launches: q/k/v GEMV with the attention RMSNorm folded in; rotary, KV
        append and GQA in one; o GEMV adding into the residual; gate/up GEMV with the MLP
        RMSNorm folded in; down GEMV taking SwiGLU of its input and adding into the residual."""
        cfg, lib = self.cfg, N.lib()
        st = torch.cuda.current_stream(self.device).cuda_stream

        def ok(rc, what):
            if rc:
                N.check(rc, what)

        torch.index_select(self.embed, 0, tok, out=self.bx)
        for li, lw in enumerate(self.layers):
            lw["qkv"].matmul_fused(self.bx, self.bqkv, rms_gamma=lw["norm_attn"], rms_eps=cfg.eps, stream=st)
            ok(lib.msq_rope_gqa_decode(None, st, self.bqkv.data_ptr(), cfg.heads, cfg.kv_heads, cfg.head_dim,
                                       self.cos.data_ptr(), self.sin.data_ptr(), pos.data_ptr(), self.kc[li].data_ptr(),
                                       self.vc[li].data_ptr(), self.battn.data_ptr(), cfg.max_seq),
               "msq_rope_gqa_decode")
            lw["o"].matmul_fused(self.battn, self.bx, accumulate=True, stream=st)
            lw["gate_up"].matmul_fused(self.bx, self.bgu, rms_gamma=lw["norm_mlp"], rms_eps=cfg.eps, stream=st)
            lw["down"].matmul_fused(self.bgu, self.bx, swiglu=True, accumulate=True, stream=st)
        self.lm_head.matmul_fused(self.bx, self.blogits, rms_gamma=self.norm_final, rms_eps=cfg.eps, stream=st)
        ok(lib.msq_argmax(None, st, self.blogits.data_ptr(), cfg.vocab, tok.data_ptr(), pos.data_ptr()), "msq_argmax")
        return self.blogits[0]

    def generate(self, prompt: torch.Tensor, n_new: int, path: int = N.PATH_AUTO_SPLIT) -> torch.Tensor:
        """Greedy: the prompt in one pass, then n_new - 1 decode steps; the new tokens [n_new]."""
        logits = self.prefill(prompt, path)
        tok = torch.argmax(logits).view(1)
        pos = torch.tensor([prompt.shape[0]], device=self.device)
        out = [tok.clone()]
        for _ in range(n_new - 1):
            self.decode_step(tok, pos)
            out.append(tok.clone())
        return torch.cat(out)

    def free(self) -> None:
        for lw in self.layers:
            for name in ("qkv", "o", "gate_up", "down"):
                lw[name].free()
        self.lm_head.free()


# ---------------------------------------------------------------- the same decoder as a graph
def build_decoder_graph(cfg: DecoderConfig, weights: dict, device: torch.device | str):
    """The decoder as an in-memory graph of the op types an INT4 decoder export uses, for the
    engine's node loop (one token per run).

    Inputs: `input_ids` int64 [1, 1] and `seqlens_k` int64 [1] (the token's position), both on
    the device. Outputs: `logits` [1, 1, vocab] and `next_token` int64 [1, 1] (greedy). Per
    layer: SimplifiedLayerNormalization (layer 0) or SkipSimplifiedLayerNormalization (the
    residual add of the previous layer), MatMulNBits of the packed q/k/v, GroupQueryAttention
    (packed QKV, rotary in the op, the layer's KV cache as past/present), MatMulNBits o,
    SkipSimplifiedLayerNormalization, MatMulNBits gate and up, Sigmoid and two Mul (SwiGLU),
    MatMulNBits down; then the final SkipSimplifiedLayerNormalization, the LM head and ArgMax.
    The KV caches are initializers the attention nodes update in place."""
    from .kernels import GraphNode, ModelGraph
    dev = torch.device(device)
    n_q, n_kv = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    init: dict = {"embed": weights["embed"], "final_norm": weights["norm_final"]}
    half = cfg.head_dim // 2
    inv = cfg.rope_theta ** (-np.arange(half, dtype=np.float64) * 2.0 / cfg.head_dim)
    ang = np.arange(cfg.max_seq, dtype=np.float64)[:, None] * inv[None, :]
    init["cos_cache"] = torch.from_numpy(np.cos(ang).astype(np.float32)).to(dev)
    init["sin_cache"] = torch.from_numpy(np.sin(ang).astype(np.float32)).to(dev)
    nodes: list = []

    def mnb(name: str, a: str, w: dict, n: int, k: int, out: str) -> None:
        init[f"{name}.B"] = w["b"]
        init[f"{name}.scales"] = w["scales"].reshape(-1)
        init[f"{name}.zero_points"] = w["zp"]
        nodes.append(GraphNode("MatMulNBits", name, [a, f"{name}.B", f"{name}.scales", f"{name}.zero_points"], [out],
                               {"N": n, "K": k, "bits": 4, "block_size": cfg.block_size}))

    eps = {"epsilon": cfg.eps}
    nodes.append(GraphNode("Gather", "embed", ["embed", "input_ids"], ["x_0"], {"axis": 0}))
    resid, pending = "x_0", None  # pending: the previous layer's down-projection output
    for li, lw in enumerate(weights["layers"]):
        p = f"l{li}."
        init[p + "attn_norm"], init[p + "mlp_norm"] = lw["norm_attn"], lw["norm_mlp"]
        cache = (1, cfg.kv_heads, cfg.max_seq, cfg.head_dim)
        init[p + "past_key"] = torch.zeros(cache, device=dev)
        init[p + "past_value"] = torch.zeros(cache, device=dev)
        if pending is None:
            nodes.append(GraphNode("SimplifiedLayerNormalization", p + "attn_norm", [resid, p + "attn_norm"],
                                   [p + "h"], eps))
        else:
            nodes.append(GraphNode("SkipSimplifiedLayerNormalization", p + "attn_norm",
                                   [pending, resid, p + "attn_norm"], [p + "h", "", "", p + "resid_a"], eps))
            resid = p + "resid_a"
        mnb(p + "qkv", p + "h", _cat([lw["q"], lw["k"], lw["v"]]), n_q + 2 * n_kv, cfg.hidden, p + "qkv")
        nodes.append(GraphNode("GroupQueryAttention", p + "attn",
                               [p + "qkv", "", "", p + "past_key", p + "past_value", "seqlens_k", "",
                                "cos_cache", "sin_cache"],
                               [p + "attn", p + "present_key", p + "present_value"],
                               {"num_heads": cfg.heads, "kv_num_heads": cfg.kv_heads, "do_rotary": 1}))
        mnb(p + "o", p + "attn", lw["o"], cfg.hidden, n_q, p + "o")
        nodes.append(GraphNode("SkipSimplifiedLayerNormalization", p + "mlp_norm", [p + "o", resid, p + "mlp_norm"],
                               [p + "h2", "", "", p + "resid_b"], eps))
        resid = p + "resid_b"
        mnb(p + "gate", p + "h2", lw["gate"], cfg.inter, cfg.hidden, p + "gate")
        mnb(p + "up", p + "h2", lw["up"], cfg.inter, cfg.hidden, p + "up")
        nodes.append(GraphNode("Sigmoid", p + "sig", [p + "gate"], [p + "sig"]))
        nodes.append(GraphNode("Mul", p + "silu", [p + "gate", p + "sig"], [p + "silu"]))
        nodes.append(GraphNode("Mul", p + "act", [p + "silu", p + "up"], [p + "act"]))
        mnb(p + "down", p + "act", lw["down"], cfg.hidden, cfg.inter, p + "down")
        pending = p + "down"
    nodes.append(GraphNode("SkipSimplifiedLayerNormalization", "final_norm", [pending, resid, "final_norm"],
                           ["h_final", "", "", "resid_final"], eps))
    mnb("lm_head", "h_final", weights["lm_head"], cfg.vocab, cfg.hidden, "logits")
    nodes.append(GraphNode("ArgMax", "argmax", ["logits"], ["next_token"], {"axis": -1, "keepdims": 0}))
    return ModelGraph(["input_ids", "seqlens_k"], ["logits", "next_token"], nodes, init)


class EngineDecoder:
    """Greedy decoding through the engine: the graph of build_decoder_graph run by CudaEngine
    on the registry of llm_ops (MatMulNBits and the decoder's other op types on the device),
    one token per run after the prompt, which goes through one run of all its tokens.
    With fuse (the default) the graph first goes through graph_fusion.fuse_decode_graph, which
    folds the norms, SwiGLU and residual adds into MatMulNBitsFused nodes."""

    def __init__(self, cfg: DecoderConfig, weights: dict, device: torch.device | str, fuse: bool = True,
                 path: int = N.PATH_AUTO_SPLIT):
        from .engine import CudaEngine
        from .graph_fusion import fuse_decode_graph
        from .llm_ops import create_decoder_registry
        self.cfg = cfg
        self.device = torch.device(device)
        self.graph = build_decoder_graph(cfg, weights, self.device)
        if fuse:
            self.graph = fuse_decode_graph(self.graph)
        self.engine = CudaEngine(self.graph, create_decoder_registry(self.device, path))
        self._graph = None

    def step(self, tok: torch.Tensor, pos: int) -> dict:
        """One run: tok int64 [1, 1] on the device at position pos."""
        if self._graph is not None:
            self._tok.copy_(tok.reshape(1, 1))
            self._pos.fill_(pos)
            self._graph.replay()
            return self._out
        p = torch.full((1,), pos, dtype=torch.int64, device=self.device)
        return self.engine.run({"input_ids": tok, "seqlens_k": p})

    def capture(self) -> None:
        """Captures one engine run in a CUDA graph over fixed input buffers; later steps copy
        the token and position in and replay it (every value of a run stays on the device and
        the positions are read there, so the node loop's launches replay unchanged). The
        warm-up run before the capture writes cache row 0, which the next prompt rewrites."""
        self._tok = torch.zeros(1, 1, dtype=torch.int64, device=self.device)
        self._pos = torch.zeros(1, dtype=torch.int64, device=self.device)
        cur = torch.cuda.current_stream(self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            self.engine.run({"input_ids": self._tok, "seqlens_k": self._pos})
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._out = self.engine.run({"input_ids": self._tok, "seqlens_k": self._pos})
        cur.wait_stream(s)
        self._graph = g

    def release(self) -> None:
        self._graph, self._out = None, None

    def prefill(self, ids: torch.Tensor) -> dict:
        """The whole prompt (int64 [S] on the device) in one eager run from position 0; the last
        position's `logits` [1, 1, vocab] and `next_token` [1, 1]."""
        out = self.engine.run({"input_ids": ids.reshape(1, -1),
                               "seqlens_k": torch.full((1,), ids.numel() - 1, dtype=torch.int64, device=self.device)})
        return {"logits": out["logits"][:, -1:], "next_token": out["next_token"][:, -1:]}

    def generate(self, prompt: torch.Tensor, n_new: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The n_new greedy tokens after the prompt, and the logits that chose the first."""
        ids = prompt.to(self.device, torch.int64).reshape(-1)
        if ids.numel() + n_new - 1 > self.cfg.max_seq:
            raise ModelSharpException(f"prompt of {ids.numel()} tokens + {n_new} new exceeds max_seq {self.cfg.max_seq}")
        out = self.prefill(ids)
        first_logits = out["logits"].reshape(-1).clone()
        toks = [out["next_token"].reshape(1).clone()]
        for j in range(1, n_new):
            out = self.step(toks[-1].reshape(1, 1), ids.numel() + j - 1)
            toks.append(out["next_token"].reshape(1).clone())
        return torch.cat(toks), first_logits
