"""Host-side checks of the decoder around the op (no GPU).

* the 7B shape's MatMulNBits bytes per decoded token (the unit of the decode roofline);
* the CPU checker's decoder (oracle/decoder.py) against itself: a token decoded through the
  KV cache gives the logits of a full pass over the whole sequence, so the cache, rotary
  positions and causal masking of the checker are consistent before the GPU is compared
  with it;
* the algebra the fused decode GEMV relies on: RMSNorm folded in as x * gamma with the
  1/rms scale applied to the dot product equals norm-then-MatMulNBits to fp32 rounding.
"""
import numpy as np
import pytest

from modelsharp_b200.decoder import DecoderConfig, make_weights, proj_shapes, weight_bytes_per_token, weights_to_host
from oracle import decoder as od
from oracle import oracle

TINY = DecoderConfig(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, inter=96, vocab=50, max_seq=24)


def test_7b_bytes_per_token():
    assert weight_bytes_per_token(DecoderConfig()) == 4_555_096_064


def test_projection_shapes_agree_with_checker():
    for cfg in (DecoderConfig(), TINY):
        assert proj_shapes(cfg) == od.proj_shapes(cfg)


@pytest.fixture(scope="module")
def tiny_weights():
    return weights_to_host(make_weights(TINY, 5, "cpu"))


def _cache(cfg):
    return {"k": np.zeros((cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim), np.float32),
            "v": np.zeros((cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim), np.float32),
            "rope": od.rope_tables(cfg)}


def test_checker_cached_decoding_equals_full_pass(tiny_weights):
    rng = np.random.default_rng(3)
    tokens = rng.integers(0, TINY.vocab, 12)
    full = od.forward(tiny_weights, TINY, tokens, 0, _cache(TINY))       # [12, vocab]
    cache = _cache(TINY)
    od.forward(tiny_weights, TINY, tokens[:7], 0, cache)
    for p in range(7, 12):
        step = od.forward(tiny_weights, TINY, tokens[p:p + 1], p, cache)[0]
        assert oracle.rel_l2(step, full[p]) <= 1e-5


def test_checker_generate_is_greedy(tiny_weights):
    prompt = np.asarray([1, 7, 3, 9])
    toks, logits = od.generate(tiny_weights, TINY, prompt, 5)
    assert len(toks) == 5 and len(logits) == 5
    for t, lg in zip(toks, logits):
        assert t == int(np.argmax(lg))


def test_rope_tables_and_single_key_attention():
    cos, sin = od.rope_tables(TINY)
    np.testing.assert_allclose(cos * cos + sin * sin, 1.0, rtol=1e-6)
    np.testing.assert_array_equal(cos[0], 1.0)
    np.testing.assert_array_equal(sin[0], 0.0)
    rng = np.random.default_rng(4)
    q = rng.standard_normal((1, TINY.heads * TINY.head_dim)).astype(np.float32)
    kc = rng.standard_normal((TINY.kv_heads, TINY.max_seq, TINY.head_dim)).astype(np.float32)
    vc = rng.standard_normal((TINY.kv_heads, TINY.max_seq, TINY.head_dim)).astype(np.float32)
    out = od.attention(q, kc, vc, 0, TINY).reshape(TINY.heads, TINY.head_dim)
    group = TINY.heads // TINY.kv_heads
    for h in range(TINY.heads):  # one visible key: the output is its value row
        np.testing.assert_allclose(out[h], vc[h // group, 0], rtol=1e-6)


@pytest.mark.parametrize("bs", [32, 128])
def test_rmsnorm_folded_into_the_dot_product(bs):
    """(x * gamma) . W^T scaled by 1/rms equals rms_norm(x) . W^T to fp32 rounding."""
    from modelsharp_b200 import synth
    K, N_ = 512, 96
    c = synth.make_case(9, 2, N_, K, 4, bs, "packed", scale_lo=0.001, scale_hi=0.01)
    rng = np.random.default_rng(bs)
    x = (rng.standard_normal((2, K)) * 3).astype(np.float32)
    gamma = rng.uniform(0.8, 1.2, K).astype(np.float32)
    ref = oracle.managed(dict(c, a=od.rms_norm(x, gamma, 1e-5), M=2))
    inv = 1.0 / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-5)
    folded = oracle.managed(dict(c, a=(x * gamma).astype(np.float32), M=2)) * inv
    assert oracle.rel_l2(folded, ref) <= 1e-6


def test_decoder_graph_is_wired_for_the_engine():
    """Every node input is a graph input, an initializer or an earlier node's output, and every
    op type has a kernel in the decoder registry."""
    from modelsharp_b200.decoder import build_decoder_graph
    from modelsharp_b200.llm_ops import create_decoder_registry
    w = make_weights(TINY, 5, "cpu")
    g = build_decoder_graph(TINY, w, "cpu")
    known = set(g.inputs) | set(g.initializers)
    reg = create_decoder_registry("cpu")
    for node in g.nodes:
        for name in node.inputs:
            assert name == "" or name in known, (node.name, name)
        known |= {o for o in node.outputs if o}
        assert reg.try_get(node.op_type)[0], node.op_type
    assert set(g.outputs) <= known
    ops = [n.op_type for n in g.nodes]
    assert ops.count("MatMulNBits") == 5 * TINY.layers + 1
    assert ops.count("GroupQueryAttention") == TINY.layers
    assert g.initializers["l0.past_key"].shape == (1, TINY.kv_heads, TINY.max_seq, TINY.head_dim)


def test_engine_rejects_unknown_ops_and_unsupported_forms():
    from modelsharp_b200 import CudaEngine, GraphContext, GraphNode, ModelGraph, UnsupportedOperatorException
    from modelsharp_b200.errors import ModelSharpException
    from modelsharp_b200.llm_ops import GroupQueryAttentionKernel, create_decoder_registry
    g = ModelGraph(["x"], ["y"], [GraphNode("RotaryEmbedding", "r", ["x"], ["y"])])
    with pytest.raises(UnsupportedOperatorException):
        CudaEngine(g, create_decoder_registry("cpu")).run({"x": np.zeros(4, np.float32)})
    gqa = GroupQueryAttentionKernel()
    base = {"num_heads": 4, "kv_num_heads": 2, "do_rotary": 1}
    unpacked = GraphNode("GroupQueryAttention", "a", ["q", "k", "v", "pk", "pv", "s", "", "c", "n"], ["o"], base)
    with pytest.raises(ModelSharpException, match="packed QKV"):
        gqa.execute(unpacked, GraphContext({}))
    no_rotary = GraphNode("GroupQueryAttention", "a", ["q", "", "", "pk", "pv", "s", "", "c", "n"], ["o"],
                          dict(base, do_rotary=0))
    with pytest.raises(ModelSharpException, match="do_rotary"):
        gqa.execute(no_rotary, GraphContext({}))


# ---- the engine-level fusion pass, checked with a CPU executor of the graph's op types
def _np(t):
    return t.numpy() if hasattr(t, "numpy") else np.asarray(t)


def _ref_run(graph, feeds, cfg, state):
    """Runs a decoder graph on the CPU with the checker's restatements (state: the KV caches)."""
    env = {k: v for k, v in graph.initializers.items()}
    env.update(state)
    env.update(feeds)
    cos, sin = od.rope_tables(cfg)

    def mnb(node, a):
        n, k, bs = (int(node.attributes[x]) for x in ("N", "K", "block_size"))
        a2 = np.ascontiguousarray(np.asarray(a, np.float32).reshape(-1, k))
        case = dict(a=a2, b=_np(env[node.inputs[1]]), scales=_np(env[node.inputs[2]]).reshape(-1),
                    zp=_np(env[node.inputs[3]]), zp_kind="packed", M=a2.shape[0], N=n, K=k, bits=4, block_size=bs)
        return oracle.managed(case).reshape(*np.asarray(a).shape[:-1], n)

    for node in graph.nodes:
        op, ins = node.op_type, node.inputs
        if op == "Gather":
            out = [_np(env[ins[0]])[np.asarray(env[ins[1]]).reshape(-1)].reshape(1, 1, -1)]
        elif op == "SimplifiedLayerNormalization":
            out = [od.rms_norm(env[ins[0]], _np(env[ins[1]]), node.attributes["epsilon"])]
        elif op == "SkipSimplifiedLayerNormalization":
            s = (env[ins[0]] + env[ins[1]]).astype(np.float32)
            out = [od.rms_norm(s, _np(env[ins[2]]), node.attributes["epsilon"]), None, None, s]
        elif op == "MatMulNBits":
            out = [mnb(node, env[ins[0]])]
        elif op == "MatMulNBitsFused":
            x = np.asarray(env[ins[0]], np.float32)
            if ins[4]:
                x = od.rms_norm(x, _np(env[ins[4]]), node.attributes["epsilon"])
            if int(node.attributes.get("swiglu", 0)):
                k = int(node.attributes["K"])
                gt, up = x[..., :k], x[..., k:]
                x = (gt / (np.float32(1.0) + np.exp(-gt)) * up).astype(np.float32)
            y = mnb(node, x)
            out = [(env[ins[5]] + y).astype(np.float32) if len(ins) > 5 and ins[5] else y]
        elif op == "GroupQueryAttention":
            h, kvh, d = node.attributes["num_heads"], node.attributes["kv_num_heads"], cfg.head_dim
            qkv = np.asarray(env[ins[0]]).reshape(1, -1)
            pos = int(np.asarray(env[ins[5]]).reshape(-1)[0])
            p = np.asarray([pos])
            q = od.rope(qkv[:, :h * d], h, d, p, cos, sin)
            k = od.rope(qkv[:, h * d:(h + kvh) * d], kvh, d, p, cos, sin)
            kc, vc = env[ins[3]], env[ins[4]]
            kc[0, :, pos] = k.reshape(kvh, d)
            vc[0, :, pos] = qkv[0, (h + kvh) * d:].reshape(kvh, d)
            out = [od.attention(q, kc[0], vc[0], pos, cfg).reshape(1, 1, -1), kc, vc]
        elif op == "Sigmoid":
            out = [(1.0 / (1.0 + np.exp(-env[ins[0]]))).astype(np.float32)]
        elif op == "Mul":
            out = [(env[ins[0]] * env[ins[1]]).astype(np.float32)]
        elif op == "ArgMax":
            out = [np.argmax(env[ins[0]], axis=-1)]
        else:
            raise AssertionError(op)
        for name, v in zip(node.outputs, out):
            if name:
                env[name] = v
    return {o: env[o] for o in graph.outputs}


def _ref_generate(graph, cfg, prompt, n_new):
    state = {k: np.zeros(tuple(v.shape), np.float32) for k, v in graph.initializers.items() if "past_" in k}
    out, toks, logits = None, [], []
    for i, t in enumerate(prompt):
        out = _ref_run(graph, {"input_ids": np.asarray([[t]]), "seqlens_k": np.asarray([i])}, cfg, state)
    for j in range(n_new):
        toks.append(int(out["next_token"].reshape(-1)[0]))
        logits.append(out["logits"].reshape(-1))
        if j + 1 < n_new:
            out = _ref_run(graph, {"input_ids": np.asarray([[toks[-1]]]), "seqlens_k": np.asarray([len(prompt) + j])},
                           cfg, state)
    return toks, logits


def test_fusion_pass_structure_and_semantics():
    from modelsharp_b200.decoder import build_decoder_graph
    from modelsharp_b200.graph_fusion import fuse_decode_graph
    from modelsharp_b200.llm_ops import create_decoder_registry
    w = make_weights(TINY, 5, "cpu")
    g = build_decoder_graph(TINY, w, "cpu")
    f = fuse_decode_graph(g)
    ops = [n.op_type for n in f.nodes]
    assert ops.count("MatMulNBitsFused") == 4 * TINY.layers + 1
    for gone in ("MatMulNBits", "SimplifiedLayerNormalization", "SkipSimplifiedLayerNormalization", "Sigmoid", "Mul"):
        assert gone not in ops, gone
    assert len(f.nodes) == 5 * TINY.layers + 3  # Gather, 5 per layer, LM head, ArgMax
    assert [n.op_type for n in g.nodes].count("Sigmoid") == TINY.layers  # the source graph is untouched
    known = set(f.inputs) | set(f.initializers)
    reg = create_decoder_registry("cpu")
    for node in f.nodes:
        assert all(x == "" or x in known for x in node.inputs), node.name
        known |= {o for o in node.outputs if o}
        assert reg.try_get(node.op_type)[0]
    prompt = [3, 17, 42, 8, 1]
    t_plain, l_plain = _ref_generate(g, TINY, prompt, 3)
    t_fused, l_fused = _ref_generate(f, TINY, prompt, 3)
    assert t_plain == t_fused
    for a, b in zip(l_plain, l_fused):
        assert oracle.rel_l2(b, a) <= 1e-5
    # the plain graph's CPU run is the checker's decoder
    ref_tokens, _ = od.generate(weights_to_host(w), TINY, np.asarray(prompt), 3)
    assert t_plain == list(ref_tokens)


def test_fusion_keeps_a_residual_that_is_read_later():
    """No in-place add into a value that a later node still reads."""
    from modelsharp_b200 import GraphNode, ModelGraph
    from modelsharp_b200.graph_fusion import fuse_decode_graph
    mnb = {"N": 8, "K": 8, "bits": 4, "block_size": 32}
    nodes = [GraphNode("MatMulNBits", "p", ["a", "B", "S", "Z"], ["y"], mnb),
             GraphNode("SkipSimplifiedLayerNormalization", "n", ["y", "r", "g"], ["h", "", "", "s"], {}),
             GraphNode("MatMulNBits", "c", ["h", "B", "S", "Z"], ["o"], mnb),
             GraphNode("Mul", "late", ["r", "o"], ["z"])]
    g = ModelGraph(["a", "r"], ["z"], nodes, {"B": 0, "S": 0, "Z": 0, "g": 0})
    f = fuse_decode_graph(g)
    assert [n.op_type for n in f.nodes] == [n.op_type for n in nodes]  # r is a graph input and read later


def test_fusion_leaves_unmatched_patterns_alone():
    """Gate and up of different widths, a norm whose output is read by a non-MatMulNBits node and
    a SwiGLU without zero points stay as they are."""
    from modelsharp_b200 import GraphNode, ModelGraph
    from modelsharp_b200.graph_fusion import fuse_decode_graph

    def mnb(name, a, n, k, zp=True):
        return GraphNode("MatMulNBits", name, [a, name + ".B", name + ".S"] + ([name + ".Z"] if zp else []), [name],
                         {"N": n, "K": k, "bits": 4, "block_size": 32})

    def swiglu(gate_n, up_n, zp=True):
        return [mnb("gate", "h", gate_n, 64, zp), mnb("up", "h", up_n, 64, zp),
                GraphNode("Sigmoid", "sg", ["gate"], ["sg"]), GraphNode("Mul", "si", ["gate", "sg"], ["si"]),
                GraphNode("Mul", "act", ["si", "up"], ["act"]), mnb("down", "act", 64, gate_n, zp)]

    inits = {f"{n}.{t}": 0 for n in ("gate", "up", "down") for t in ("B", "S", "Z")}
    for nodes in (swiglu(128, 96), swiglu(128, 128, zp=False)):
        g = ModelGraph(["h"], ["down"], nodes, dict(inits))
        assert [n.op_type for n in fuse_decode_graph(g).nodes] == [n.op_type for n in nodes]
    norm_read_elsewhere = [GraphNode("SimplifiedLayerNormalization", "n", ["x", "g"], ["h"], {"epsilon": 1e-5}),
                           mnb("p", "h", 64, 64), GraphNode("Mul", "m", ["h", "p"], ["z"])]
    g = ModelGraph(["x"], ["z"], norm_read_elsewhere, {"g": 0, "p.B": 0, "p.S": 0, "p.Z": 0})
    assert [n.op_type for n in fuse_decode_graph(g).nodes] == [n.op_type for n in norm_read_elsewhere]
