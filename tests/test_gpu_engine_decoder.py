"""The decoder as a graph run by the engine's node loop, against the CPU decoder of the checker.

build_decoder_graph turns the small Llama-shaped decoder into MatMulNBits, norm, attention,
SwiGLU and ArgMax nodes; CudaEngine runs it one token at a time on the CUDA registry of
llm_ops, as built and after graph_fusion folds norms, SwiGLU and residual adds into
MatMulNBitsFused nodes. Every projection takes the exact decode GEMV, so the greedy tokens must equal the
checker's and the CudaDecoder's, and the logits that chose the first token must agree with
the checker's to 1e-5 relative L2 (the prompt goes through one run of all its tokens); on the
default route the prompt's projections take the tensor-core GEMM and its logits agree to 5e-3.
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import _native as N
from modelsharp_b200.decoder import CudaDecoder, DecoderConfig, EngineDecoder, make_weights, weights_to_host
from oracle import decoder as od
from oracle import oracle

pytestmark = pytest.mark.gpu

SMALL = DecoderConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512, vocab=1000, max_seq=64)


@pytest.fixture(scope="module")
def setup(cuda_device):
    w = make_weights(SMALL, 3, cuda_device)
    host = weights_to_host(w)
    prompt = torch.randint(0, SMALL.vocab, (20,), generator=torch.Generator().manual_seed(11))
    yield w, host, prompt


@pytest.mark.parametrize("fuse", [False, True])
def test_engine_tokens_and_logits_match_checker(cuda_device, setup, fuse):
    w, host, prompt = setup
    n_new = 10
    ref_tokens, ref_logits = od.generate(host, SMALL, prompt.numpy(), n_new)
    eng = EngineDecoder(SMALL, w, cuda_device, fuse=fuse, path=N.PATH_GEMV)
    if fuse:
        assert {n.op_type for n in eng.graph.nodes} == {"Gather", "MatMulNBitsFused", "GroupQueryAttention", "ArgMax"}
    tokens, first_logits = eng.generate(prompt.to(cuda_device), n_new)
    assert oracle.rel_l2(first_logits.cpu().numpy(), ref_logits[0]) <= 1e-5
    np.testing.assert_array_equal(tokens.cpu().numpy(), ref_tokens)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()


def test_engine_matches_direct_decoder(cuda_device, setup):
    w, _, prompt = setup
    dec = CudaDecoder(SMALL, w, cuda_device)
    direct = dec.generate(prompt.to(cuda_device), 8, N.PATH_GEMV).cpu().numpy()
    dec.free()
    eng = EngineDecoder(SMALL, w, cuda_device, path=N.PATH_GEMV)
    tokens, _ = eng.generate(prompt.to(cuda_device), 8)
    np.testing.assert_array_equal(tokens.cpu().numpy(), direct)


def test_engine_step_writes_the_cache_row(cuda_device, setup):
    w, _, _ = setup
    eng = EngineDecoder(SMALL, w, cuda_device)
    pk = eng.graph.initializers["l1.past_key"]
    pk.zero_()
    out = eng.step(torch.tensor([[5]], device=cuda_device), 3)
    torch.cuda.synchronize(cuda_device)
    assert out["next_token"].shape == (1, 1) and out["logits"].shape == (1, 1, SMALL.vocab)
    rows = pk[0].abs().sum(dim=(0, 2)).cpu().numpy()
    assert rows[3] > 0 and np.count_nonzero(rows) == 1  # only row 3 of the cache was written


def test_engine_graph_replay_matches_eager(cuda_device, setup):
    w, _, prompt = setup
    eng = EngineDecoder(SMALL, w, cuda_device, path=N.PATH_GEMV)
    eager, eager_logits = eng.generate(prompt.to(cuda_device), 8)
    eng.capture()
    replayed, replay_logits = eng.generate(prompt.to(cuda_device), 8)
    eng.release()
    np.testing.assert_array_equal(replayed.cpu().numpy(), eager.cpu().numpy())
    assert torch.equal(replay_logits, eager_logits)


def test_engine_prompt_on_tensor_cores(cuda_device, setup):
    """The default route: the 20-token prompt's projections on the tensor-core GEMM (weights
    entering as fp16), attention over the prompt in one run; logits within 5e-3."""
    w, host, prompt = setup
    _, ref_logits = od.generate(host, SMALL, prompt.numpy(), 1)
    eng = EngineDecoder(SMALL, w, cuda_device)
    out = eng.prefill(prompt.to(cuda_device))
    assert oracle.rel_l2(out["logits"].reshape(-1).cpu().numpy(), ref_logits[0]) <= 5e-3
