"""The INT4 decoder built on the backend against the CPU decoder of the parity checker.

A small Llama-shaped configuration (2 layers, hidden 256, 4 query / 2 key-value heads of 64,
SwiGLU 512, vocabulary 1000, block_size 32): with every projection on the exact decode
GEMV (fp32 accumulate, rel-L2 ~1e-7 per matmul) the greedy tokens must equal the checker's
and the logits must agree to 1e-5; with the prompt on the tensor-core GEMM (weights entering
as fp16) the prompt logits must agree to 5e-3. The decode step replayed from a CUDA graph
must give the same tokens as eager steps.
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import _native as N
from modelsharp_b200.decoder import CudaDecoder, DecoderConfig, make_weights, weights_to_host
from oracle import decoder as od
from oracle import oracle

pytestmark = pytest.mark.gpu

SMALL = DecoderConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512, vocab=1000, max_seq=64)


@pytest.fixture(scope="module")
def small(cuda_device):
    w = make_weights(SMALL, 3, cuda_device)
    host = weights_to_host(w)
    dec = CudaDecoder(SMALL, w, cuda_device)
    prompt = torch.randint(0, SMALL.vocab, (20,), generator=torch.Generator().manual_seed(11))
    yield dec, host, prompt
    dec.free()


def test_exact_path_tokens_and_logits_match_checker(cuda_device, small):
    dec, host, prompt = small
    n_new = 12
    ref_tokens, ref_logits = od.generate(host, SMALL, prompt.numpy(), n_new)
    logits = dec.prefill(prompt.to(cuda_device), N.PATH_GEMV)
    assert oracle.rel_l2(logits.cpu().numpy(), ref_logits[0]) <= 1e-5
    tokens = dec.generate(prompt.to(cuda_device), n_new, N.PATH_GEMV).cpu().numpy()
    np.testing.assert_array_equal(tokens, ref_tokens)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()


def test_gemm_prompt_logits_close(cuda_device, small):
    dec, host, prompt = small
    _, ref_logits = od.generate(host, SMALL, prompt.numpy(), 1)
    logits = dec.prefill(prompt.to(cuda_device), N.PATH_GEMM)  # 20 rows on the tensor-core GEMM
    assert oracle.rel_l2(logits.cpu().numpy(), ref_logits[0]) <= 5e-3


def test_graph_replayed_decode_matches_eager(cuda_device, small):
    dec, host, prompt = small
    p = prompt.to(cuda_device)
    eager = dec.generate(p, 8, N.PATH_GEMV).cpu().numpy()
    logits = dec.prefill(p, N.PATH_GEMV)
    tok = torch.argmax(logits).view(1)
    pos = torch.tensor([p.shape[0]], device=cuda_device)
    first = tok.clone()
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        dec.decode_step(tok.clone(), pos.clone())  # warm-up outside capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            dec.decode_step(tok, pos)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    # the warm-up and capture wrote cache rows; restart from the prompt
    dec.prefill(p, N.PATH_GEMV)
    tok.copy_(first)
    pos.fill_(p.shape[0])
    got = [int(first)]
    for _ in range(7):
        g.replay()
        got.append(int(tok))
    np.testing.assert_array_equal(np.asarray(got), eager)
    del g
