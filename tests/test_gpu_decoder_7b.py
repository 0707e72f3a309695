"""configs[4] at full size: the synthetic 7B INT4 decoder (32 layers, hidden 4096, 32 / 8 heads
of 128, SwiGLU 14336, vocabulary 32000, block_size 32) decodes 128 greedy tokens after a
512-token prompt of uniform random ids, on the default route (the prompt on the tcgen05 GEMM,
every decode token one fused step on the decode GEMV), and every token must be the one the
CPU checker picks (oracle/decoder.py, fp32 throughout).

The checker runs once, teacher-forced: one pass over prompt + generated tokens gives the
logits of all 128 steps, and the tokens are the checker's own greedy decoding exactly when each
is that pass's argmax. The test reports the checker's top-2 logit margin per step (the
smallest, and where), and the GPU logits' largest deviation from the checker's, so a token
that differs can be read against the margin it differed at.
"""
import numpy as np
import pytest
import torch

from modelsharp_b200 import _native as N
from modelsharp_b200.decoder import CudaDecoder, DecoderConfig, make_weights, weights_to_host
from oracle import decoder as od

pytestmark = pytest.mark.gpu

N_PROMPT, N_NEW = 512, 128


def test_7b_greedy_tokens_match_checker(cuda_device):
    cfg = DecoderConfig()
    w = make_weights(cfg, 0, cuda_device)
    host = weights_to_host(w)
    dec = CudaDecoder(cfg, w, cuda_device)
    del w
    prompt = torch.randint(0, cfg.vocab, (N_PROMPT,), generator=torch.Generator().manual_seed(1))
    p = prompt.to(cuda_device)
    logits = [dec.prefill(p).clone()]  # default route: 512 rows on the tensor-core GEMM
    tok = torch.argmax(logits[0]).view(1)
    pos = torch.tensor([N_PROMPT], device=cuda_device)
    tokens = [tok.clone()]
    for _ in range(N_NEW - 1):
        logits.append(dec.decode_step(tok, pos).clone())
        tokens.append(tok.clone())
    torch.cuda.synchronize(cuda_device)
    assert N.lib().msq_device_status(None, None) == N.MSQ_OK, N.last_error()
    gen = torch.cat(tokens).cpu().numpy()
    gpu_logits = torch.stack(logits).cpu().numpy()
    dec.free()

    r = od.greedy_check(host, cfg, prompt.numpy(), gen, return_logits=True)
    dev = np.abs(gpu_logits - r["logits"]).max(axis=1)
    step = r["min_margin_step"]
    summary = (f"{r['matches']}/{r['steps']} tokens equal; smallest top-2 margin {r['min_margin']:.4g} at step {step} "
               f"(GPU logit deviation there {dev[step]:.3g}); largest GPU logit deviation {dev.max():.3g} "
               f"(step {int(dev.argmax())}); first mismatch {r['first_mismatch']}")
    print(summary)
    if r["first_mismatch"] is not None:
        s = r["first_mismatch"]
        summary += f"; margin at the mismatch {r['margins'][s]:.4g}, GPU deviation there {dev[s]:.3g}"
    assert r["matches"] == N_NEW, summary
