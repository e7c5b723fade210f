"""Layers stacked along the batch axis (the ragged bench's per-sequence batching).

One ``dropkv_compress`` call over L layers of one sequence ([L, Hkv, Lk, D])
must give every layer what a call over that layer alone gives: the scores within
floating-point reordering (the launch may split the rows over a different number
of CTAs, so partial sums are merged in another order), and, given the batched
call's own scores, exactly the kept indices and rows that the per-row selection
and gather produce.
"""

import numpy as np
import pytest
import torch

from dropkv_b200 import ops
from dropkv_b200.workloads import llama_layer, make_qkv

pytestmark = pytest.mark.gpu


def _stack(L, Lk, seed0):
    qs, ks, vs = [], [], []
    for i in range(L):
        q, k, v = make_qkv(llama_layer(Lk, seed=seed0 + i), "cuda")
        qs.append(q)
        ks.append(k)
        vs.append(v)
    return torch.cat(qs), torch.cat(ks), torch.cat(vs)


@pytest.mark.parametrize("round_p", [False, True])
@pytest.mark.parametrize("L,Lk", [(32, 4096), (6, 40000), (3, 65536)])
def test_layers_batched_match_single(L, Lk, round_p):
    Q, K, V = _stack(L, Lk, 100 * L)
    wl = llama_layer(Lk)
    kl = wl.keep_len()
    comp = ops.Compressor(L, wl.Hq, wl.Hkv, wl.Lq, Lk, wl.D, wl.dtype, wl.window_size, wl.kernel_size, kl,
                          round_p=round_p, keep_scores=True)
    idx, kc, vc = comp.run(Q, K, V)
    torch.cuda.synchronize()
    # exact p: only the order of fp32 partial sums differs. p rounded to bf16: a
    # reordered sum may flip one rounding (2^-8 relative in p), so the bf16
    # tolerance of the score tests applies.
    rtol, atol = (1e-2, 1e-3) if round_p else (1e-4, 1e-9)
    for layer in range(L):
        s1 = ops.scores(Q[layer:layer + 1], K[layer:layer + 1], V[layer:layer + 1], wl.window_size,
                        round_p=round_p)[0]
        sb = comp.scores[layer]
        # key 0 is the attention sink of this distribution: p near 1 makes its score
        # ill-conditioned, so only its finiteness is compared
        assert torch.isfinite(sb).all()
        np.testing.assert_allclose(sb[:, 1:].cpu().numpy(), s1[:, 1:].cpu().numpy(), rtol=rtol, atol=atol)
        want = ops.select_keep_indices(comp.scores[layer:layer + 1], wl.kernel_size, wl.window_size, kl)
        assert torch.equal(idx[layer:layer + 1], want)
        kw, vw = ops.gather_compressed(K[layer:layer + 1], V[layer:layer + 1], want)
        assert torch.equal(kc[layer:layer + 1].view(torch.int16), kw.view(torch.int16))
        assert torch.equal(vc[layer:layer + 1].view(torch.int16), vw.view(torch.int16))
