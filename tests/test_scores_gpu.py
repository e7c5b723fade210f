"""Parity of the CUDA scorer with the reference (golden fixtures) and the oracle.

Tolerances: fp32 inputs rtol 1e-5 / atol 1e-6; bf16/fp16 inputs with exact p
rtol 1e-3 / atol 1e-4 (the reference's own kernel-vs-reference tolerance,
tests/test_dropkv_triton.py:136 of the reference); with p rounded to the input
dtype rtol 1e-2 / atol 1e-3 (a rounding flip of one p changes its weight by up to
2^-7 relative).  Positions where attention saturates (max p >= 0.99) are
ill-conditioned in the reference formula and are checked for finiteness only.
"""

import math
import zlib

import numpy as np
import pytest
import torch

from parity import (DTYPE_NAME, assert_scores_close, golden_cases, input_digest, load_golden,
                    well_conditioned)
from dropkv_b200 import ops
from dropkv_b200.workloads import Workload, make_qkv
from oracle import dropkv_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-6), torch.float16: (1e-3, 1e-4), torch.bfloat16: (1e-3, 1e-4)}
TOL_ROUND = (1e-2, 1e-3)


def _golden_inputs(name):
    z, wl = load_golden(name)
    Q, K, V = make_qkv(wl, "cpu")
    assert input_digest(Q, K, V) == str(z["digest"])
    return z, wl, Q, K, V


@pytest.mark.parametrize("name", golden_cases())
def test_scores_match_reference_golden(name):
    z, wl, Q, K, V = _golden_inputs(name)
    if "scores_exact" not in z:
        pytest.skip("Lq < window: no reference scores")
    cond = well_conditioned(O.max_attention(Q.float().numpy(), K.float().numpy(), wl.window_size))
    Qc, Kc, Vc = Q.cuda(), K.cuda(), V.cuda()
    got = ops.scores(Qc, Kc, Vc, wl.window_size, round_p=False).cpu().numpy()
    rtol, atol = TOL[wl.dtype]
    assert_scores_close(got, z["scores_exact"], rtol, atol, mask=cond, what=f"{name} exact")
    got_r = ops.scores(Qc, Kc, Vc, wl.window_size, round_p=True).cpu().numpy()
    rtol, atol = (TOL_ROUND if wl.dtype != torch.float32 else TOL[wl.dtype])
    assert_scores_close(got_r, z["scores_round"], rtol, atol, mask=cond, what=f"{name} round")


@pytest.mark.parametrize("cfg", [
    dict(B=1, Hq=32, Hkv=8, D=128, Lq=64, Lk=512),     # Llama, Lq < Lk
    dict(B=1, Hq=14, Hkv=2, D=64, Lq=64, Lk=512),      # Qwen M=56
    dict(B=2, Hq=32, Hkv=8, D=128, Lq=64, Lk=256),     # batch 2
    dict(B=1, Hq=8, Hkv=8, D=128, Lq=32, Lk=256),      # MHA
    dict(B=1, Hq=4, Hkv=2, D=128, Lq=64, Lk=8192),     # split-K heavy
    dict(B=1, Hq=8, Hkv=2, D=32, Lq=16, Lk=300),       # D=32
    dict(B=1, Hq=4, Hkv=1, D=256, Lq=16, Lk=333),      # D=256
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_scores_match_oracle(cfg, dtype):
    wl = Workload(dtype=dtype, seed=zlib.crc32(repr((cfg, str(dtype))).encode()) % 1000, **cfg)
    Q, K, V = make_qkv(wl, "cpu")
    Qn, Kn, Vn = (t.float().numpy() for t in (Q, K, V))
    cond = well_conditioned(O.max_attention(Qn, Kn, 8))
    want = O.scores_reference(Qn, Kn, Vn, 8)
    got = ops.scores(Q.cuda(), K.cuda(), V.cuda(), 8, round_p=False).cpu().numpy()
    assert_scores_close(got, want, *TOL[dtype], mask=cond)
    if dtype != torch.float32:
        want_r = O.scores_reference(Qn, Kn, Vn, 8, round_p=DTYPE_NAME[dtype])
        got_r = ops.scores(Q.cuda(), K.cuda(), V.cuda(), 8, round_p=True).cpu().numpy()
        assert_scores_close(got_r, want_r, *TOL_ROUND, mask=cond)


def test_large_window_beyond_tile():
    """window 65 > a 64-key tile: splits past the causal bound stay NaN-free
    (reference tests/test_dropkv_triton.py:1654-1743)."""
    wl = Workload(B=1, Hq=4, Hkv=2, D=128, Lq=1344, Lk=1344, window_size=65, seed=7)
    Q, K, V = make_qkv(wl, "cpu")
    got = ops.scores(Q.cuda(), K.cuda(), V.cuda(), 65, round_p=False).cpu().numpy()
    assert np.isfinite(got).all()
    Qn, Kn, Vn = (t.float().numpy() for t in (Q, K, V))
    want = O.scores_reference(Qn, Kn, Vn, 65)
    cond = well_conditioned(O.max_attention(Qn, Kn, 65))
    assert_scores_close(got, want, *TOL[torch.bfloat16], mask=cond)


def test_noncontiguous_q_and_determinism():
    wl = Workload(B=1, Hq=32, Hkv=8, D=128, Lq=64, Lk=640, seed=3)
    Q, K, V = (t.cuda() for t in make_qkv(wl, "cpu"))
    Qnc = Q.transpose(2, 3).contiguous().transpose(2, 3)
    assert not Qnc.is_contiguous()
    a = ops.dropkv_scores_cuda(Q, K, V)
    b = ops.dropkv_scores_cuda(Qnc, K, V)
    c = ops.dropkv_scores_cuda(Q, K, V)
    assert torch.equal(a, b) and torch.equal(a, c)


def test_l_equals_w_finite():
    wl = Workload(B=1, Hq=32, Hkv=8, D=128, Lq=8, Lk=8, seed=4)
    Q, K, V = (t.cuda() for t in make_qkv(wl, "cpu"))
    s = ops.dropkv_scores_cuda(Q, K, V, match_pytorch_precision=False)
    assert torch.isfinite(s).all()


def test_zero_values_give_zero_scores():
    """With V = 0 every term of the score vanishes: no masked or padded row may
    leak a non-zero (or NaN) contribution."""
    wl = Workload(B=1, Hq=4, Hkv=1, D=64, Lq=8, Lk=200, seed=5)
    Q, K, V = (t.cuda() for t in make_qkv(wl, "cpu"))
    s = ops.scores(Q, K, torch.zeros_like(V), 8, round_p=False)
    assert torch.count_nonzero(s) == 0


@pytest.mark.parametrize("Lk", [32768, 131072])
def test_full_size_llama_layer_properties(Lk):
    """BASELINE shapes: finite scores, and one head against the oracle."""
    from dropkv_b200.workloads import llama_layer
    wl = llama_layer(Lk)
    Q, K, V = make_qkv(wl, "cuda")
    s = ops.dropkv_scores_cuda(Q, K, V, match_pytorch_precision=False)
    assert s.shape == (1, 8, Lk) and torch.isfinite(s).all()
    h = 3
    Qn = Q[:, 4 * h:4 * h + 4].float().cpu().numpy()
    Kn = K[:, h:h + 1].float().cpu().numpy()
    Vn = V[:, h:h + 1].float().cpu().numpy()
    want = O.scores_reference(Qn, Kn, Vn, 8)
    cond = well_conditioned(O.max_attention(Qn, Kn, 8))
    assert_scores_close(s[:, h:h + 1].cpu().numpy(), want, *TOL[torch.bfloat16], mask=cond)
