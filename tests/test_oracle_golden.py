"""Pin the CPU oracle against outputs of the reference itself (tests/golden).

The fixtures were produced by running the reference's ``dropkv_scores_reference``
and its PyTorch eviction path (``DropKVCache(use_triton=False)``) on seeded inputs
(tests/golden/make_golden.py).  This file needs no GPU.
"""

import numpy as np
import pytest
import torch

from parity import (DTYPE_NAME, assert_scores_close, dilate, golden_cases, input_digest,
                    keep_set_mismatch, load_golden, well_conditioned)
from dropkv_b200.workloads import make_qkv
from oracle import dropkv_oracle as O

CASES = golden_cases()


def _inputs(name):
    z, wl = load_golden(name)
    Q, K, V = make_qkv(wl, "cpu")
    assert input_digest(Q, K, V) == str(z["digest"]), (
        f"{name}: the seeded generator no longer reproduces the fixture inputs")
    return z, wl, Q.float().numpy(), K.float().numpy(), V.float().numpy()


def test_fixture_set_present():
    assert len(CASES) >= 10


@pytest.mark.parametrize("name", CASES)
def test_oracle_scores_match_reference(name):
    z, wl, Q, K, V = _inputs(name)
    if "scores_exact" not in z:
        pytest.skip("Lq < window: the reference scorer rejects it (dropkv_triton.py:62)")
    cond = well_conditioned(O.max_attention(Q, K, wl.window_size))
    se = O.scores_reference(Q, K, V, wl.window_size)
    assert_scores_close(se, z["scores_exact"], rtol=1e-5, atol=1e-6, mask=cond, what="exact")
    sr = O.scores_reference(Q, K, V, wl.window_size, round_p=DTYPE_NAME[wl.dtype])
    assert_scores_close(sr, z["scores_round"], rtol=1e-5, atol=1e-6, mask=cond, what="round")
    # ill-conditioned positions exist only where attention saturates
    assert np.isfinite(se).all() and np.isfinite(sr).all()


@pytest.mark.parametrize("name", CASES)
def test_oracle_selection_matches_reference_cache_path(name):
    z, wl, Q, K, V = _inputs(name)
    W = min(wl.window_size, wl.Lq)
    sc = O.scores_cache_path(Q, K, V, W, dtype=DTYPE_NAME[wl.dtype])
    pooled = O.pool_and_protect(sc, wl.kernel_size, wl.window_size)
    kl = O.keep_len(wl.Lk, wl.keep_ratio, wl.window_size)
    idx = O.select_keep_indices(pooled, kl)
    ref = z["keep_idx_cache"]
    assert idx.shape == ref.shape
    ill = dilate(~well_conditioned(O.max_attention(Q, K, W)), wl.kernel_size // 2)
    bad = keep_set_mismatch(idx, ref, pooled, allowed=ill)
    assert not bad, f"{name}: kept sets differ beyond ties at {bad[:8]}"
    assert (np.diff(idx, axis=-1) > 0).all(), "indices must be strictly ascending"
    Kc, Vc = O.gather_compressed(K, V, ref)
    Kc_t = torch.from_numpy(Kc).to(wl.dtype).double().sum().item()
    Vc_t = torch.from_numpy(Vc).to(wl.dtype).double().sum().item()
    assert Kc_t == pytest.approx(float(z["kc_sum"]), rel=1e-12, abs=1e-9)
    assert Vc_t == pytest.approx(float(z["vc_sum"]), rel=1e-12, abs=1e-9)


@pytest.mark.parametrize("field,sfield", [("keep_idx_round", "scores_round"), ("keep_idx_exact", "scores_exact")])
@pytest.mark.parametrize("name", CASES)
def test_oracle_select_matches_reference_select(name, field, sfield):
    """Given the reference's own scores, the oracle's pool / protect / top-k / sort
    keeps exactly the positions the reference's selection keeps
    (dropkv_cache.py:462-477); only the order of exact ties may differ."""
    z, wl = load_golden(name)
    if field not in z.files:
        pytest.skip("Lq < window: no reference scorer output")
    pooled = O.pool_and_protect(z[sfield], wl.kernel_size, wl.window_size)
    kl = z[field].shape[-1]
    idx = O.select_keep_indices(pooled, kl)
    bad = keep_set_mismatch(idx, z[field], pooled)
    assert not bad, f"{name}/{field}: kept sets differ beyond exact ties at {bad[:8]}"


SINK_HEADS = 8


def _keeps_key0(idx):
    return [bool((idx[0, h] == 0).any()) for h in range(SINK_HEADS)]


def test_reference_paths_disagree_only_where_attention_saturates():
    """sink_bf16_4k: key 0 is an attention sink whose softmax probability is 1.0
    (fp32) in some window row of every head.  There the weight (p/(1-p+eps))^2
    reaches ~1e12 and multiplies a cancelled ||v - y||^2, so each of the
    reference's own eviction paths scores the sink with its own fp32 noise
    (dropkv_triton.py:88-106, dropkv_cache.py:431-460) and keeps or evicts it by
    that noise's sign.  The paths agree everywhere else, up to the boundary
    positions those decisions displace and the near-ties the cache path's bf16 y
    moves (dropkv_cache.py:434)."""
    z, wl, Q, K, V = _inputs("sink_bf16_4k")
    pmax = O.max_attention(Q, K, wl.window_size)
    sat = pmax >= 0.99
    assert int(sat.sum()) == SINK_HEADS and sat[..., 0].all(), "exactly key 0 saturates in every head"
    cache, rnd, exact = z["keep_idx_cache"], z["keep_idx_round"], z["keep_idx_exact"]
    assert _keeps_key0(cache) == [False, True, True, True, True, False, True, True]
    assert _keeps_key0(rnd) == [True, True, False, True, False, True, True, False]
    assert _keeps_key0(exact) == [True, False, True, False, False, True, True, False]
    # the sink's raw scores are noise of either sign, orders of magnitude above the rest
    sr = z["scores_round"][0, :, 0]
    assert (np.abs(sr) > 1e5).all() and (sr < 0).any() and (sr > 0).any()
    near = dilate(sat, wl.kernel_size // 2)
    pooled = O.pool_and_protect(z["scores_round"], wl.kernel_size, wl.window_size)
    bad = keep_set_mismatch(rnd, cache, pooled, allowed=near, rel_band=2e-2)
    assert not bad, f"round vs cache path differ away from the sink at {bad[:8]}"


def test_select_breaks_ties_to_lower_index():
    pooled = np.array([[1.0, 2.0, 2.0, 2.0, 0.5, 2.0]], dtype=np.float32)
    assert O.select_keep_indices(pooled, 3).tolist() == [[1, 2, 3]]
    assert O.select_keep_indices(pooled, 5).tolist() == [[0, 1, 2, 3, 5]]


def test_ordered_keys_monotone():
    vals = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], dtype=np.float32)
    k = O.ordered_keys(vals).astype(np.int64)
    assert (np.diff(k) >= 0).all()
    assert k[3] == k[4]


def test_pool_protect_matches_torch():
    rng = np.random.default_rng(0)
    s = rng.standard_normal((2, 3, 97)).astype(np.float32)
    for ks in (1, 3, 11):
        got = O.pool_and_protect(s, ks, 8)
        t = torch.nn.functional.max_pool1d(torch.from_numpy(s), kernel_size=ks, padding=ks // 2, stride=1)
        big = t.amax(dim=-1, keepdim=True) + 1.0
        t[:, :, -8:] = big
        np.testing.assert_array_equal(got, t.numpy())


def test_keep_len_rule():
    assert O.keep_len(128, 0.3, 8) == 38
    assert O.keep_len(128, 0.3, 8, total_tokens=512) == 128
    assert O.keep_len(128, 0.3, 8, total_tokens=200) == 60
    assert O.keep_len(64, 0.01, 8, total_tokens=10) == 8
    assert O.keep_len(512, 0.8, 8, max_keep_len=100) == 100
    assert O.keep_len(32768, 0.1, 8) == 3276


def test_bf16_rounding_matches_torch():
    x = torch.randn(10000, dtype=torch.float32) * torch.logspace(-20, 20, 10000)
    x = torch.cat([x, torch.tensor([1.0 - 2 ** -9, 1.0 - 2 ** -10, 0.99951171875, 1.0])])
    got = O.round_to_bf16(x.numpy())
    np.testing.assert_array_equal(got, x.to(torch.bfloat16).float().numpy())
