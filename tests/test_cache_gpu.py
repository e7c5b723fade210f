"""The cache and the fused eviction call on the GPU, against the reference.

* compress on the golden inputs keeps the same positions as the reference's own
  eviction path (keep_idx_cache fixtures), up to exact ties and the neighbourhoods
  of ill-conditioned (saturated-attention) positions;
* the state machine behaves like dropkv_cache.py:493-622 (the scenarios of the
  reference's TestCacheGuards / TestChunkedPrefill / TestBudgetEviction).
"""

import numpy as np
import pytest
import torch

from parity import (DTYPE_NAME, assert_kept_report, dilate, golden_cases, input_digest, keep_set_mismatch,
                    kept_set_report, load_golden, well_conditioned)
from dropkv_b200 import DropKVCache, ops, prefill_chunked
from dropkv_b200.workloads import Workload, make_qkv
from oracle import dropkv_oracle as O

pytestmark = pytest.mark.gpu

LLAMA = dict(B=1, Hq=32, Hkv=8, D=128)


def _qkv(L, seed=0, **cfg):
    c = dict(LLAMA)
    c.update(cfg)
    wl = Workload(Lq=L, Lk=L, seed=seed, **c)
    return tuple(t.cuda() for t in make_qkv(wl, "cpu"))


@pytest.mark.parametrize("name", golden_cases())
def test_compress_matches_reference_cache_path(name):
    z, wl = load_golden(name)
    Q, K, V = make_qkv(wl, "cpu")
    assert input_digest(Q, K, V) == str(z["digest"])
    W = min(wl.window_size, wl.Lq)
    kl = O.keep_len(wl.Lk, wl.keep_ratio, wl.window_size)
    idx, kc, vc, sc = ops.compress(Q.cuda(), K.cuda(), V.cuda(), W, wl.kernel_size, kl,
                                   protect_window=wl.window_size, return_scores=True)
    idx = idx.cpu().numpy()
    ref = z["keep_idx_cache"]
    assert idx.shape == ref.shape
    # bit-exact selection given our scores
    pooled = O.pool_and_protect(sc.cpu().numpy(), wl.kernel_size, wl.window_size)
    np.testing.assert_array_equal(idx, O.select_keep_indices(pooled, kl))
    # against the reference: ties, rounding-level near-ties, saturated neighbourhoods
    Qn, Kn, Vn = (t.float().numpy() for t in (Q, K, V))
    ref_pooled = O.pool_and_protect(O.scores_cache_path(Qn, Kn, Vn, W, dtype=DTYPE_NAME[wl.dtype]),
                                    wl.kernel_size, wl.window_size)
    ill = dilate(~well_conditioned(O.max_attention(Qn, Kn, W)), wl.kernel_size // 2)
    rel = 1e-5 if wl.dtype == torch.float32 else 1e-2
    bad = keep_set_mismatch(idx, ref, ref_pooled, allowed=ill, rel_band=rel)
    assert not bad, f"{name}: kept sets differ beyond ties at {bad[:8]}"
    # gather: bit-exact rows of K/V at our indices
    it = torch.from_numpy(idx)
    ek = torch.gather(K, 2, it[..., None].expand(-1, -1, -1, wl.D))
    ev = torch.gather(V, 2, it[..., None].expand(-1, -1, -1, wl.D))
    assert torch.equal(kc.cpu(), ek) and torch.equal(vc.cpu(), ev)


@pytest.mark.parametrize("name", golden_cases())
def test_compress_matches_reference_selection(name):
    """Against the kept sets of the reference's own selection on the reference
    formula's scores with p rounded (keep_idx_round, the semantics of the
    reference's Triton branch): every difference is classified and bounded
    (parity.kept_set_report / assert_kept_report), with near-ties limited to the
    score tolerance. On sink_bf16_4k the sink (key 0) is kept where all three of
    the reference's paths keep it."""
    z, wl = load_golden(name)
    if "keep_idx_round" not in z.files:
        pytest.skip("Lq < window: no reference scorer output")
    Q, K, V = make_qkv(wl, "cpu")
    W = wl.window_size
    kl = z["keep_idx_round"].shape[-1]
    idx, _, _ = ops.compress(Q.cuda(), K.cuda(), V.cuda(), W, wl.kernel_size, kl)
    idx = idx.cpu().numpy()
    Qn, Kn = Q.float().numpy(), K.float().numpy()
    sat = O.max_attention(Qn, Kn, W) >= 0.99
    pooled = O.pool_and_protect(z["scores_round"], wl.kernel_size, W)
    rel = 1e-5 if wl.dtype == torch.float32 else 1e-2
    rep = kept_set_report(idx, z["keep_idx_round"], pooled, sat, wl.kernel_size // 2, rel_band=rel)
    print(f"\n[parity] {name} vs keep_idx_round: "
          + str({k: v for k, v in rep.items() if k != "unexplained"}))
    assert_kept_report(rep, wl.kernel_size // 2, name)
    if name == "sink_bf16_4k":
        paths = [z[f] for f in ("keep_idx_cache", "keep_idx_round", "keep_idx_exact")]
        for h in range(wl.Hkv):
            votes = {bool((p[0, h] == 0).any()) for p in paths}
            if len(votes) == 1:
                assert bool((idx[0, h] == 0).any()) == votes.pop(), f"head {h}: sink decision"


def test_chunked_equals_single_pass_bitwise():
    Q, K, V = _qkv(256, seed=1)
    single = DropKVCache(keep_ratio=0.3, window_size=8, kernel_size=11)
    single.update(Q, K, V, layer_idx=0)
    chunked = DropKVCache(keep_ratio=0.3, window_size=8, kernel_size=11)
    chunked._prefill_mode = "accumulate"
    chunked.update(Q[:, :, :128], K[:, :, :128], V[:, :, :128], layer_idx=0)
    chunked._prefill_mode = "evict_accumulated"
    chunked.update(Q[:, :, 128:], K[:, :, 128:], V[:, :, 128:], layer_idx=0)
    assert torch.equal(chunked.key_cache[0], single.key_cache[0])
    assert torch.equal(chunked.value_cache[0], single.value_cache[0])


def test_hf_four_argument_form():
    Q, K, V = _qkv(128, seed=2)
    c = DropKVCache(keep_ratio=0.3)
    rk, rv = c.update(K, V, 0, {"query_states": Q})
    assert rk.shape[-2] == 128 and c.key_cache[0].shape[-2] == max(int(0.3 * 128), 8, 1)
    c2 = DropKVCache(keep_ratio=0.3)
    c2.update(K, V, 0, {"sin": None})
    assert c2.key_cache[0].shape[-2] == 128


def test_keep_idx_and_gather_api():
    Q, K, V = _qkv(300, seed=3)
    c = DropKVCache(keep_ratio=0.25)
    idx = c._compute_keep_indices(Q, K, V)
    assert idx.shape == (1, 8, 75) and idx.dtype == torch.int64
    assert bool((idx[..., 1:] > idx[..., :-1]).all())
    assert bool((idx[..., -8:] == torch.arange(292, 300, device="cuda")).all())  # protected tail
    kc, vc = c._gather_compressed(K, V, idx)
    assert torch.equal(kc, torch.gather(K, 2, idx[..., None].expand(-1, -1, -1, 128)))
    assert c._compute_keep_indices(Q, K, V, total_tokens=2000).shape[-1] == 300
    assert c._compute_keep_indices(Q, K, V, total_tokens=2000, max_keep_len=50).shape[-1] == 50


def test_short_query_chunk_uses_shorter_window():
    """Lq < window: scoring window min(window, Lq), protection still window_size
    (reference dropkv_cache.py:399-407, 466-467)."""
    Q, K, V = _qkv(256, seed=4)
    c = DropKVCache(keep_ratio=0.3, window_size=8)
    idx = c._compute_keep_indices(Q[:, :, -4:], K, V)
    assert idx.shape == (1, 8, 76)
    assert bool((idx[..., -8:] == torch.arange(248, 256, device="cuda")).all())
    want = O.scores_reference(Q[:, :, -4:].float().cpu().numpy(), K.float().cpu().numpy(),
                              V.float().cpu().numpy(), 4, round_p="bf16")
    got = ops.scores(Q[:, :, -4:], K, V, 4).cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-3)


def test_fp32_inputs_evict_on_gpu():
    Q, K, V = _qkv(512, seed=5, dtype=torch.float32)
    c = DropKVCache(keep_ratio=0.1)
    c.update(Q, K, V, layer_idx=0)
    assert c.key_cache[0].shape == (1, 8, 51, 128) and c.key_cache[0].dtype == torch.float32


def test_budget_and_every_chunk_sequences():
    Q, K, V = _qkv(512, seed=6)
    c = DropKVCache(keep_ratio=0.3)
    c._evict_use_seen_tokens = True
    c._prefill_mode = "single_pass"
    c.update(Q[:, :, :64], K[:, :, :64], V[:, :, :64], layer_idx=0)
    assert c.key_cache[0].shape[2] == 19
    for end in (128, 192):
        c._prefill_mode = "evict_accumulated"
        c.update(Q[:, :, end - 64:end], K[:, :, end - 64:end], V[:, :, end - 64:end], layer_idx=0)
        assert c.key_cache[0].shape[2] == max(int(0.3 * end), 8, 1)
    cap = DropKVCache(keep_ratio=0.8)
    cap._evict_use_seen_tokens = True
    cap._budget_max_kv_tokens = 100
    cap._prefill_mode = "accumulate"
    cap.update(Q[:, :, :256], K[:, :, :256], V[:, :, :256], layer_idx=0)
    cap._prefill_mode = "evict_accumulated"
    cap.update(Q[:, :, 256:], K[:, :, 256:], V[:, :, 256:], layer_idx=0)
    assert cap.key_cache[0].shape[2] == 100


def test_decode_appends_after_eviction():
    Q, K, V = _qkv(128, seed=7)
    c = DropKVCache(keep_ratio=0.3)
    c.update(Q, K, V, layer_idx=0)
    n = c.key_cache[0].shape[2]
    qd, kd, vd = Q[:, :, :1].clone(), K[:, :, :1].clone(), V[:, :, :1].clone()
    rk, _ = c.update(qd, kd, vd, layer_idx=0)
    assert rk.shape[2] == n + 1 and c.get_seq_length() == 129
    assert c.get_mask_sizes(torch.arange(1), 0) == (n + 2, 0)


class _TinyModel:
    """Stand-in for a causal LM: one 'layer' whose Q/K/V are slices of fixed tensors
    at the chunk's absolute positions, written into the cache like an attention layer."""

    def __init__(self, Q, K, V, layers=2):
        self.Q, self.K, self.V, self.layers = Q, K, V, layers
        self.pos = 0

    def __call__(self, ids, past_key_values=None, use_cache=True):
        n = ids.shape[1]
        s = slice(self.pos, self.pos + n)
        for layer in range(self.layers):
            past_key_values.update(self.Q[:, :, s], self.K[:, :, s], self.V[:, :, s], layer_idx=layer)
        self.pos += n
        return n


@pytest.mark.parametrize("strategy", ["last_chunk", "budget", "every_chunk"])
def test_prefill_chunked_strategies(strategy):
    Q, K, V = _qkv(512, seed=8)
    cache = DropKVCache(keep_ratio=0.3)
    model = _TinyModel(Q, K, V)
    prefill_chunked(model, torch.zeros(1, 512), cache, chunk_size=128, evict_strategy=strategy,
                    max_kv_tokens=256)
    assert cache._seen_tokens == 512
    for layer in range(2):
        assert cache.key_cache[layer].shape[2] == max(int(0.3 * 512), 8, 1)
    assert cache._prefill_mode == "single_pass" and cache._budget_max_kv_tokens is None
    if strategy == "last_chunk":
        single = DropKVCache(keep_ratio=0.3)
        single.update(Q, K, V, layer_idx=0)
        assert torch.equal(single.key_cache[0], cache.key_cache[0])
