"""Full-path parity at the benchmark shapes: the kept sets of ``dropkv_compress``
for every KV head of a whole layer against the oracle (the reference formula,
dropkv_triton.py:29-109 with p rounded to bf16, then dropkv_cache.py:462-477).

Cases: the config-2 layer (32K keys), the 128K-token bench layer, config 4's
final eviction (Lq = 4096 tail-aligned queries over 131072 keys, keep_ratio 0.1
and 0.25), three config-5 units (the first, longest and shortest sequence of
the seeded ragged batch) and the bench layer's head shares of 1, 2 and 4 KV
heads (what one rank scores when the heads are split over 8, 4 and 2 GPUs).  Inputs are generated on the CPU from the seed and
copied to the GPU, so both sides see identical bits.

What must hold, per case:
* scores within rtol 1e-2 / atol 1e-3 of the oracle at every position whose
  softmax probability stays below 0.99 in all window rows;
* the selection is bit-exact given the kernel's own scores;
* against the oracle's kept sets, every difference falls in a class that
  ``parity.kept_set_report`` names -- the pooling neighbourhood of a saturated
  position (the attention sink; its reference score is fp32 cancellation noise
  that the reference's own paths decide differently, see
  test_oracle_golden.test_reference_paths_disagree_only_where_attention_saturates),
  the boundary positions those displace, exact ties, and near-ties within the
  score tolerance -- and each class stays within the bounds of
  ``parity.assert_kept_report``.
The per-case counts are printed (pytest -s) for the design notes.
"""

import json

import numpy as np
import pytest
import torch

from parity import assert_kept_report, assert_scores_close, kept_set_report, well_conditioned
from dropkv_b200 import ops
from dropkv_b200.sharding import ragged_lengths
from dropkv_b200.workloads import llama_layer, make_qkv
from oracle import dropkv_oracle as O

pytestmark = pytest.mark.gpu


def _cfg5_units():
    lengths = ragged_lengths(16, 4096, 65536, 5)
    picks = [0, int(np.argmax(lengths)), int(np.argmin(lengths))]
    ratios = [0.1, 0.25, 0.5]
    return [(f"cfg5_seq{s}_lk{lengths[s]}_kr{kr}", llama_layer(lengths[s], keep_ratio=kr, seed=1000 * s + 7))
            for s, kr in zip(picks, ratios)]


CASES = [
    ("cfg2_llama_32k", llama_layer(32768)),
    ("bench_llama_128k", llama_layer(131072)),
    ("cfg4_final_lq4096_kr0.1", llama_layer(131072, keep_ratio=0.1, seed=100, Lq=4096)),
    ("cfg4_final_lq4096_kr0.25", llama_layer(131072, keep_ratio=0.25, seed=100, Lq=4096)),
] + _cfg5_units()


def _check_layer(name, wl, Q, K, V):
    """The kept sets, scores and gathered rows of one ``dropkv_compress`` call on
    (Q, K, V) (CPU tensors) against the oracle; returns the kernel's outputs."""
    W, ks = wl.window_size, wl.kernel_size
    kl = wl.keep_len()
    Hkv = K.shape[1]
    D = K.shape[3]
    idx, kc, vc, sc = ops.compress(Q.cuda(), K.cuda(), V.cuda(), W, ks, kl, return_scores=True)
    idx, sc = idx.cpu().numpy(), sc.cpu().numpy()
    Qn, Kn, Vn = (t.float().numpy() for t in (Q, K, V))
    pmax = O.max_attention(Qn, Kn, W)
    sat = pmax >= 0.99
    want = O.scores_reference(Qn, Kn, Vn, W, round_p="bf16")
    assert_scores_close(sc, want, rtol=1e-2, atol=1e-3, mask=well_conditioned(pmax), what=f"{name} scores")
    # selection bit-exact given the kernel's scores
    np.testing.assert_array_equal(idx, O.select_keep_indices(O.pool_and_protect(sc, ks, W), kl))
    ref_pooled = O.pool_and_protect(want, ks, W)
    ref_idx = O.select_keep_indices(ref_pooled, kl)
    rep = kept_set_report(idx, ref_idx, ref_pooled, sat, ks // 2, rel_band=1e-2)
    key0 = {"ours": [bool((idx[0, h] == 0).any()) for h in range(Hkv)],
            "oracle": [bool((ref_idx[0, h] == 0).any()) for h in range(Hkv)]}
    print(f"\n[parity] {name}: " + json.dumps({k: v for k, v in rep.items() if k != "unexplained"})
          + f" key0={json.dumps(key0)}")
    assert_kept_report(rep, ks // 2, name)
    # gather: bit-exact rows at the kernel's indices (checked on the GPU)
    it = torch.from_numpy(idx).cuda()
    Kd = K.cuda()
    assert torch.equal(kc, torch.gather(Kd, 2, it[..., None].expand(-1, -1, -1, D)))
    del Kd
    Vd = V.cuda()
    assert torch.equal(vc, torch.gather(Vd, 2, it[..., None].expand(-1, -1, -1, D)))
    return idx, sc


@pytest.mark.parametrize("name,wl", CASES, ids=[c[0] for c in CASES])
def test_full_layer_kept_sets_match_oracle(name, wl):
    Q, K, V = make_qkv(wl, "cpu")
    _check_layer(name, wl, Q, K, V)


@pytest.mark.parametrize("nheads", [1, 2, 4])
def test_head_share_of_the_bench_layer_matches_oracle(nheads):
    """The last ``nheads`` KV heads of the 128K bench layer: the share of the last
    rank when ``bench.py --gpus N`` splits the heads over N = 8 / nheads ranks.
    Fewer heads give wider CTA groups per head (148 CTAs for one head), a merge
    over more partials and a different plan than the whole layer's."""
    wl = llama_layer(131072)
    Q, K, V = make_qkv(wl, "cpu")
    g = wl.Hq // wl.Hkv
    h0 = wl.Hkv - nheads
    Qs, Ks, Vs = Q[:, h0 * g:].contiguous(), K[:, h0:].contiguous(), V[:, h0:].contiguous()
    idx, sc = _check_layer(f"bench_llama_128k_heads{h0}-{wl.Hkv - 1}", wl, Qs, Ks, Vs)
    # the same call again, and replayed from a CUDA graph, gives the same bits
    Qd, Kd, Vd = Qs.cuda(), Ks.cuda(), Vs.cuda()
    comp = ops.Compressor(1, nheads * g, nheads, wl.Lq, wl.Lk, wl.D, wl.dtype, wl.window_size,
                          wl.kernel_size, wl.keep_len(), keep_scores=True)
    comp.run(Qd, Kd, Vd)
    np.testing.assert_array_equal(comp.scores.cpu().numpy(), sc)
    np.testing.assert_array_equal(comp.keep_idx.cpu().numpy(), idx)
    comp.capture(Qd, Kd, Vd)
    for _ in range(3):
        comp.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(comp.scores.cpu().numpy(), sc)
    np.testing.assert_array_equal(comp.keep_idx.cpu().numpy(), idx)
