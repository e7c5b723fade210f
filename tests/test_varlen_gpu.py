"""The ragged batch in one call (``dropkv_compress_varlen``): per sequence it keeps
exactly what ``dropkv_compress`` keeps with the same keep_len (the same scorer,
and a selection and gather that are exact), and keep_len itself -- evaluated on
the device from the reference's rule (dropkv_cache.py:470-473) with per-sequence
total_tokens / max_keep_len (the chunked-prefill policies, dropkv_cache.py:749-788)
-- equals the oracle's host arithmetic."""

import numpy as np
import pytest
import torch

from dropkv_b200 import _lib, ops
from dropkv_b200.workloads import Workload, make_qkv
from oracle import dropkv_oracle as O
from parity import assert_kept_report, kept_set_report, well_conditioned

pytestmark = pytest.mark.gpu


def _batch(specs, dtype=torch.bfloat16, Hq=32, Hkv=8, D=128, seed=0):
    """specs: (B, Lq, Lk) per sequence -> lists Qs, Ks, Vs (seeded, one workload each)."""
    Qs, Ks, Vs = [], [], []
    for i, (B, Lq, Lk) in enumerate(specs):
        wl = Workload(B=B, Hq=Hq, Hkv=Hkv, D=D, Lq=Lq, Lk=Lk, dtype=dtype, seed=seed + 101 * i)
        Q, K, V = make_qkv(wl, "cuda")
        Qs.append(Q)
        Ks.append(K)
        Vs.append(V)
    return Qs, Ks, Vs


def _assert_same_as_per_sequence(Qs, Ks, Vs, keep_len, outs, window=8, kernel_size=11):
    for i, (Q, K, V) in enumerate(zip(Qs, Ks, Vs)):
        kl = int(keep_len[i])
        W = min(window, Q.shape[2])
        idx, kc, vc = ops.compress(Q, K, V, W, kernel_size, kl, protect_window=window)
        gi, gk, gv = outs[i]
        assert torch.equal(gi[:, :, :kl], idx), f"sequence {i}: kept positions differ"
        assert torch.equal(gk[:, :, :kl], kc) and torch.equal(gv[:, :, :kl], vc), f"sequence {i}: rows differ"


SPECS = [
    (2, 8, 4096),     # two layers of one sequence
    (1, 8, 65536),    # the longest config-5 length
    (1, 64, 777),     # Lq > window: the last 8 rows score
    (3, 8, 20000),
    (1, 8, 8),        # Lk = window: everything kept
    (1, 4, 300),      # Lq < window: min(window, Lq) rows score, protection still covers window
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_varlen_equals_per_sequence_compress(dtype):
    Qs, Ks, Vs = _batch(SPECS, dtype=dtype, seed=3)
    keep_len, outs = ops.compress_varlen(Qs, Ks, Vs, 8, 11, 0.1)
    want = [O.keep_len(Lk, 0.1, 8) for (_, _, Lk) in SPECS]
    assert keep_len.cpu().tolist() == want
    _assert_same_as_per_sequence(Qs, Ks, Vs, keep_len.cpu(), outs)


def test_varlen_fp32_uses_the_cuda_core_scorer_and_still_matches():
    specs = [(1, 8, 1000), (2, 8, 3000)]
    Qs, Ks, Vs = _batch(specs, dtype=torch.float32, Hq=8, Hkv=2, D=64, seed=9)
    keep_len, outs = ops.compress_varlen(Qs, Ks, Vs, 8, 11, 0.25)
    _assert_same_as_per_sequence(Qs, Ks, Vs, keep_len.cpu(), outs)


def test_device_keep_len_rule_matches_the_oracle():
    """total_tokens / max_keep_len per sequence on the device, including the
    budget cap of 0 (nothing kept, outputs untouched), a negative entry (no cap),
    total_tokens far above and below Lk, and a cap below the rule."""
    specs = [(1, 8, 4096)] * 8
    Qs, Ks, Vs = _batch(specs, seed=5)
    total = [None, 20000, 100, 4096, 1 << 40, 7, 50000, 4096]
    mkl = [None, 500, 3000, 0, -1, 2, None, 100]
    caps = [4096, 4096, 4096, 4096, 4096, 4096, 300, 4096]
    kr = 0.3
    comp = ops.VarlenCompressor([(1, 8, 4096)] * 8, 32, 8, 128, torch.bfloat16, 8, 11, kr, caps=caps)
    sentinel = 123456789
    for idx, kc, vc in comp.outputs:
        idx.fill_(sentinel)
    tt = torch.tensor([4096 if t is None else t for t in total], dtype=torch.int64, device="cuda")
    keep_len, outs = comp.run(Qs, Ks, Vs, total_tokens=tt, max_keep_len=mkl)
    got = keep_len.cpu().tolist()
    want = []
    for t, m, cap in zip(total, mkl, caps):
        kl = O.keep_len(4096, kr, 8, total_tokens=4096 if t is None else t,
                        max_keep_len=None if (m is None or m < 0) else m)
        want.append(min(kl, cap))
    assert got == want
    assert got[3] == 0 and bool((outs[3][0] == sentinel).all()), "keep_len 0 leaves the outputs untouched"
    _assert_same_as_per_sequence([q for q, k in zip(Qs, got) if k], [k for k, n in zip(Ks, got) if n],
                                 [v for v, n in zip(Vs, got) if n], [k for k in got if k],
                                 [o for o, n in zip(outs, got) if n])
    for i, kl in enumerate(got):  # rows past keep_len are untouched
        if 0 < kl < caps[i]:
            assert bool((outs[i][0][:, :, kl:] == sentinel).all())


def test_varlen_matches_the_oracle_on_a_small_ragged_batch():
    specs = [(1, 8, 600), (1, 8, 2500), (2, 8, 1300)]
    Qs, Ks, Vs = _batch(specs, Hq=8, Hkv=2, D=64, seed=21)
    keep_len, outs = ops.compress_varlen(Qs, Ks, Vs, 8, 11, 0.1)
    for i, (Q, K, V) in enumerate(zip(Qs, Ks, Vs)):
        Qn, Kn, Vn = (t.float().cpu().numpy() for t in (Q, K, V))
        s = O.scores_reference(Qn, Kn, Vn, 8, round_p="bf16")
        pooled = O.pool_and_protect(s, 11, 8)
        kl = int(keep_len[i])
        assert kl == O.keep_len(K.shape[2], 0.1, 8)
        want = O.select_keep_indices(pooled, kl)
        got = outs[i][0][:, :, :kl].cpu().numpy()
        sat = ~well_conditioned(O.max_attention(Qn, Kn, 8))
        rep = kept_set_report(got, want, pooled, sat, 5, 1e-2)
        assert_kept_report(rep, 5, f"sequence {i}")
        Kc, Vc = O.gather_compressed(Kn, Vn, got)
        np.testing.assert_array_equal(outs[i][1][:, :, :kl].float().cpu().numpy(), Kc)
        np.testing.assert_array_equal(outs[i][2][:, :, :kl].float().cpu().numpy(), Vc)


def test_more_sequences_than_one_call_takes():
    n = _lib.VARLEN_MAX_SEQS + 3
    specs = [(1, 8, 64 + 37 * i) for i in range(n)]
    Qs, Ks, Vs = _batch(specs, Hq=4, Hkv=1, D=64, seed=1)
    keep_len, outs = ops.compress_varlen(Qs, Ks, Vs, 8, 11, 0.5)
    assert keep_len.cpu().tolist() == [O.keep_len(Lk, 0.5, 8) for (_, _, Lk) in specs]
    _assert_same_as_per_sequence(Qs, Ks, Vs, keep_len.cpu(), outs)


def test_varlen_call_is_one_c_call_and_graph_capturable():
    specs = [(2, 8, 5000), (1, 8, 12000)]
    Qs, Ks, Vs = _batch(specs, seed=8)
    comp = ops.VarlenCompressor(specs, 32, 8, 128, torch.bfloat16, 8, 11, 0.1,
                                caps=[O.keep_len(Lk, 0.1, 8) for (_, _, Lk) in specs])
    n0 = _lib.launch_count()
    comp.run(Qs, Ks, Vs)
    torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    assert launches == 2 * len(specs) + 2, "per sequence a memset and a scorer; one select, one gather"
    first = [tuple(t.clone() for t in o) for o in comp.outputs]
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        comp.run(Qs, Ks, Vs)
    torch.cuda.current_stream().wait_stream(side)
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        comp.run(Qs, Ks, Vs)
    for o in comp.outputs:
        for t in o:
            t.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(first, comp.outputs):
        assert all(torch.equal(x, y) for x, y in zip(a, b))


def test_varlen_status_word_collects_a_scorer_timeout():
    """The test hook makes every tensor-core scorer launch give up at its first
    group barrier after 1 ms: the OR of the status words in the varlen workspace
    is non-zero, and with the hook off the next call is correct again."""
    specs = [(1, 8, 8192), (1, 8, 4096)]
    Qs, Ks, Vs = _batch(specs, seed=13)
    comp = ops.VarlenCompressor(specs, 32, 8, 128, torch.bfloat16, 8, 11, 0.1)
    lib = _lib.load()
    _lib.check(lib.dropkv_test_scorer_waits(1_000_000, 1), "test hook")
    try:
        with pytest.raises(_lib.DropKVError) as err:
            comp.run(Qs, Ks, Vs)  # DROPKV_CHECK_STATUS=1 (tests/conftest.py) reads the status word
        assert err.value.code == _lib.ERR_DEVICE
    finally:
        _lib.check(lib.dropkv_test_scorer_waits(0, 0), "test hook off")
    keep_len, outs = comp.run(Qs, Ks, Vs)
    assert int(comp.workspace[:4].view(torch.int32).item()) == 0
    _assert_same_as_per_sequence(Qs, Ks, Vs, keep_len.cpu(), outs)
