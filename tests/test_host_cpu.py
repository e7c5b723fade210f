"""Host-side logic that needs no GPU: the C ABI library's exports, the wrapper's
precondition checks (same AssertionError texts as dropkv_triton.py:679-707), the
cache state machine paths that do not evict, and prefill_chunked's validation and
cleanup (the reference's fake-model tests, tests/test_dropkv_triton.py:845-1331)."""

import ctypes
import os
import re

import pytest
import torch

import dropkv_b200
from dropkv_b200 import DropKVCache, _lib, ops, prefill_chunked
from dropkv_b200.workloads import keep_len_rule

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "dropkv_b200.h")).read()
    return sorted(set(re.findall(r"DROPKV_API\s+[\w\s\*]+?\b(dropkv_\w+)\s*\(", hdr)))


def test_library_loads_and_exports_every_declared_symbol():
    syms = _declared_symbols()
    assert len(syms) >= 9
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/dropkv_b200.h but not exported"
    assert set(syms) <= set(_lib.SIGNATURES), "ctypes binding misses a declared symbol"
    assert dropkv_b200.version().startswith("dropkv_b200")


def test_workspace_queries_without_gpu():
    lib = _lib.load()
    n = lib.dropkv_scores_workspace_size(1, 32, 8, 32768, 128, 8)
    assert n > 0 and n % 256 == 0
    assert lib.dropkv_select_workspace_size(1, 8, 32768) >= 8 * 32768 * 4
    assert lib.dropkv_compress_workspace_size(1, 32, 8, 32768, 128, 8) > n
    assert lib.dropkv_scores_workspace_size(1, 7, 2, 100, 128, 8) == 0  # Hq % Hkv != 0


def test_c_abi_rejects_bad_arguments_without_touching_the_gpu():
    lib = _lib.load()
    rc = lib.dropkv_scores(None, 0, 0, 0, 0, 8, None, None, 2, 1, 32, 8, 64, 128, 8, 1e-6, 1,
                           None, None, 0, None)
    assert rc == _lib.ERR_ARG
    assert "non-NULL" in lib.dropkv_last_error().decode()
    rc = lib.dropkv_select(None, 1, 8, 100, 10, 8, 10, None, None, 0, None)
    assert rc == _lib.ERR_ARG and "odd" in lib.dropkv_last_error().decode()
    rc = lib.dropkv_select(None, 1, 8, 100, 11, 8, 101, None, None, 0, None)
    assert rc == _lib.ERR_ARG and "keep_len" in lib.dropkv_last_error().decode()


def _varlen_seqs(specs, align=4096):
    """ctypes table of a ragged batch with placeholder (never dereferenced) pointers."""
    seqs = (_lib.VarlenSeq * len(specs))()
    for i, (B, Lq, Lk, cap) in enumerate(specs):
        sq = seqs[i]
        sq.q, sq.k, sq.v = align, 2 * align, 3 * align
        sq.q_sb, sq.q_sh, sq.q_ss, sq.q_sd = 32 * Lq * 128, Lq * 128, 128, 1
        sq.Lq, sq.B, sq.Lk, sq.cap = Lq, B, Lk, cap
        sq.keep_idx, sq.k_out, sq.v_out = 4 * align, 5 * align, 6 * align
    return seqs


def test_varlen_workspace_layout_without_gpu():
    lib = _lib.load()
    specs = [(2, 8, 1000, 100), (1, 8, 70000, 7000), (3, 16, 4096, 4096)]
    seqs = _varlen_seqs(specs)
    n = lib.dropkv_compress_varlen_workspace_size(3, seqs, 32, 8, 128, 8)
    scratch = max(lib.dropkv_scores_workspace_size(B, 32, 8, Lk, 128, min(8, Lq)) for B, Lq, Lk, _ in specs)
    rows = 0
    for B, _, Lk, _ in specs:
        rows += -(-(B * 8 * Lk * 4) // 256) * 256  # each sequence's score rows, 256-byte aligned
    assert n == -(-(256 + scratch) // 256) * 256 + rows
    assert lib.dropkv_compress_varlen_workspace_size(0, seqs, 32, 8, 128, 8) == 0
    assert lib.dropkv_compress_varlen_workspace_size(_lib.VARLEN_MAX_SEQS + 1, seqs, 32, 8, 128, 8) == 0


@pytest.mark.parametrize("change,code,text", [
    (dict(n=0), _lib.ERR_ARG, "n_seq"),
    (dict(n=_lib.VARLEN_MAX_SEQS + 1), _lib.ERR_ARG, "n_seq"),
    (dict(keep_ratio=0.0), _lib.ERR_ARG, "keep_ratio"),
    (dict(keep_ratio=1.5), _lib.ERR_ARG, "keep_ratio"),
    (dict(keep_ratio=float("nan")), _lib.ERR_ARG, "keep_ratio"),
    (dict(cap=0), _lib.ERR_ARG, "cap"),
    (dict(cap=5001), _lib.ERR_ARG, "cap"),
    (dict(Lk=300000, cap=10), _lib.ERR_UNSUPPORTED, "one-launch selection"),
    (dict(B=9000), _lib.ERR_ARG, "65535"),
    (dict(k=4100), _lib.ERR_ARG, "16-byte"),
    (dict(kernel_size=4), _lib.ERR_ARG, "odd"),
    (dict(keep_len_out=None), _lib.ERR_ARG, "keep_len_out"),
])
def test_varlen_rejects_bad_arguments_without_touching_the_gpu(change, code, text):
    lib = _lib.load()
    B, Lk, cap = change.get("B", 1), change.get("Lk", 5000), change.get("cap", 500)
    seqs = _varlen_seqs([(1, 8, 1000, 100), (B, 8, Lk, cap)])
    if "k" in change:
        seqs[1].k = change["k"]
    n = change.get("n", 2)
    rc = lib.dropkv_compress_varlen(n, seqs, _lib.DTYPE_BF16, 32, 8, 128, 8, 1e-6, _lib.ROUND_BF16,
                                    change.get("kernel_size", 11), 8, change.get("keep_ratio", 0.1), 8, None,
                                    None, change.get("keep_len_out", 4096), None, 0, None)
    assert rc == code
    assert text in lib.dropkv_last_error().decode()


def test_kv_stride_detection_for_model_views():
    """A model's [B, L, Hkv, D] projections viewed as [B, Hkv, L, D] are read in
    place (strides passed to dropkv_compress_kv_strides); layouts with split rows
    or strides off 16-byte multiples are not."""
    B, L, H, D = 2, 40, 4, 64
    k = torch.zeros(B, L, H, D, dtype=torch.bfloat16).transpose(1, 2)
    assert ops._kv_strides(k, k) == (L * H * D, D, H * D)
    assert ops._kv_strides(k[:1], k[:1]) == (H * D, D, H * D)   # B = 1: the batch stride is moot
    rows_split = torch.zeros(B, H, L, 2 * D, dtype=torch.bfloat16)[..., ::2]
    assert ops._kv_strides(rows_split, rows_split) is None
    odd = torch.zeros(B, L, H, D + 4, dtype=torch.bfloat16).transpose(1, 2)[..., :D]
    assert ops._kv_strides(odd, odd) is None          # a row stride of 68 elements: not 16-byte aligned
    packed = torch.zeros(B, H, L, D, dtype=torch.bfloat16)
    assert ops._kv_strides(packed, packed) == (H * L * D, L * D, D)
    assert ops._kv_strides(k, packed) is None         # K and V must share the layout


def test_kv_strides_entry_rejects_bad_strides_without_touching_the_gpu():
    lib = _lib.load()
    base = 4096
    for sb, sh, ss in [(0, 64, 128), (4096, 64, 60), (4096, 68, 128), (4100, 64, 128)]:
        rc = lib.dropkv_compress_kv_strides(base, 0, 0, 0, 1, 8, base, base, sb, sh, ss, _lib.DTYPE_BF16, 1, 8, 2,
                                            100, 64, 8, 1e-6, _lib.ROUND_BF16, 11, 8, 10, None, base, base, base,
                                            base, 1 << 20, None)
        assert rc == _lib.ERR_ARG, (sb, sh, ss)
        assert "strides" in lib.dropkv_last_error().decode()


def _mk(B=1, Hq=32, Hkv=8, Lq=64, Lk=64, D=128, dtype=torch.bfloat16):
    return (torch.randn(B, Hq, Lq, D).to(dtype), torch.randn(B, Hkv, Lk, D).to(dtype),
            torch.randn(B, Hkv, Lk, D).to(dtype))


@pytest.mark.parametrize("kw,shape,match", [
    (dict(window_size=0), {}, "positive int"),
    ({}, dict(Lq=4, Lk=4), "must be >= window_size"),
    ({}, dict(Lq=4, Lk=256), r"Lq.*must be >= window_size"),
    ({}, dict(Lq=64, Lk=4), r"Lk.*must be >= window_size"),
    ({}, dict(Lq=512, Lk=64), r"Lq.*must be <= Lk"),
    ({}, dict(Hq=7, Hkv=4), "divisible"),
    ({}, {}, "CUDA"),
])
def test_scores_guards_match_reference(kw, shape, match):
    Q, K, V = _mk(**shape)
    with pytest.raises(AssertionError, match=match):
        ops.dropkv_scores_cuda(Q, K, V, **kw)


def test_product_path_refuses_cpu_tensors():
    Q, K, V = _mk()
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.scores(Q, K, V, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.compress(Q, K, V, 8, 11, 16)


def test_keep_len_rule_matches_reference_arithmetic():
    assert keep_len_rule(128, 0.3, 8) == 38
    assert keep_len_rule(128, 0.3, 8, total_tokens=512) == 128
    assert keep_len_rule(128, 0.3, 8, total_tokens=200) == 60
    assert keep_len_rule(64, 0.01, 8, total_tokens=10) == 8
    assert keep_len_rule(512, 0.8, 8, max_keep_len=100) == 100
    c = DropKVCache(keep_ratio=0.3, window_size=8)
    assert c._keep_len(128, None, None) == 38 and c._keep_len(128, 200, None) == 60


def test_constructor_validation():
    with pytest.raises(ValueError, match="keep_ratio"):
        DropKVCache(keep_ratio=0.0)
    with pytest.raises(ValueError, match="window_size"):
        DropKVCache(window_size=0)
    with pytest.raises(ValueError, match="kernel_size"):
        DropKVCache(kernel_size=4)
    with pytest.raises(NotImplementedError):
        DropKVCache().batch_split(2, 1)


def test_state_machine_paths_without_eviction():
    Q, K, V = _mk(Lq=64, Lk=64)
    c = DropKVCache(keep_ratio=0.3)
    c._prefill_mode = "accumulate"
    c.update(Q[:, :, :32], K[:, :, :32], V[:, :, :32], layer_idx=0)
    assert c.key_cache[0].shape[2] == 32 and c._seen_tokens == 32
    c.update(Q[:, :, 32:], K[:, :, 32:], V[:, :, 32:], layer_idx=0)
    assert c.key_cache[0].shape[2] == 64 and c._seen_tokens == 64
    # HF 4-arg call without query_states: stored in full
    c2 = DropKVCache()
    c2.update(K, V, 0, {"sin": None})
    assert c2.key_cache[0].shape[2] == 64
    # sequence shorter than the window: stored in full
    c3 = DropKVCache(window_size=16)
    c3.update(Q[:, :, :8], K[:, :, :8], V[:, :, :8], layer_idx=0)
    assert c3.key_cache[0].shape[2] == 8
    # skipped layer index
    with pytest.raises(ValueError, match="Use DynamicCache"):
        DropKVCache().update(Q, K, V, layer_idx=2)


def test_invalid_modes_raise():
    Q, K, V = _mk(Lq=8, Lk=8)
    c = DropKVCache(window_size=16)
    c._prefill_mode = "typo_mode"
    with pytest.raises(ValueError, match="Invalid _prefill_mode"):
        c.update(Q, K, V, layer_idx=0)
    c = DropKVCache()
    c._prefill_mode = "accumulate"
    c.update(Q, K, V, layer_idx=0)
    c._prefill_mode = "bogus"
    with pytest.raises(ValueError, match="Invalid _prefill_mode"):
        c.update(Q[:, :, :1], K[:, :, :1], V[:, :, :1], layer_idx=0)


def test_prefill_chunked_validation():
    c = DropKVCache(keep_ratio=0.3, window_size=8)
    with pytest.raises(TypeError):
        prefill_chunked(object(), torch.zeros(1, 100), object())
    with pytest.raises(ValueError, match="chunk_size.*window_size"):
        prefill_chunked(object(), torch.zeros(1, 100), c, chunk_size=4)
    with pytest.raises(ValueError, match="evict_strategy"):
        prefill_chunked(object(), torch.zeros(1, 100), c, chunk_size=32, evict_strategy="x")
    with pytest.raises(ValueError, match="window_size"):
        prefill_chunked(object(), torch.zeros(1, 100), c, chunk_size=32, evict_strategy="budget",
                        max_kv_tokens=4)
    with pytest.raises(ValueError, match="sequence-shaped"):
        prefill_chunked(object(), torch.zeros(1, 100), c, chunk_size=32,
                        attention_mask=torch.ones(1, 100))
    c.key_cache.append(torch.zeros(1, 8, 10, 128))
    c.value_cache.append(torch.zeros(1, 8, 10, 128))
    with pytest.raises(ValueError, match="fresh.*empty.*cache"):
        prefill_chunked(object(), torch.zeros(1, 100), c)


@pytest.mark.parametrize("strategy", ["last_chunk", "budget"])
def test_prefill_chunked_cleans_up_after_failure(strategy):
    calls = {"n": 0}

    def model(ids, past_key_values=None, use_cache=True):
        calls["n"] += 1
        if calls["n"] > 1:
            raise RuntimeError("simulated failure")
        Q, K, V = _mk(Lq=ids.shape[1], Lk=ids.shape[1])
        past_key_values._prefill_mode = "accumulate"  # stay on the host: no eviction
        for layer in range(2):
            past_key_values.update(Q, K, V, layer_idx=layer)

    c = DropKVCache(keep_ratio=0.3, window_size=8)
    with pytest.raises(RuntimeError, match="simulated failure"):
        prefill_chunked(model, torch.zeros(1, 100), c, chunk_size=32, evict_strategy=strategy,
                        max_kv_tokens=64)
    assert len(c.key_cache) == 0 and len(c.value_cache) == 0 and c._seen_tokens == 0
    assert c._prefill_mode == "single_pass"
    assert c._evict_use_seen_tokens is False and c._budget_max_kv_tokens is None


def test_layer_store_access_and_crop():
    """Layer indexing, iteration and crop of the cache's own store."""
    Q, K, V = _mk(Lq=16, Lk=16)
    c = DropKVCache(keep_ratio=0.5)
    c._prefill_mode = "accumulate"
    c.update(None, K, V, 0)
    c.update(None, K[:, :, :4], V[:, :, :4], 0)
    c.update(None, K, V, 1)
    assert len(c) == 2 and c.get_seq_length() == 20
    k0, v0 = c[0]
    assert torch.equal(k0, torch.cat([K, K[:, :, :4]], dim=2))
    assert [t[0].shape[2] for t in c] == [20, 16]
    with pytest.raises(KeyError):
        c[2]
    c.crop(10)
    assert c.get_seq_length() == 10 and c.key_cache[0].shape[2] == 10 and c.key_cache[1].shape[2] == 10
    c.crop(-4)
    assert c.get_seq_length() == 6 and c.value_cache[0].shape[2] == 6


@pytest.mark.parametrize("storage", ["cat", "buffer"])
def test_buffer_storage_non_evicting_paths_on_cpu(storage):
    """Accumulating prefill and decode appends need no GPU: the row buffers must
    hold exactly what the concatenating storage holds."""
    torch.manual_seed(0)
    K = torch.randn(1, 2, 40, 16)
    V = torch.randn(1, 2, 40, 16)
    c = DropKVCache(keep_ratio=0.5, storage=storage)
    c._prefill_mode = "accumulate"
    for s in range(0, 32, 8):
        c.update(None, K[:, :, s:s + 8], V[:, :, s:s + 8], layer_idx=0)
    c._prefill_mode = "single_pass"
    for t in range(32, 40):
        rk, rv = c.update(None, K[:, :, t:t + 1], V[:, :, t:t + 1], layer_idx=0)
    assert torch.equal(c.key_cache[0], K) and torch.equal(c.value_cache[0], V)
    assert torch.equal(rk, K) and torch.equal(rv, V)
    c.crop(30)
    c.update(None, K[:, :, :1], V[:, :, :1], layer_idx=0)
    assert torch.equal(c.key_cache[0], torch.cat([K[:, :, :30], K[:, :, :1]], dim=2))
    with pytest.raises(ValueError):
        DropKVCache(storage="ring")


def test_phase_table_from_synthetic_trace():
    """The scorer's phase-trace reader: header, layout and per-round medians."""
    import torch
    from dropkv_b200 import diagnostics as dg
    ctas, rounds, nev = 3, 2, 9
    stamps = torch.zeros(ctas, rounds, nev, dtype=torch.int64)
    for c in range(ctas):
        for r in range(rounds):
            base = 1_000_000 + r * 50_000 + c * 100
            stamps[c, r] = base + torch.arange(nev) * (1000 * (c + 1))  # phases of 1, 2, 3 us
    off = 256
    ws = torch.zeros(off + 256 + 8 * (3 + stamps.numel()), dtype=torch.uint8)
    tr = ws[off + 256:].view(torch.int64)
    tr[:3] = torch.tensor([ctas, rounds, nev])
    tr[3:] = stamps.flatten()
    t = dg.read_trace(ws, off)
    rows = dg.phase_table(t)
    assert len(rows) == 2 and set(dg.PHASES) <= set(rows[0])
    assert all(abs(rows[r][p] - 2.0) < 1e-9 for r in range(2) for p in dg.PHASES)  # median of 1, 2, 3
    assert abs(rows[1]["start_us"] - 50.1) < 1e-9
    bad = torch.zeros(1024, dtype=torch.uint8)
    with pytest.raises(ValueError, match="no scorer trace"):
        dg.read_trace(bad, 256)
