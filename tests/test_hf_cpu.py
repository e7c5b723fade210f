"""Transformers integration (dropkv_b200.hf), host side, on CPU.

The CUDA eviction call is replaced by the numpy oracle here (tests are the one
place the oracle may stand in), so these tests check the plumbing the reference
patch adds to Transformers (patches/dropkv_transformers.patch): query states
reach the cache, the first update with them evicts, later updates append, the
logical length drives RoPE positions and the mask sizes follow the stored K/V.
"""

import pytest
import torch

transformers = pytest.importorskip("transformers")

from dropkv_b200 import hf  # noqa: E402
from oracle import dropkv_oracle as O  # noqa: E402


def _oracle_compress(Q, K, V, window, kernel_size, keep_len, **_):
    Qn, Kn, Vn = (t.detach().float().numpy() for t in (Q, K, V))
    s = O.scores_reference(Qn, Kn, Vn, window, round_p=None if Q.dtype == torch.float32 else "bf16")
    idx = O.select_keep_indices(O.pool_and_protect(s, kernel_size, window), keep_len)
    it = torch.from_numpy(idx)
    D = K.shape[-1]
    e = it[..., None].expand(-1, -1, -1, D)
    return it, torch.gather(K, 2, e), torch.gather(V, 2, e)


@pytest.fixture
def oracle_backend(monkeypatch):
    calls = []

    def fake(Q, K, V, window, kernel_size, keep_len, **kw):
        calls.append((tuple(Q.shape), tuple(K.shape), window, kernel_size, keep_len))
        return _oracle_compress(Q, K, V, window, kernel_size, keep_len)

    monkeypatch.setattr(hf.ops, "compress", fake)
    return calls


def _tiny_qwen2(layers=2):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=97, hidden_size=64, intermediate_size=128, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      rope_theta=10000.0, tie_word_embeddings=True)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def test_layer_validation_messages():
    with pytest.raises(ValueError, match="keep_ratio"):
        hf.DropKVLayer(keep_ratio=0.0)
    with pytest.raises(ValueError, match="window_size"):
        hf.DropKVLayer(window_size=0)
    with pytest.raises(ValueError, match="odd"):
        hf.DropKVLayer(kernel_size=4)
    with pytest.raises(ValueError, match="num_layers"):
        hf.DropKVCache()


def test_keep_len_rule():
    lay = hf.DropKVLayer(keep_ratio=0.1, window_size=8)
    assert lay.keep_len(1000) == 100
    assert lay.keep_len(50) == 8          # window floor
    assert hf.DropKVLayer(keep_ratio=1.0).keep_len(37) == 37


def test_first_query_update_evicts_then_appends(oracle_backend):
    lay = hf.DropKVLayer(keep_ratio=0.25, window_size=4, kernel_size=3)
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 4, 40, 16, generator=g)
    k = torch.randn(1, 2, 40, 16, generator=g)
    v = torch.randn(1, 2, 40, 16, generator=g)
    ko, vo = lay.update(k, v, {"query_states": q})
    assert ko is k and vo is v                      # full K/V for this step's attention
    assert lay.keys.shape == (1, 2, 10, 16)         # int(0.25 * 40)
    assert lay.get_seq_length() == 40               # logical length
    assert lay.get_mask_sizes(1) == (11, 0)         # stored + new token
    assert lay.get_mask_sizes(torch.arange(3)) == (13, 0)
    _, ek, _ = _oracle_compress(q, k, v, 4, 3, 10)
    assert torch.equal(lay.keys, ek)
    k1, v1 = torch.randn(1, 2, 1, 16), torch.randn(1, 2, 1, 16)
    ko, vo = lay.update(k1, v1, {"query_states": torch.randn(1, 4, 1, 16)})
    assert ko.shape[2] == 11 and torch.equal(ko[:, :, -1:], k1)
    assert lay.get_seq_length() == 41
    assert len(oracle_backend) == 1                 # a late query does not evict again


def test_short_prefill_and_missing_query(oracle_backend, caplog):
    lay = hf.DropKVLayer(window_size=8)
    k = torch.randn(1, 2, 5, 16)
    lay.update(k, k, {"query_states": torch.randn(1, 4, 5, 16)})
    assert lay.keys.shape[2] == 5 and not oracle_backend
    lay2 = hf.DropKVLayer()
    with caplog.at_level("WARNING"):
        lay2.update(k, k, None)
    assert "query_states" in caplog.text
    assert lay2.keys.shape[2] == 5


def test_head_mismatch_raises(oracle_backend):
    lay = hf.DropKVLayer(window_size=4)
    k = torch.randn(1, 3, 20, 16)
    with pytest.raises(ValueError, match="divisible"):
        lay.update(k, k, {"query_states": torch.randn(1, 4, 20, 16)})


def test_crop_and_reset(oracle_backend):
    lay = hf.DropKVLayer(keep_ratio=0.5, window_size=4)
    q, k = torch.randn(1, 4, 32, 16), torch.randn(1, 2, 32, 16)
    lay.update(k, k, {"query_states": q})
    lay.crop(10)
    assert lay.keys.shape[2] == 10 and lay.get_seq_length() == 10
    lay.reset()
    assert lay.keys.numel() == 0 and not lay._prefilled


def test_model_prefill_and_decode_through_cache(oracle_backend):
    model = _tiny_qwen2(layers=2)
    assert hf.enable_query_states(model) == 2
    cache = hf.DropKVCache(model.config, keep_ratio=0.25, window_size=4, kernel_size=3)
    ids = torch.randint(0, 97, (1, 48), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        out = model(input_ids=ids, past_key_values=cache, use_cache=True)
        assert len(oracle_backend) == 2
        assert [c[4] for c in oracle_backend] == [12, 12]
        assert all(lay.keys.shape[2] == 12 for lay in cache.layers)
        assert cache.get_seq_length() == 48
        tok = out.logits[:, -1:].argmax(-1)
        out2 = model(input_ids=tok, past_key_values=cache, use_cache=True)
    assert all(lay.keys.shape[2] == 13 for lay in cache.layers)
    assert cache.get_seq_length() == 49
    assert torch.isfinite(out2.logits).all()
    # the prefill step attends over the full K/V: same logits as without eviction
    with torch.no_grad():
        ref = model(input_ids=ids, use_cache=False)
    torch.testing.assert_close(out.logits, ref.logits, rtol=1e-5, atol=1e-5)


def _capture_qkv(model, ids):
    seen = {}

    class Grab(hf.DropKVCache):
        def update(self, k, v, layer_idx, cache_kwargs=None):
            seen["qkv"] = (cache_kwargs["query_states"], k, v)
            return k, v

    with torch.no_grad():
        model(input_ids=ids, past_key_values=Grab(model.config), use_cache=True)
    return seen["qkv"]


def test_decode_rope_positions_follow_logical_length(oracle_backend):
    """A decode token after eviction gets position 48 (not 12): its logits match
    a cache without eviction holding the same 12 rows, fed position 48."""
    model = _tiny_qwen2(layers=1)
    hf.enable_query_states(model)
    cache = hf.DropKVCache(model.config, keep_ratio=0.25, window_size=4, kernel_size=3)
    ids = torch.randint(0, 97, (1, 48), generator=torch.Generator().manual_seed(4))
    nxt = torch.tensor([[5]])
    with torch.no_grad():
        model(input_ids=ids, past_key_values=cache, use_cache=True)
        got = model(input_ids=nxt, past_key_values=cache, use_cache=True).logits
        full = transformers.DynamicCache(config=model.config)
        model(input_ids=ids, past_key_values=full, use_cache=True)
        idx = _oracle_compress(*_capture_qkv(model, ids), 4, 3, 12)[0]
        lay = full.layers[0]
        e = idx[..., None].expand(-1, -1, -1, lay.keys.shape[-1])
        lay.keys = torch.gather(lay.keys, 2, e)
        lay.values = torch.gather(lay.values, 2, e)
        want = model(input_ids=nxt, past_key_values=full, position_ids=torch.tensor([[48]]), use_cache=True).logits
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def test_make_cache_parses_generation_strings():
    from transformers import Qwen2Config
    cfg = Qwen2Config(num_hidden_layers=3, hidden_size=64, num_attention_heads=4, num_key_value_heads=2)
    c = hf.make_cache(cfg, backend="DropKV", keep_ratio="0.2", window_size="16", kernel_size="5", use_triton="false")
    assert len(c.layers) == 3
    lay = c.layers[0]
    assert (lay.keep_ratio, lay.window_size, lay.kernel_size, lay.use_triton) == (0.2, 16, 5, False)
    with pytest.raises(ValueError, match="backend"):
        hf.make_cache(cfg, backend="quanto")


def test_generate_wiring(oracle_backend):
    model = _tiny_qwen2(layers=2)
    ids = torch.randint(0, 97, (1, 40), generator=torch.Generator().manual_seed(5))
    out = hf.generate(model, ids, backend="DropKV", keep_ratio="0.25", window_size="4", kernel_size="3",
                      max_new_tokens=5, min_new_tokens=5, do_sample=False, pad_token_id=0)
    assert out.shape == (1, 45)
    assert len(oracle_backend) == 2


def test_attention_falls_back_to_sdpa_on_cpu():
    q = torch.randn(1, 4, 3, 16)
    k = torch.randn(1, 2, 9, 16)

    class M(torch.nn.Module):
        num_key_value_groups = 2
        is_causal = True

    out, _ = hf.dropkv_attention_forward(M(), q, k, k, None, scaling=0.25)
    assert out.shape == (1, 3, 4, 16)
