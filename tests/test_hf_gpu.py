"""Transformers integration (dropkv_b200.hf) on the GPU: a small random-init
Qwen2 model evicts through the CUDA library at prefill and decodes over the
compressed cache with dropkv_decode_attention."""

import numpy as np
import pytest
import torch

transformers = pytest.importorskip("transformers")

from dropkv_b200 import _lib, hf  # noqa: E402
from oracle import dropkv_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


def _model(head_dim=64, layers=2, attn="sdpa"):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=1000, hidden_size=7 * head_dim, intermediate_size=512, num_hidden_layers=layers,
                      num_attention_heads=7, num_key_value_heads=1, max_position_embeddings=4096,
                      rope_theta=1e6, tie_word_embeddings=True)
    torch.manual_seed(0)
    m = Qwen2ForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    m.config._attn_implementation = attn
    return m


def _capture(model, ids):
    got = {}

    class Grab(hf.DropKVCache):
        def update(self, k, v, layer_idx, cache_kwargs=None):
            got[layer_idx] = (cache_kwargs["query_states"], k, v)
            return k, v

    with torch.no_grad():
        model(input_ids=ids, past_key_values=Grab(model.config), use_cache=True)
    return got


def test_prefill_evicts_like_the_oracle():
    model = _model()
    hf.enable_query_states(model)
    ids = torch.randint(0, 1000, (1, 700), generator=torch.Generator().manual_seed(7)).cuda()
    cache = hf.DropKVCache(model.config, keep_ratio=0.1, window_size=8, kernel_size=11)
    n0 = _lib.launch_count()
    with torch.no_grad():
        model(input_ids=ids, past_key_values=cache, use_cache=True)
    torch.cuda.synchronize()
    assert _lib.launch_count() > n0
    qkv = _capture(model, ids)
    for li, layer in enumerate(cache.layers):
        q, k, v = qkv[li]
        assert layer.keys.shape == (1, 1, 70, 64)
        qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
        s = O.scores_reference(qn, kn, vn, 8, round_p="bf16")
        idx = O.select_keep_indices(O.pool_and_protect(s, 11, 8), 70)
        # the kept rows are rows of K, in order; the kept set matches the oracle's up to near-ties
        rows = layer.keys[0, 0].float().cpu().numpy()
        kk = kn[0, 0]
        pos = [int(np.flatnonzero((kk == r).all(axis=1))[0]) for r in rows]
        assert pos == sorted(pos)
        overlap = len(set(pos) & set(idx[0, 0].tolist())) / 70
        assert overlap >= 0.95, overlap


def test_decode_attention_matches_sdpa_over_the_compressed_cache():
    hf.register_attention("dropkv")
    ids = torch.randint(0, 1000, (1, 600), generator=torch.Generator().manual_seed(8)).cuda()
    logits = {}
    for attn in ("sdpa", "dropkv"):
        model = _model(attn=attn)
        hf.enable_query_states(model)
        cache = hf.DropKVCache(model.config, keep_ratio=0.2, window_size=8, kernel_size=11)
        outs = []
        with torch.no_grad():
            out = model(input_ids=ids, past_key_values=cache, use_cache=True)
            tok = out.logits[:, -1:].argmax(-1)
            for _ in range(4):
                out = model(input_ids=tok, past_key_values=cache, use_cache=True)
                outs.append(out.logits.float())
                tok = out.logits[:, -1:].argmax(-1)
        logits[attn] = torch.cat(outs, 1)
        assert all(lay.keys.shape[2] == 120 + 4 for lay in cache.layers)
    torch.testing.assert_close(logits["dropkv"], logits["sdpa"], rtol=2e-2, atol=2e-2)


def test_generate_wiring():
    model = _model()
    ids = torch.randint(0, 1000, (1, 300), generator=torch.Generator().manual_seed(9)).cuda()
    out = hf.generate(model, ids, backend="DropKV", keep_ratio="0.1", window_size="8", kernel_size="11",
                      max_new_tokens=5, min_new_tokens=5, do_sample=False, pad_token_id=0)
    assert out.shape == (1, 305)
