"""Preallocated row-buffer storage for the chunked prefill (scope row f1).

``dropkv_compress_strided`` must give the same kept rows as ``dropkv_compress`` on
the same data (it reads K/V with a capacity stride and writes into a buffer), and
``DropKVCache(storage="buffer")`` must hold exactly what the reference's
``torch.cat`` storage holds (dropkv_cache.py:581-617) after every prefill strategy
and after decode steps.
"""

import pytest
import torch

from dropkv_b200 import DropKVCache, ops, prefill_chunked
from dropkv_b200.workloads import Workload, make_qkv

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32)


@pytest.mark.parametrize("cfg", [
    dict(Hq=32, Hkv=8, D=128, Lk=1000, dtype=torch.bfloat16),
    dict(Hq=32, Hkv=8, D=128, Lk=32768, dtype=torch.bfloat16),
    dict(Hq=14, Hkv=2, D=64, Lk=4097, dtype=torch.bfloat16),
    dict(Hq=8, Hkv=2, D=128, Lk=777, dtype=torch.float16),
    dict(Hq=8, Hkv=2, D=128, Lk=555, dtype=torch.float32),   # CUDA-core scorer
])
def test_compress_strided_equals_compress(cfg):
    Lk, dtype = cfg.pop("Lk"), cfg.pop("dtype")
    wl = Workload(B=1, Lq=16, Lk=Lk, dtype=dtype, seed=Lk % 97, **cfg)
    Q, K, V = make_qkv(wl, "cuda")
    kl = max(int(0.1 * Lk), 8)
    idx, kc, vc = ops.compress(Q, K, V, 8, 11, kl)
    cap, cap_out = Lk + 256, kl + 64
    Kb = torch.zeros(1, wl.Hkv, cap, wl.D, dtype=dtype, device="cuda")
    Vb = torch.zeros_like(Kb)
    Kb[:, :, :Lk] = K
    Vb[:, :, :Lk] = V
    Ko = torch.full((1, wl.Hkv, cap_out, wl.D), 7.0, dtype=dtype, device="cuda")
    Vo = torch.full_like(Ko, 7.0)
    idx2 = ops.compress_strided(Q, Kb, Vb, Lk, 8, 11, kl, Ko, Vo)
    assert torch.equal(idx, idx2)
    assert torch.equal(_bits(Ko[:, :, :kl]), _bits(kc)) and torch.equal(_bits(Vo[:, :, :kl]), _bits(vc))
    assert bool((Ko[:, :, kl:] == 7.0).all())  # rows past keep_len untouched


class _TinyModel:
    def __init__(self, Q, K, V, layers=2):
        self.Q, self.K, self.V, self.layers = Q, K, V, layers
        self.pos = 0
        self.returned = []

    def __call__(self, ids, past_key_values=None, use_cache=True):
        n = ids.shape[1]
        s = slice(self.pos, self.pos + n)
        for layer in range(self.layers):
            k, v = past_key_values.update(self.Q[:, :, s], self.K[:, :, s], self.V[:, :, s], layer_idx=layer)
            self.returned.append((k.clone(), v.clone()))
        self.pos += n
        return n


@pytest.mark.parametrize("strategy", ["last_chunk", "budget", "every_chunk"])
def test_buffer_storage_equals_cat_storage(strategy):
    wl = Workload(B=1, Hq=32, Hkv=8, D=128, Lq=1000, Lk=1000, seed=21)
    Q, K, V = make_qkv(wl, "cuda")
    caches, models = [], []
    for storage in ("cat", "buffer"):
        cache = DropKVCache(keep_ratio=0.3, storage=storage)
        model = _TinyModel(Q, K, V)
        prefill_chunked(model, torch.zeros(1, 1000), cache, chunk_size=256, evict_strategy=strategy,
                        max_kv_tokens=300)
        # two decode steps on the compressed cache
        for t in range(2):
            d = slice(1000 - 2 + t, 1000 - 1 + t)
            for layer in range(2):
                k, v = cache.update(Q[:, :, d], K[:, :, d], V[:, :, d], layer_idx=layer)
                model.returned.append((k.clone(), v.clone()))
        caches.append(cache)
        models.append(model)
    a, b = caches
    assert a._seen_tokens == b._seen_tokens
    for layer in range(2):
        assert torch.equal(_bits(a.key_cache[layer]), _bits(b.key_cache[layer]))
        assert torch.equal(_bits(a.value_cache[layer]), _bits(b.value_cache[layer]))
    assert len(models[0].returned) == len(models[1].returned)
    for (ka, va), (kb, vb) in zip(models[0].returned, models[1].returned):
        assert torch.equal(_bits(ka), _bits(kb)) and torch.equal(_bits(va), _bits(vb))


def test_buffer_storage_single_pass_and_crop():
    wl = Workload(B=1, Hq=32, Hkv=8, D=128, Lq=512, Lk=512, seed=22)
    Q, K, V = make_qkv(wl, "cuda")
    out = []
    for storage in ("cat", "buffer"):
        c = DropKVCache(keep_ratio=0.2, storage=storage)
        c.update(Q, K, V, layer_idx=0)
        for t in range(3):
            c.update(Q[:, :, t:t + 1], K[:, :, t:t + 1], V[:, :, t:t + 1], layer_idx=0)
        c.crop(50)
        c.update(Q[:, :, :1], K[:, :, :1], V[:, :, :1], layer_idx=0)
        out.append((c.key_cache[0].clone(), c.value_cache[0].clone()))
    assert torch.equal(_bits(out[0][0]), _bits(out[1][0])) and torch.equal(_bits(out[0][1]), _bits(out[1][1]))
