"""Decode attention over the (compressed) cache: ``dropkv_decode_attention``.

Checked against a plain PyTorch fp32 reference of the same op (softmax(scale
Q K^T) V per KV-head group, the query rows tail-aligned to the keys), on
contiguous caches and on the row-buffer views ``DropKVCache(storage="buffer")``
hands out. Tolerance: inputs in bf16/fp16, fp32 accumulation, output rounded to
the input dtype -> rtol 2e-2 / atol 2e-3 on outputs of magnitude ~1.
"""

import pytest
import torch

from dropkv_b200 import DropKVCache, ops

pytestmark = pytest.mark.gpu


def _reference(Q, K, V, scale):
    B, Hq, Lq, D = Q.shape
    Hkv, L = K.shape[1], K.shape[2]
    g = Hq // Hkv
    q = Q.float()
    k = K.float().repeat_interleave(g, dim=1)
    v = V.float().repeat_interleave(g, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) * scale
    qpos = torch.arange(Lq, device=Q.device)[:, None]
    kpos = torch.arange(L, device=Q.device)[None, :]
    s = s.masked_fill(kpos > (L - Lq + qpos), float("-inf"))
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, dim=-1), v)


@pytest.mark.parametrize("B,Hq,Hkv,Lq,L,D", [
    (1, 32, 8, 1, 13107, 128),    # Llama-3.1-8B layer, 128K compressed to 10 %
    (2, 32, 8, 1, 4096, 128),
    (1, 14, 2, 1, 819, 64),       # Qwen2-0.5B shapes (g = 7)
    (1, 8, 8, 1, 100, 128),       # MHA
    (3, 16, 2, 1, 5000, 64),      # g = 8
    (1, 32, 8, 2, 3000, 128),     # two query rows: 8 rows per group
    (1, 16, 2, 4, 777, 128),      # 32 rows per group: four row blocks
    (1, 4, 1, 1, 1, 64),          # a single key
    (1, 32, 8, 1, 131072, 128),   # the uncompressed 128K cache
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_attention_matches_torch(B, Hq, Hkv, Lq, L, D, dtype):
    g = torch.Generator(device="cuda").manual_seed(L + Hq)
    Q = torch.randn(B, Hq, Lq, D, device="cuda", generator=g).to(dtype)
    K = (torch.randn(B, Hkv, L, D, device="cuda", generator=g) * 2).to(dtype)
    V = torch.randn(B, Hkv, L, D, device="cuda", generator=g).to(dtype)
    scale = D ** -0.5
    got = ops.decode_attention(Q, K, V)
    want = _reference(Q, K, V, scale)
    torch.testing.assert_close(got.float(), want, rtol=2e-2, atol=2e-3)
    again = ops.decode_attention(Q, K, V)  # the workspace is reused: counters reset
    assert torch.equal(got, again)


def test_decode_attention_strided_buffers_and_scale():
    # rows inside a larger buffer, as the row-buffer cache hands them out
    B, Hq, Hkv, L, cap, D = 2, 32, 8, 3000, 4096, 128
    g = torch.Generator(device="cuda").manual_seed(7)
    Kb = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).bfloat16()
    Vb = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).bfloat16()
    Q = torch.randn(B, Hq, 1, D, device="cuda", generator=g).bfloat16()
    got = ops.decode_attention(Q, Kb[:, :, :L], Vb[:, :, :L], scale=0.05)
    want = _reference(Q, Kb[:, :, :L], Vb[:, :, :L], 0.05)
    torch.testing.assert_close(got.float(), want, rtol=2e-2, atol=2e-3)


def test_decode_over_compressed_buffer_cache():
    # prefill 2048 tokens, evict to 30 %, then decode steps attending over the cache
    B, Hq, Hkv, D, L0 = 1, 32, 8, 128, 2048
    g = torch.Generator(device="cuda").manual_seed(11)
    Q = torch.randn(B, Hq, L0 + 4, D, device="cuda", generator=g).bfloat16()
    K = torch.randn(B, Hkv, L0 + 4, D, device="cuda", generator=g).bfloat16()
    V = torch.randn(B, Hkv, L0 + 4, D, device="cuda", generator=g).bfloat16()
    cache = DropKVCache(keep_ratio=0.3, storage="buffer")
    cache.update(Q[:, :, :L0], K[:, :, :L0], V[:, :, :L0], layer_idx=0)
    for t in range(4):
        s = slice(L0 + t, L0 + t + 1)
        k, v = cache.update(Q[:, :, s], K[:, :, s], V[:, :, s], layer_idx=0)
        got = ops.decode_attention(Q[:, :, s], k, v)
        torch.testing.assert_close(got.float(), _reference(Q[:, :, s], k, v, D ** -0.5), rtol=2e-2, atol=2e-3)


def test_decode_attention_rejects_bad_input():
    Q = torch.randn(1, 6, 1, 128, device="cuda").bfloat16()
    K = torch.randn(1, 4, 10, 128, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        ops.decode_attention(Q, K, K)          # 6 query heads over 4 KV heads
    with pytest.raises(TypeError):
        ops.decode_attention(Q.float(), K.float(), K.float())


def _split(Q, K_new, V_new, K_buf, V_buf, pos, scale=None):
    n = K_new.shape[2]
    K_buf[:, :, pos:pos + n] = K_new
    V_buf[:, :, pos:pos + n] = V_new
    return ops.decode_attention(Q, K_buf[:, :, :pos + n], V_buf[:, :, :pos + n], scale=scale)


@pytest.mark.parametrize("B,Hq,Hkv,Lq,n,pos,cap,D", [
    (1, 32, 8, 1, 1, 13107, 13200, 128),   # the Llama decode step over the compressed cache
    (2, 32, 8, 1, 1, 3000, 4096, 128),
    (1, 14, 2, 1, 1, 818, 900, 64),        # Qwen2-0.5B shapes
    (1, 16, 2, 4, 4, 777, 800, 128),       # four new rows (speculative / multi-token step)
    (1, 8, 8, 2, 3, 0, 16, 128),           # empty cache: every key is new
    (3, 16, 2, 1, 2, 4998, 5000, 64),      # rows up to the buffer's end
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_append_attention_equals_append_then_attend(B, Hq, Hkv, Lq, n, pos, cap, D, dtype):
    g = torch.Generator(device="cuda").manual_seed(pos + n + Hq)
    Q = torch.randn(B, Hq, Lq, D, device="cuda", generator=g).to(dtype)
    K_buf = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).to(dtype)
    V_buf = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).to(dtype)
    K_new = (torch.randn(B, Hkv, n, D, device="cuda", generator=g) * 2).to(dtype)
    V_new = torch.randn(B, Hkv, n, D, device="cuda", generator=g).to(dtype)
    K2, V2 = K_buf.clone(), V_buf.clone()
    want = _split(Q, K_new, V_new, K2, V2, pos)
    got = ops.decode_append_attention(Q, K_new, V_new, K_buf, V_buf, pos)
    torch.cuda.synchronize()
    assert torch.equal(got, want)                 # bit-identical to the two-call path
    assert torch.equal(K_buf, K2) and torch.equal(V_buf, V2)   # rows stored, nothing else touched
    ref = _reference(Q, K_buf[:, :, :pos + n], V_buf[:, :, :pos + n], D ** -0.5)
    torch.testing.assert_close(got.float(), ref, rtol=2e-2, atol=2e-3)


def test_decode_append_attention_from_projection_view():
    # the token's K/V straight from a [B, 1, Hkv, D] projection (transposed view)
    B, Hq, Hkv, D, pos, cap = 2, 32, 8, 128, 2000, 2048
    g = torch.Generator(device="cuda").manual_seed(5)
    Q = torch.randn(B, 1, Hq, D, device="cuda", generator=g).bfloat16().transpose(1, 2)
    proj_k = torch.randn(B, 1, Hkv, D, device="cuda", generator=g).bfloat16()
    proj_v = torch.randn(B, 1, Hkv, D, device="cuda", generator=g).bfloat16()
    K_buf = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).bfloat16()
    V_buf = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).bfloat16()
    K2, V2 = K_buf.clone(), V_buf.clone()
    kn, vn = proj_k.transpose(1, 2), proj_v.transpose(1, 2)
    want = _split(Q, kn, vn, K2, V2, pos, scale=0.07)
    got = ops.decode_append_attention(Q, kn, vn, K_buf, V_buf, pos, scale=0.07)
    assert torch.equal(got, want)
    assert torch.equal(K_buf, K2) and torch.equal(V_buf, V2)


def test_decode_append_attention_rejects_bad_input():
    Q = torch.randn(1, 8, 1, 128, device="cuda").bfloat16()
    kb = torch.zeros(1, 4, 16, 128, device="cuda").bfloat16()
    kn = torch.zeros(1, 4, 1, 128, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        ops.decode_append_attention(Q, kn, kn, kb, kb, 16)    # no room for the row
    with pytest.raises(ValueError):
        ops.decode_append_attention(Q, kn, kn, kb, kb, -1)
    with pytest.raises(TypeError):
        ops.decode_append_attention(Q, kn.half(), kn.half(), kb, kb, 3)
