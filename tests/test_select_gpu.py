"""Selection (pool + protect + top-k + sort) and gather: bit-exact against the oracle.

Given identical scores, the kept index sets must be identical (ties resolve to
the lower index on both sides) and the gathered rows bit-identical.
"""

import numpy as np
import pytest
import torch

from dropkv_b200 import ops
from oracle import dropkv_oracle as O

pytestmark = pytest.mark.gpu


def _check(scores: torch.Tensor, kernel_size: int, protect: int, keep_len: int):
    got = ops.select_keep_indices(scores.cuda(), kernel_size, protect, keep_len).cpu().numpy()
    pooled = O.pool_and_protect(scores.numpy(), kernel_size, protect)
    want = O.select_keep_indices(pooled, keep_len)
    np.testing.assert_array_equal(got, want)
    return got


@pytest.mark.parametrize("Lk", [1, 7, 8, 100, 4095, 4096, 4097, 12345, 32768])
@pytest.mark.parametrize("keep_frac", [0.0, 0.1, 0.5, 1.0])
def test_select_matches_oracle_random(Lk, keep_frac):
    g = torch.Generator().manual_seed(Lk)
    s = torch.randn(2, 3, Lk, generator=g)
    kl = max(1, min(Lk, int(keep_frac * Lk)))
    _check(s, 11, 8, kl)


@pytest.mark.parametrize("kernel_size", [1, 3, 11, 31])
def test_select_kernel_sizes(kernel_size):
    g = torch.Generator().manual_seed(kernel_size)
    s = torch.rand(1, 4, 3000, generator=g)
    _check(s, kernel_size, 8, 300)


def test_select_heavy_ties():
    # quantised scores: large plateaus, many exact ties at the threshold
    g = torch.Generator().manual_seed(0)
    s = torch.randint(0, 5, (2, 2, 5000), generator=g).float()
    _check(s, 11, 8, 777)
    _check(torch.zeros(1, 2, 1000), 11, 8, 100)       # every value equal
    _check(torch.full((1, 1, 64), -3.0), 1, 0, 10)    # negative constant, no protection


def test_select_negative_and_signed_zero():
    s = torch.tensor([[[-0.0, 0.0, -1.0, 2.0, -5.0, 0.0, -0.0, 3.0, -2.0, 1.0] * 30]])
    _check(s, 1, 0, 50)
    _check(s, 3, 4, 120)


def test_select_protect_absorbed_in_fp32():
    # amax + 1 == amax in fp32: protected positions tie with the maximum
    s = torch.rand(1, 2, 2000)
    s[0, 0, 100] = 1e12
    s[0, 1, 1500] = 3e9
    _check(s, 11, 8, 16)
    _check(s, 11, 8, 9)
    _check(s, 11, 64, 30)


def test_select_protect_longer_than_row():
    s = torch.randn(1, 2, 10)
    _check(s, 11, 32, 5)


def test_select_large_row():
    g = torch.Generator().manual_seed(3)
    s = torch.randn(1, 8, 131072, generator=g)
    got = _check(s, 11, 8, 13107)
    assert (np.diff(got, axis=-1) > 0).all()


@pytest.mark.parametrize("shape", [(1, 1, 131072), (1, 20, 40000), (4, 8, 8192), (2, 16, 65536)])
def test_select_row_counts(shape):
    # the launch picks the cluster size from the row count and the resident
    # clusters; every choice must give the same kept set
    g = torch.Generator().manual_seed(shape[1])
    s = torch.rand(*shape, generator=g) ** 4  # crowded exponents, as pooled scores are
    _check(s, 11, 8, shape[-1] // 7)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_gather_bit_exact(dtype, D):
    g = torch.Generator().manual_seed(D)
    K = torch.randn(2, 3, 777, D, generator=g).to(dtype)
    V = torch.randn(2, 3, 777, D, generator=g).to(dtype)
    idx = torch.sort(torch.stack([torch.randperm(777, generator=g)[:100] for _ in range(6)]).view(2, 3, 100), dim=-1).values
    kc, vc = ops.gather_compressed(K.cuda(), V.cuda(), idx.cuda())
    ek = torch.gather(K, 2, idx[..., None].expand(-1, -1, -1, D))
    ev = torch.gather(V, 2, idx[..., None].expand(-1, -1, -1, D))
    iv = torch.int32 if dtype == torch.float32 else torch.int16
    assert torch.equal(kc.cpu().view(iv), ek.view(iv))
    assert torch.equal(vc.cpu().view(iv), ev.view(iv))


def test_gather_unaligned_views():
    """Contiguous K/V starting 2 bytes past an allocation: only 2-byte alignment."""
    K = torch.randn(1, 2, 64, 64, dtype=torch.bfloat16)
    V = torch.randn(1, 2, 64, 64, dtype=torch.bfloat16)
    kb = torch.empty(K.numel() + 1, dtype=torch.bfloat16, device="cuda")
    vb = torch.empty(V.numel() + 1, dtype=torch.bfloat16, device="cuda")
    Kd = kb[1:].view(K.shape)
    Vd = vb[1:].view(V.shape)
    Kd.copy_(K)
    Vd.copy_(V)
    assert Kd.is_contiguous() and Kd.data_ptr() % 16 != 0
    idx = torch.tensor([[[0, 5, 63], [1, 2, 3]]])
    kc, vc = ops.gather_compressed(Kd, Vd, idx.cuda())
    assert torch.equal(kc.cpu(), torch.gather(K, 2, idx[..., None].expand(-1, -1, -1, 64)))
    assert torch.equal(vc.cpu(), torch.gather(V, 2, idx[..., None].expand(-1, -1, -1, 64)))
