"""Seeded synthetic inputs for the eviction path.

The reference ships no datasets or golden vectors for this path (its tests draw
unseeded ``torch.randn``, tests/test_dropkv_triton.py:86-91), so every workload
here is generated from a seed with the shapes and value distributions of the
benchmark configurations:

* ``randn``      -- Q, K, V ~ N(0, 1), the distribution of the reference tests.
* ``heavy``      -- config 1: N(0, 1) plus ``n_heavy`` key positions (seeded draw)
                    boosted by ``boost * normalize(mean of the group's query window)``.
* ``llama_sink`` -- config 2: N(0, 1) with ``n_outlier`` seeded outlier channels of
                    K scaled by ``outlier_scale`` and key position 0 replaced by an
                    attention sink ``sink_alpha * normalize(mean query window)``.

Outlier channels are applied to K only.  Scaling the same channels of both Q and K
by 8 gives logits with a standard deviation near 8, so the softmax saturates to
exactly 1.0 in fp32 on ordinary keys; the score's weight (p / (1 - p + eps))^2 then
reaches 1e12 and multiplies a fully cancelled ||v - y||^2, and every
implementation (the reference's own Triton path included) returns rounding noise
there.  With K-only outliers and ``sink_alpha = 64`` the median sink probability
over the window rows is about 0.5 and no ordinary key saturates.

All generation runs on the requested device with a ``torch.Generator`` of that
device, so CPU-generated tensors are bit-reproducible for a given torch build.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

__all__ = [
    "Workload",
    "make_qkv",
    "CONFIG1",
    "CONFIG2",
    "llama_layer",
    "keep_len_rule",
]


@dataclass(frozen=True)
class Workload:
    """Shape and distribution of one eviction problem (one layer)."""

    B: int
    Hq: int
    Hkv: int
    D: int
    Lq: int
    Lk: int
    dtype: torch.dtype = torch.bfloat16
    window_size: int = 8
    kernel_size: int = 11
    keep_ratio: float = 0.1
    dist: str = "randn"
    seed: int = 0
    extra: dict = field(default_factory=dict, compare=False, hash=False)

    @property
    def g(self) -> int:
        return self.Hq // self.Hkv

    @property
    def M(self) -> int:
        return self.g * min(self.window_size, self.Lq)

    @property
    def positions(self) -> int:
        """Units of the metric: (sequence, KV head, key position) triples."""
        return self.B * self.Hkv * self.Lk

    def keep_len(self) -> int:
        return keep_len_rule(self.Lk, self.keep_ratio, self.window_size)

    def algorithmic_bytes(self) -> int:
        """HBM bytes the path must move: K and V read once, the Q window read once,
        K_c, V_c and the int64 keep indices written once."""
        e = torch.empty((), dtype=self.dtype).element_size()
        kl = self.keep_len()
        per_head = self.Lk * 2 * self.D * e + kl * (2 * self.D * e + 8) + self.g * min(self.window_size, self.Lq) * self.D * e
        return self.B * self.Hkv * per_head


def keep_len_rule(seq_len: int, keep_ratio: float, window_size: int,
                  total_tokens: int | None = None, max_keep_len: int | None = None) -> int:
    """keep_len = min(L, max(int(ratio * base), window, 1)), capped by max_keep_len.

    Mirrors dropkv_cache.py:470-473 (host arithmetic in Python floats, then int()).
    """
    base = total_tokens if total_tokens is not None else seq_len
    kl = min(seq_len, max(int(keep_ratio * base), window_size, 1))
    if max_keep_len is not None:
        kl = min(kl, max_keep_len)
    return kl


def _gen(device) -> torch.Generator:
    return torch.Generator(device=device)


def make_qkv(wl: Workload, device="cpu"):
    """Return (Q, K, V) for ``wl``: Q [B,Hq,Lq,D], K/V [B,Hkv,Lk,D], contiguous."""
    device = torch.device(device)
    g = _gen(device)
    g.manual_seed(int(wl.seed))
    B, Hq, Hkv, D, Lq, Lk = wl.B, wl.Hq, wl.Hkv, wl.D, wl.Lq, wl.Lk
    Q = torch.randn(B, Hq, Lq, D, generator=g, device=device, dtype=torch.float32)
    K = torch.randn(B, Hkv, Lk, D, generator=g, device=device, dtype=torch.float32)
    V = torch.randn(B, Hkv, Lk, D, generator=g, device=device, dtype=torch.float32)
    W = min(wl.window_size, Lq)
    grp = Hq // Hkv
    if wl.dist == "randn":
        pass
    elif wl.dist == "heavy":
        n_heavy = int(wl.extra.get("n_heavy", 4))
        boost = float(wl.extra.get("boost", 3.0))
        qbar = Q[:, :, Lq - W:, :].reshape(B, Hkv, grp * W, D).mean(dim=2)  # [B,Hkv,D]
        u = qbar / qbar.norm(dim=-1, keepdim=True)
        pos = torch.randperm(max(Lk - W, 1), generator=g, device=device)[:n_heavy]
        K[:, :, pos, :] += boost * u[:, :, None, :]
    elif wl.dist == "llama_sink":
        n_out = int(wl.extra.get("n_outlier", 2))
        scale = float(wl.extra.get("outlier_scale", 8.0))
        alpha = float(wl.extra.get("sink_alpha", 64.0))
        ch = torch.randperm(D, generator=g, device=device)[:n_out]
        K[..., ch] *= scale
        qbar = Q[:, :, Lq - W:, :].reshape(B, Hkv, grp * W, D).mean(dim=2)
        u = qbar / qbar.norm(dim=-1, keepdim=True)
        K[:, :, 0, :] = alpha * u
    else:
        raise ValueError(f"unknown distribution {wl.dist!r}")
    return (Q.to(wl.dtype).contiguous(), K.to(wl.dtype).contiguous(), V.to(wl.dtype).contiguous())


# CPU reference case.
CONFIG1 = Workload(B=1, Hq=8, Hkv=2, D=64, Lq=64, Lk=1024, dtype=torch.float32,
                   dist="heavy", seed=1, extra={"n_heavy": 4, "boost": 3.0})

# one Llama-3.1-8B-shaped layer at Lk=32768.
CONFIG2 = Workload(B=1, Hq=32, Hkv=8, D=128, Lq=8, Lk=32768, dtype=torch.bfloat16,
                   dist="llama_sink", seed=2,
                   extra={"n_outlier": 2, "outlier_scale": 8.0, "sink_alpha": 64.0})


def llama_layer(Lk: int, keep_ratio: float = 0.1, seed: int = 2, B: int = 1,
                Lq: int = 8) -> Workload:
    """A Llama-3.1-8B attention layer (Hq=32, Hkv=8, D=128, bf16) with the config-2
    value distribution at context ``Lk``."""
    return Workload(B=B, Hq=32, Hkv=8, D=128, Lq=Lq, Lk=Lk, dtype=torch.bfloat16,
                    keep_ratio=keep_ratio, dist="llama_sink", seed=seed,
                    extra={"n_outlier": 2, "outlier_scale": 8.0, "sink_alpha": 64.0})


def inv_sqrt(D: int) -> float:
    return 1.0 / math.sqrt(D)
