"""CPU oracle for the DropKV prefill eviction path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and its
``--impl reference`` arm) may import it.  The product path (``dropkv_b200``)
never calls it and fails loudly when its CUDA library is missing.

It restates, in numpy float32, the reference's algorithm for the path:

* ``scores_reference``   -- dropkv_triton.py:29-109 (``dropkv_scores_reference``):
  per KV head, the last W query rows of its GQA group, logits Q K^T / sqrt(D) with
  the tail-aligned causal mask (dropkv_triton.py:81-85), fp32 softmax, optional
  rounding of p to the input dtype (dropkv_triton.py:88-92), y = p V, weight
  W = (p / (1 - p + eps))^2, and the score sum_m W * ||v - y_m||^2 expanded as
  termA - termB + termC (dropkv_triton.py:94-106, dropkv_cache.py:436-460),
  averaged over the group (dropkv_triton.py:108).
* ``select_keep_indices`` -- dropkv_cache.py:462-477: max_pool1d(kernel_size,
  padding kernel_size//2, stride 1), protection of the last ``window_size``
  positions with amax + 1, top-k, ascending sort.  ``torch.topk`` leaves the order
  of tied values unspecified; this oracle breaks ties by the lower index, the rule
  the CUDA kernels implement, so kept sets agree exactly given identical scores.
* ``gather_compressed``  -- dropkv_cache.py:479-491.
* ``keep_len``           -- dropkv_cache.py:470-473.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own functions on
seeded inputs and stores their outputs; ``tests/test_oracle_golden.py`` checks this
restatement against those fixtures.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "round_to_bf16",
    "round_to_fp16",
    "scores_reference",
    "pool_and_protect",
    "ordered_keys",
    "select_keep_indices",
    "gather_compressed",
    "keep_len",
    "compress",
]


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even) and widen back."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    # NaN stays NaN (quiet)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.float32("nan")
    return out


def round_to_fp16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def _round_p(p: np.ndarray, round_p: str | None) -> np.ndarray:
    if round_p is None or round_p == "fp32":
        return p
    if round_p == "bf16":
        return round_to_bf16(p)
    if round_p == "fp16":
        return round_to_fp16(p)
    raise ValueError(f"round_p must be None, 'fp32', 'bf16' or 'fp16', got {round_p!r}")


def scores_reference(Q, K, V, window_size: int = 8, eps: float = 1e-6,
                     round_p: str | None = None) -> np.ndarray:
    """DropKV eviction scores, float32 [B, Hkv, Lk].

    Q [B,Hq,Lq,D], K/V [B,Hkv,Lk,D] (any float dtype; computed in float32).
    Q is tail-aligned with K: query row Lq-1 sits at key position Lk-1.
    Follows dropkv_triton.py:57-109 with the GQA group vectorised over its
    g*W rows (the formulation of dropkv_cache.py:411-460).
    """
    Q = np.asarray(Q, dtype=np.float32)
    K = np.asarray(K, dtype=np.float32)
    V = np.asarray(V, dtype=np.float32)
    B, Hq, Lq, D = Q.shape
    Hkv, Lk = K.shape[1], K.shape[2]
    W = int(window_size)
    assert Lq >= W, f"Lq ({Lq}) must be >= window_size ({W})"
    assert Lk >= W, f"Lk ({Lk}) must be >= window_size ({W})"
    assert Lq <= Lk, f"Lq ({Lq}) must be <= Lk ({Lk}) (Q must be tail-aligned suffix)"
    assert Hq % Hkv == 0, f"Hq ({Hq}) must be divisible by Hkv ({Hkv})"
    g = Hq // Hkv
    M = g * W
    scale = np.float32(math.sqrt(D))
    eps32 = np.float32(eps)
    # Row m = gi*W + w may attend keys j <= Lk - W + w (dropkv_triton.py:81-85).
    w_of_m = np.arange(M) % W
    masked = np.arange(Lk)[None, :] > (Lk - W + w_of_m)[:, None]
    out = np.zeros((B, Hkv, Lk), dtype=np.float32)
    for b in range(B):
        for h in range(Hkv):
            Qw = Q[b, h * g:(h + 1) * g, Lq - W:, :].reshape(M, D)
            Kh = K[b, h]
            Vh = V[b, h]
            logits = (Qw @ Kh.T) / scale
            logits[masked] = -np.inf
            mx = logits.max(axis=1, keepdims=True)
            e = np.exp(logits - mx)
            p = e / e.sum(axis=1, keepdims=True)
            p = _round_p(p, round_p)
            y = p @ Vh                                     # [M, D]
            Wm = (p / (np.float32(1.0) - p + eps32)) ** 2  # [M, Lk]
            termA = Wm.sum(axis=0) * (Vh * Vh).sum(axis=1)
            termB = np.float32(2.0) * (Vh * (Wm.T @ y)).sum(axis=1)
            termC = Wm.T @ (y * y).sum(axis=1)
            out[b, h] = termA - termB + termC
    out /= np.float32(g)
    return out


def scores_cache_path(Q, K, V, window_size: int = 8, eps: float = 1e-6,
                      dtype: str = "bf16") -> np.ndarray:
    """Scores of the reference's PyTorch eviction path, dropkv_cache.py:401-460.

    Differs from ``scores_reference`` only in precision: p is rounded to the input
    dtype (dropkv_cache.py:431) and y = p V is produced in the input dtype
    (dropkv_cache.py:434; float32 accumulation, one rounding of each element).
    ``window_size`` is already min(window, Lq) (dropkv_cache.py:407).
    """
    Q = np.asarray(Q, dtype=np.float32)
    K = np.asarray(K, dtype=np.float32)
    V = np.asarray(V, dtype=np.float32)
    B, Hq, Lq, D = Q.shape
    Hkv, Lk = K.shape[1], K.shape[2]
    W = int(window_size)
    g = Hq // Hkv
    M = g * W
    rnd = {"bf16": round_to_bf16, "fp16": round_to_fp16, "fp32": lambda a: a}[dtype]
    scale = np.float32(math.sqrt(D))
    eps32 = np.float32(eps)
    w_of_m = np.arange(M) % W
    masked = np.arange(Lk)[None, :] > (Lk - W + w_of_m)[:, None]
    out = np.zeros((B, Hkv, Lk), dtype=np.float32)
    for b in range(B):
        for h in range(Hkv):
            Qw = Q[b, h * g:(h + 1) * g, Lq - W:, :].reshape(M, D)
            Kh, Vh = K[b, h], V[b, h]
            logits = (Qw @ Kh.T) / scale
            logits[masked] = -np.inf
            mx = logits.max(axis=1, keepdims=True)
            e = np.exp(logits - mx)
            p = rnd(e / e.sum(axis=1, keepdims=True))
            y = rnd(p @ Vh)
            Wm = (p / (np.float32(1.0) - p + eps32)) ** 2
            termA = Wm.sum(axis=0) * (Vh * Vh).sum(axis=1)
            termB = np.float32(2.0) * ((Wm.T * (Vh @ y.T)).sum(axis=1))
            termC = Wm.T @ (y * y).sum(axis=1)
            out[b, h] = (termA - termB + termC) / np.float32(g)
    return out


def max_attention(Q, K, window_size: int = 8) -> np.ndarray:
    """max over the window rows of the fp32 softmax probability, [B, Hkv, Lk].

    Positions where this reaches ~1 are ill-conditioned in the reference's score:
    the weight (p / (1 - p + eps))^2 grows towards 1e12 and multiplies
    ||v - y||^2, which is itself a cancellation when y ~ v.  Parity tests use it to
    separate those positions from the rest.
    """
    Q = np.asarray(Q, dtype=np.float32)
    K = np.asarray(K, dtype=np.float32)
    B, Hq, Lq, D = Q.shape
    Hkv, Lk = K.shape[1], K.shape[2]
    W = int(window_size)
    g = Hq // Hkv
    M = g * W
    masked = np.arange(Lk)[None, :] > (Lk - W + np.arange(M) % W)[:, None]
    out = np.zeros((B, Hkv, Lk), dtype=np.float32)
    for b in range(B):
        for h in range(Hkv):
            Qw = Q[b, h * g:(h + 1) * g, Lq - W:, :].reshape(M, D)
            logits = (Qw @ K[b, h].T) / np.float32(math.sqrt(D))
            logits[masked] = -np.inf
            e = np.exp(logits - logits.max(axis=1, keepdims=True))
            out[b, h] = (e / e.sum(axis=1, keepdims=True)).max(axis=0)
    return out


def pool_and_protect(scores: np.ndarray, kernel_size: int, window_size: int) -> np.ndarray:
    """max_pool1d(k, pad k//2, stride 1) then last ``window_size`` := amax + 1.

    dropkv_cache.py:464-467.  Padding is -inf, so windows are truncated at the
    row ends.
    """
    s = np.asarray(scores, dtype=np.float32)
    r = kernel_size // 2
    L = s.shape[-1]
    pad = np.full(s.shape[:-1] + (L + 2 * r,), -np.inf, dtype=np.float32)
    pad[..., r:r + L] = s
    win = np.lib.stride_tricks.sliding_window_view(pad, kernel_size, axis=-1)
    pooled = win.max(axis=-1).astype(np.float32)
    big = pooled.max(axis=-1, keepdims=True) + np.float32(1.0)
    if window_size > 0:
        pooled[..., -window_size:] = np.broadcast_to(big, pooled[..., -window_size:].shape)
    return pooled


def ordered_keys(x: np.ndarray) -> np.ndarray:
    """Map float32 to uint32 so that unsigned order equals float order (-0 == +0)."""
    x = np.asarray(x, dtype=np.float32) + np.float32(0.0)  # -0.0 -> +0.0
    u = x.view(np.uint32)
    neg = (u & np.uint32(0x80000000)) != 0
    return np.where(neg, ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def select_keep_indices(pooled: np.ndarray, keep_len: int) -> np.ndarray:
    """Top-``keep_len`` positions per row, ties to the lower index, ascending.

    dropkv_cache.py:474-475 (torch.topk then torch.sort).
    """
    keys = ordered_keys(pooled)
    lead = keys.shape[:-1]
    L = keys.shape[-1]
    flat = keys.reshape(-1, L)
    res = np.empty((flat.shape[0], keep_len), dtype=np.int64)
    for i in range(flat.shape[0]):
        order = np.argsort(~flat[i], kind="stable")  # descending key, ascending index
        res[i] = np.sort(order[:keep_len])
    return res.reshape(lead + (keep_len,))


def gather_compressed(K: np.ndarray, V: np.ndarray, keep_idx: np.ndarray):
    """K_c, V_c = K/V rows at ``keep_idx`` along the sequence axis
    (dropkv_cache.py:479-491)."""
    idx = keep_idx[..., None]
    return (np.take_along_axis(K, idx, axis=2), np.take_along_axis(V, idx, axis=2))


def keep_len(seq_len: int, keep_ratio: float, window_size: int,
             total_tokens: int | None = None, max_keep_len: int | None = None) -> int:
    """dropkv_cache.py:470-473."""
    base = total_tokens if total_tokens is not None else seq_len
    kl = min(seq_len, max(int(keep_ratio * base), window_size, 1))
    if max_keep_len is not None:
        kl = min(kl, max_keep_len)
    return kl


def compress(Q, K, V, window_size: int = 8, kernel_size: int = 11, keep_ratio: float = 0.1,
             eps: float = 1e-6, round_p: str | None = None, total_tokens=None, max_keep_len=None):
    """The whole path: scores -> pool/protect -> top-k -> sort -> gather.

    The scoring window is min(window_size, Lq) and protection always covers
    ``window_size`` positions (dropkv_cache.py:407, 466-467).
    """
    Lq, Lk = Q.shape[2], K.shape[2]
    W = min(window_size, Lq)
    s = scores_reference(Q, K, V, W, eps, round_p)
    pooled = pool_and_protect(s, kernel_size, window_size)
    kl = keep_len(Lk, keep_ratio, window_size, total_tokens, max_keep_len)
    idx = select_keep_indices(pooled, kl)
    Kc, Vc = gather_compressed(np.asarray(K), np.asarray(V), idx)
    return s, pooled, idx, Kc, Vc
