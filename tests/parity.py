"""Comparison helpers shared by the parity tests (test infrastructure)."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from dropkv_b200.workloads import Workload  # noqa: E402

# A position whose softmax probability reaches this value in some window row is
# ill-conditioned in the reference score (w = (p/(1-p+eps))^2 >= 1e4 multiplies a
# cancelled ||v - y||^2); its score is compared only for finiteness.
ILL_P = 0.99

DTYPE_NAME = {torch.float32: "fp32", torch.bfloat16: "bf16", torch.float16: "fp16"}


def workload_from_json(s: str) -> Workload:
    d = json.loads(s)
    d["dtype"] = getattr(torch, d["dtype"])
    return Workload(**d)


def golden_cases():
    names = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))
    return names


def load_golden(name: str):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return z, workload_from_json(str(z["workload"]))


def input_digest(Q, K, V) -> str:
    import hashlib
    h = hashlib.sha256()
    for t in (Q, K, V):
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def well_conditioned(pmax: np.ndarray) -> np.ndarray:
    return pmax < ILL_P


def assert_scores_close(got: np.ndarray, want: np.ndarray, rtol: float, atol: float,
                        mask: np.ndarray | None = None, what: str = "scores"):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    if mask is None:
        mask = np.ones(got.shape, dtype=bool)
    diff = np.abs(got - want)
    bad = (diff > atol + rtol * np.abs(want)) & mask
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {int(mask.sum())} positions outside rtol={rtol} atol={atol}; "
            f"first at {tuple(int(x) for x in i)}: got {got[tuple(i)]!r} want {want[tuple(i)]!r}")


def keep_set_mismatch(idx_a: np.ndarray, idx_b: np.ndarray, pooled: np.ndarray,
                      allowed: np.ndarray | None = None, rel_band: float = 0.0):
    """Indices where two kept sets differ for a reason other than a tie.

    A difference is excused when its pooled value equals the row's keep threshold
    (an exact tie; ``rel_band`` widens this to a relative band for comparisons of
    scores computed with different rounding) or when ``allowed`` marks it (an
    ill-conditioned neighbourhood).  Each allowed difference may displace one
    element at the boundary, so values between the (k - n)-th and (k + n)-th
    largest pooled values are excused too, n being the allowed differences.
    Returns a list of (row, index) pairs that are not excused.
    """
    idx_a = np.asarray(idx_a)
    idx_b = np.asarray(idx_b)
    pooled = np.asarray(pooled, dtype=np.float32)
    k = idx_a.shape[-1]
    assert idx_b.shape == idx_a.shape
    bad = []
    for row in np.ndindex(idx_a.shape[:-1]):
        sa, sb = set(idx_a[row].tolist()), set(idx_b[row].tolist())
        d = sa ^ sb
        if not d:
            continue
        p = pooled[row]
        srt = np.sort(p)[::-1]
        thr = srt[k - 1]
        n_allowed = 0 if allowed is None else sum(1 for j in d if allowed[row][j])
        hi = srt[max(0, k - 1 - n_allowed)]
        lo = srt[min(len(srt) - 1, k - 1 + n_allowed)]
        for j in d:
            if allowed is not None and allowed[row][j]:
                continue
            if p[j] == thr:
                continue
            if n_allowed and lo <= p[j] <= hi:
                continue
            if rel_band > 0 and abs(float(p[j]) - float(thr)) <= rel_band * max(abs(float(thr)), 1e-30):
                continue
            bad.append((row, j))
    return bad


def dilate(mask: np.ndarray, r: int) -> np.ndarray:
    """Widen a boolean [.., L] mask by r positions each side (max-pool reach)."""
    out = mask.copy()
    L = mask.shape[-1]
    for s in range(1, r + 1):
        out[..., s:] |= mask[..., :L - s]
        out[..., :L - s] |= mask[..., s:]
    return out


def kept_set_report(idx_got: np.ndarray, idx_ref: np.ndarray, pooled_ref: np.ndarray,
                    saturated: np.ndarray, radius: int, rel_band: float) -> dict:
    """Classify every position in which two kept sets differ, row by row.

    ``pooled_ref`` is the reference side's pooled score row, ``saturated`` marks
    positions whose softmax probability reaches ILL_P in some window row (their
    score is fp32 cancellation noise in the reference formula), ``radius`` the
    pooling half-width.  Classes, in order of precedence:

    * ``saturated_nbhd`` -- within ``radius`` of a saturated position (its pooled
      value carries the noise);
    * ``exact_tie``      -- pooled value equal to the row's keep threshold;
    * ``displaced``      -- between the (k-n)-th and (k+n)-th largest pooled
      values, n being the row's saturated-neighbourhood differences (each of those
      moves the keep boundary by one);
    * ``near_tie``       -- within ``rel_band`` (relative) of the threshold;
    * ``unexplained``    -- anything else, listed as (row, index, value, threshold).
    """
    k = idx_ref.shape[-1]
    near = dilate(saturated, radius)
    rep = {"rows": 0, "kept": 0, "diff": 0, "saturated_positions": int(saturated.sum()),
           "saturated_nbhd": 0, "exact_tie": 0, "displaced": 0, "near_tie": 0, "unexplained": []}
    for row in np.ndindex(idx_ref.shape[:-1]):
        d = set(np.asarray(idx_got[row]).tolist()) ^ set(np.asarray(idx_ref[row]).tolist())
        rep["rows"] += 1
        rep["kept"] += k
        rep["diff"] += len(d)
        if not d:
            continue
        p = pooled_ref[row]
        srt = np.sort(p)[::-1]
        thr = srt[k - 1]
        n_sat = sum(1 for j in d if near[row][j])
        hi = srt[max(0, k - 1 - n_sat)]
        lo = srt[min(len(srt) - 1, k - 1 + n_sat)]
        for j in d:
            if near[row][j]:
                rep["saturated_nbhd"] += 1
            elif p[j] == thr:
                rep["exact_tie"] += 1
            elif n_sat and lo <= p[j] <= hi:
                rep["displaced"] += 1
            elif abs(float(p[j]) - float(thr)) <= rel_band * abs(float(thr)):
                rep["near_tie"] += 1
            else:
                rep["unexplained"].append((row, int(j), float(p[j]), float(thr)))
    return rep


def assert_kept_report(rep: dict, radius: int, what: str, near_tie_frac: float = 2e-3):
    """No unexplained difference; the excused ones bounded: a saturated position
    flips at most its pooling neighbourhood in each set (2 (2 radius + 1)) and
    displaces as many boundary positions; near-ties at most ``near_tie_frac`` of
    the kept positions plus 4 per row."""
    assert not rep["unexplained"], f"{what}: kept sets differ beyond the excused classes: {rep['unexplained'][:6]}"
    cap = 2 * (2 * radius + 1) * rep["saturated_positions"]
    assert rep["saturated_nbhd"] <= cap, f"{what}: {rep['saturated_nbhd']} saturated-neighbourhood differences > {cap}"
    assert rep["displaced"] <= cap, f"{what}: {rep['displaced']} displaced boundary positions > {cap}"
    ncap = near_tie_frac * rep["kept"] + 4 * rep["rows"]
    assert rep["near_tie"] <= ncap, f"{what}: {rep['near_tie']} near-tie differences > {ncap:.0f}"
