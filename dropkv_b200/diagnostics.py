"""Phase trace of the tensor-core scorer.

Every launch of the fused scorer (csrc/scores_tc.cu) has epilogue thread 0 of
each CTA record the globaltimer at the end of each phase of each round into the
workspace: a header of three int64 words (CTAs, rounds, events per round) and
then ``[CTA][round][event]`` nanosecond stamps. The trace sits 256 bytes after
the status word (``dropkv_scores_status_offset``). ``scorer_phases`` runs the
scorer once on a caller-provided problem and returns, per round, the median
over CTAs of each phase's duration.
"""

from __future__ import annotations

import torch

from . import _lib, ops

PHASES = ("logits", "row_max", "pv", "barrier_a", "merge", "barrier_b", "y_stage", "pass2")


def read_trace(ws: torch.Tensor, status_offset: int) -> torch.Tensor:
    """[CTAs, rounds, 9] stamps (ns, float64) from a scorer workspace."""
    tr = ws[status_offset + 256:].view(torch.int64)
    ctas, rounds, nev = (int(x) for x in tr[:3].tolist())
    if nev != len(PHASES) + 1 or ctas <= 0 or rounds <= 0:
        raise ValueError(f"no scorer trace in this workspace (header {ctas}, {rounds}, {nev})")
    return tr[3:3 + ctas * rounds * nev].view(ctas, rounds, nev).double().cpu()


def phase_table(t: torch.Tensor) -> list[dict]:
    """Per round: median over CTAs of each phase's duration (µs), the round's
    median start and the latest end, both relative to the first CTA's start."""
    t0 = t[:, 0, 0].min()
    out = []
    for r in range(t.shape[1]):
        d = (t[:, r, 1:] - t[:, r, :-1]) / 1000.0
        row = {p: float(d[:, i].median()) for i, p in enumerate(PHASES)}
        row["start_us"] = float((t[:, r, 0].median() - t0) / 1000.0)
        row["end_us"] = float((t[:, r, -1].max() - t0) / 1000.0)
        out.append(row)
    return out


def scorer_phases(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window: int, eps: float = 1e-6,
                  round_p: bool = True, warmup: int = 3) -> list[dict]:
    """Run ``dropkv_scores`` (``warmup`` + 1 times) and return the last launch's
    per-round phase durations. Only the tensor-core scorer records a trace."""
    B, Hq, Lq, D = Q.shape
    _, Hkv, Lk, _ = K.shape
    lib = _lib.load()
    dt = ops._DTYPE_CODE[Q.dtype]
    off = lib.dropkv_scores_status_offset(dt, B, Hq, Hkv, Lk, D, int(window))
    if off == _lib.NO_STATUS:
        raise ValueError("this problem runs on the CUDA-core scorer, which records no trace")
    dev = Q.device
    ws = torch.empty(lib.dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, int(window)), dtype=torch.uint8,
                     device=dev)
    out = torch.empty(B, Hkv, Lk, dtype=torch.float32, device=dev)
    for _ in range(warmup + 1):
        rc = lib.dropkv_scores(Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(), dt, B, Hq, Hkv, Lk, D,
                               int(window), float(eps), ops._ROUND_CODE[Q.dtype] if round_p else _lib.ROUND_NONE,
                               out.data_ptr(), ws.data_ptr(), ws.numel(), ops._stream(dev))
        _lib.check(rc, "dropkv_scores")
    torch.cuda.synchronize(dev)
    status = int(ws[off:off + 4].view(torch.int32).item())
    if status:
        raise _lib.DropKVError(_lib.ERR_DEVICE, f"scorer device status {status}")
    return phase_table(read_trace(ws, off))
