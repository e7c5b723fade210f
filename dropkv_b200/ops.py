"""Tensor-level operations over the C ABI (torch supplies memory and streams).

* ``dropkv_scores_cuda`` -- drop-in for ``dropkv_scores_triton``
  (dropkv_triton.py:643-828): same signature, same precondition checks with the same
  ``AssertionError`` messages (dropkv_triton.py:679-707), same output.
* ``scores``             -- the unguarded scorer used by the cache (also takes fp32
  and windows shorter than the requested one, which the reference handles in its
  PyTorch branch, dropkv_cache.py:401-460).
* ``select_keep_indices`` -- pool + protect + top-k + sort (dropkv_cache.py:462-477).
* ``gather_compressed``  -- dropkv_cache.py:479-491.
* ``compress``           -- the whole path in one C call.
* ``compress_strided``   -- the same over preallocated row buffers (in-place
  chunked prefill storage, no concatenation).
* ``compress_varlen`` / ``VarlenCompressor`` -- a ragged batch (sequences of
  different lengths) in one C call, keep_len per sequence evaluated on the device
  from the reference's rule (dropkv_cache.py:470-473) with per-sequence
  total_tokens / max_keep_len (the chunked-prefill policies, dropkv_cache.py:749-788).
"""

from __future__ import annotations

import contextlib
import functools
import math
import os

import torch

from . import _lib

# With DROPKV_CHECK_STATUS=1 every scoring call synchronises and reads the device
# status word of the tensor-core scorer (non-zero: a bounded wait timed out).
_CHECK_STATUS = os.environ.get("DROPKV_CHECK_STATUS", "0") not in ("", "0")

_DTYPE_CODE = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16,
               torch.bfloat16: _lib.DTYPE_BF16}
_ROUND_CODE = {torch.float32: _lib.ROUND_NONE, torch.float16: _lib.ROUND_F16,
               torch.bfloat16: _lib.ROUND_BF16}


def _require_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("dropkv_b200 runs on CUDA tensors only (no CPU path); got a "
                               f"tensor on {t.device}")


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_status(ws: torch.Tensor, dtype_code: int, B, Hq, Hkv, Lk, D, window, what: str):
    off = _lib.load().dropkv_scores_status_offset(dtype_code, B, Hq, Hkv, Lk, D, int(window))
    if off == _lib.NO_STATUS:
        return
    st = int(ws[off:off + 4].view(torch.int32).item())
    if st != 0:
        raise _lib.DropKVError(_lib.ERR_DEVICE, f"{what}: device status {st} (a bounded wait timed out)")


def scorer_for(dtype: torch.dtype, B, Hq, Hkv, Lk, D, window) -> str:
    """'tensor_cores' or 'cuda_cores': which scorer serves this problem."""
    r = _lib.load().dropkv_scorer_for(_DTYPE_CODE[dtype], B, Hq, Hkv, Lk, D, int(window))
    return {1: "cuda_cores", 2: "tensor_cores"}.get(r, "invalid")


@functools.lru_cache(maxsize=4096)
def _compress_plan(mode: int, device_index: int, dt: int, B: int, Hq: int, Hkv: int, Lk: int, D: int,
                   window: int, score_window: int):
    """(scorer served by the tensor cores, workspace bytes) of a compress problem on
    the current device; the answers depend only on these values (the scorer mode,
    the device's SM count and the shape), so they are computed once per key."""
    lib = _lib.load()
    tc = lib.dropkv_scorer_for(dt, B, Hq, Hkv, Lk, D, score_window) == 2
    return tc, int(lib.dropkv_compress_workspace_size(B, Hq, Hkv, Lk, D, window))


def _on_device(dev: torch.device):
    """The device guard, skipped when ``dev`` is already the current device."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


def _workspace(nbytes: int, device) -> torch.Tensor:
    # caching-allocator blocks are 512-byte aligned, above the 256 bytes the C ABI asks
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def scores(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window: int, eps: float = 1e-6,
           round_p: bool = True) -> torch.Tensor:
    """fp32 scores [B, Hkv, Lk] from the last ``window`` rows of Q.

    ``round_p`` rounds p to the input dtype before the weight (the
    ``match_pytorch_precision`` behaviour, dropkv_triton.py:584-587); it is a no-op
    for fp32 inputs.  K and V must be contiguous; Q may have any strides.
    """
    _require_cuda(Q, K, V)
    B, Hq, Lq, D = Q.shape
    _, Hkv, Lk, _ = K.shape
    dt = _DTYPE_CODE.get(Q.dtype)
    if dt is None or K.dtype != Q.dtype or V.dtype != Q.dtype:
        raise TypeError(f"Q, K, V must share one of fp32/fp16/bf16; got {Q.dtype}, {K.dtype}, {V.dtype}")
    if not (K.is_contiguous() and V.is_contiguous()):
        raise ValueError("K and V must be contiguous")
    lib = _lib.load()
    dev = Q.device
    with torch.cuda.device(dev):
        out = torch.empty(B, Hkv, Lk, dtype=torch.float32, device=dev)
        nws = lib.dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, int(window))
        ws = _workspace(nws, dev)
        rc = lib.dropkv_scores(Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(), dt,
                               B, Hq, Hkv, Lk, D, int(window), float(eps),
                               _ROUND_CODE[Q.dtype] if round_p else _lib.ROUND_NONE,
                               out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
        _lib.check(rc, "dropkv_scores")
        if _CHECK_STATUS:
            _check_status(ws, dt, B, Hq, Hkv, Lk, D, window, "dropkv_scores")
    return out


def dropkv_scores_cuda(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window_size: int = 8,
                       eps: float = 1e-6, allow_tf32: bool = True,
                       match_pytorch_precision: bool = True) -> torch.Tensor:
    """Drop-in replacement of ``dropkv_scores_triton`` (dropkv_triton.py:643-828).

    Same arguments and preconditions; ``allow_tf32`` is accepted for signature
    compatibility (y is always accumulated in fp32 here, never TF32-rounded).
    Returns scores [B, Hkv, Lk] fp32.
    """
    B, Hq, Lq, D = Q.shape
    Hkv = K.shape[1]
    Lk = K.shape[2]
    # Preconditions and messages of dropkv_triton.py:679-707.
    assert isinstance(window_size, int) and window_size > 0, (
        f"window_size must be a positive int, got {window_size}")
    assert Lq >= window_size, f"Lq ({Lq}) must be >= window_size ({window_size})"
    assert Lk >= window_size, f"Lk ({Lk}) must be >= window_size ({window_size})"
    assert Lq <= Lk, f"Lq ({Lq}) must be <= Lk ({Lk}) (Q must be tail-aligned suffix)"
    assert Hq % Hkv == 0, f"Hq ({Hq}) must be divisible by Hkv ({Hkv})"
    assert Q.is_cuda, "Inputs must be on CUDA"
    assert Q.device == K.device == V.device, "All inputs must be on same device"
    assert K.is_contiguous() and V.is_contiguous(), (
        "K and V must be contiguous (Q is sliced internally)")
    assert Q.dtype == K.dtype == V.dtype, "All inputs must have same dtype"
    assert Q.dtype in (torch.float16, torch.bfloat16), (
        f"Input dtype must be fp16 or bf16, got {Q.dtype}")
    assert K.shape == V.shape, f"K and V shape mismatch: K={K.shape}, V={V.shape}"
    assert K.shape[0] == B and K.shape[3] == D, (
        f"K batch/head_dim mismatch: expected B={B}, D={D}, got K={K.shape}")
    return scores(Q, K, V, window_size, eps, round_p=match_pytorch_precision)


def select_keep_indices(scores_: torch.Tensor, kernel_size: int, protect_window: int,
                        keep_len: int) -> torch.Tensor:
    """keep_idx [B, Hkv, keep_len] int64 ascending (dropkv_cache.py:464-475)."""
    _require_cuda(scores_)
    if scores_.dtype != torch.float32:
        raise TypeError("scores must be float32")
    s = scores_.contiguous()
    B, Hkv, Lk = s.shape
    lib = _lib.load()
    dev = s.device
    with torch.cuda.device(dev):
        idx = torch.empty(B, Hkv, keep_len, dtype=torch.int64, device=dev)
        ws = _workspace(lib.dropkv_select_workspace_size(B, Hkv, Lk), dev)
        rc = lib.dropkv_select(s.data_ptr(), B, Hkv, Lk, int(kernel_size), int(protect_window),
                               int(keep_len), idx.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
        _lib.check(rc, "dropkv_select")
    return idx


def gather_compressed(K: torch.Tensor, V: torch.Tensor, keep_idx: torch.Tensor):
    """(K_c, V_c) = rows ``keep_idx`` of K and V along dim 2 (dropkv_cache.py:479-491)."""
    _require_cuda(K, V, keep_idx)
    K = K.contiguous()
    V = V.contiguous()
    if K.shape != V.shape or K.dtype != V.dtype:
        raise ValueError("K and V must have the same shape and dtype")
    idx = keep_idx.to(torch.int64).contiguous()
    B, Hkv, Lk, D = K.shape
    kl = idx.shape[-1]
    if tuple(idx.shape[:2]) != (B, Hkv):
        raise ValueError(f"keep_idx shape {tuple(idx.shape)} does not match K {tuple(K.shape)}")
    Kc = torch.empty(B, Hkv, kl, D, dtype=K.dtype, device=K.device)
    Vc = torch.empty_like(Kc)
    if kl == 0:
        return Kc, Vc
    lib = _lib.load()
    with torch.cuda.device(K.device):
        rc = lib.dropkv_gather(K.data_ptr(), V.data_ptr(), K.element_size(), B, Hkv, Lk, D,
                               idx.data_ptr(), kl, Kc.data_ptr(), Vc.data_ptr(), _stream(K.device))
        _lib.check(rc, "dropkv_gather")
    return Kc, Vc


def _kv_strides(K: torch.Tensor, V: torch.Tensor):
    """Element strides (sequence, head, key) shared by K and V [B, Hkv, L, D] when
    their rows of D elements are contiguous, every stride is a multiple of 16 bytes
    and both start on a 16-byte boundary; else None. Size-1 dimensions take the
    packed stride, which their real stride cannot contradict."""
    if K.shape != V.shape or K.dim() != 4 or K.stride(3) != 1 or V.stride(3) != 1:
        return None
    B, Hkv, L, D = K.shape
    out = []
    for T in (K, V):
        sb, sh, ss, _ = T.stride()
        ss = D if L == 1 else ss
        sh = L * ss if Hkv == 1 else sh
        sb = Hkv * sh if B == 1 else sb
        out.append((sb, sh, ss))
    if out[0] != out[1]:
        return None
    sb, sh, ss = out[0]
    eb = K.element_size()
    if ss < D or min(sb, sh) < 1 or any((x * eb) % 16 for x in (sb, sh, ss)):
        return None
    if K.data_ptr() % 16 or V.data_ptr() % 16:
        return None
    return sb, sh, ss


def compress(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window: int, kernel_size: int,
             keep_len: int, protect_window: int | None = None, eps: float = 1e-6,
             round_p: bool = True, return_scores: bool = False):
    """scores -> pool/protect -> top-k -> sort -> gather in one C call.

    Returns (keep_idx, K_c, V_c) and, with ``return_scores``, the raw scores too.
    ``window`` is the scoring window (rows of Q used); ``protect_window`` the number
    of newest positions forced into the kept set (defaults to ``window``).
    """
    _require_cuda(Q, K, V)
    B, Hq, Lq, D = Q.shape
    _, Hkv, Lk, _ = K.shape
    dt = _DTYPE_CODE.get(Q.dtype)
    if dt is None or K.dtype != Q.dtype or V.dtype != Q.dtype:
        raise TypeError(f"Q, K, V must share one of fp32/fp16/bf16; got {Q.dtype}, {K.dtype}, {V.dtype}")
    # K/V views of another layout (a model's [B, L, Hkv, D] projections viewed as
    # [B, Hkv, L, D]) are read in place when the tensor-core scorer serves the
    # problem; otherwise they are packed first
    pw = window if protect_window is None else protect_window
    lib = _lib.load()
    dev = Q.device
    with _on_device(dev):
        tc, nws = _compress_plan(_lib.scorer_mode, torch.cuda.current_device(), dt, B, Hq, Hkv, Lk, D, int(window),
                                 min(int(window), Lq))
        strides = None if (K.is_contiguous() and V.is_contiguous()) else _kv_strides(K, V)
        if strides is not None and not tc:
            strides = None
        if strides is None:
            K = K.contiguous()
            V = V.contiguous()
        idx = torch.empty(B, Hkv, keep_len, dtype=torch.int64, device=dev)
        Kc = torch.empty(B, Hkv, keep_len, D, dtype=K.dtype, device=dev)
        Vc = torch.empty_like(Kc)
        sc = torch.empty(B, Hkv, Lk, dtype=torch.float32, device=dev) if return_scores else None
        ws = _workspace(nws, dev)
        rnd = _ROUND_CODE[Q.dtype] if round_p else _lib.ROUND_NONE
        tail = (int(kernel_size), int(pw), int(keep_len), sc.data_ptr() if sc is not None else None,
                idx.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
        if strides is None:
            rc = lib.dropkv_compress(Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(), dt,
                                     B, Hq, Hkv, Lk, D, int(window), float(eps), rnd, *tail)
            _lib.check(rc, "dropkv_compress")
        else:
            rc = lib.dropkv_compress_kv_strides(Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(),
                                                *strides, dt, B, Hq, Hkv, Lk, D, int(window), float(eps), rnd,
                                                *tail)
            _lib.check(rc, "dropkv_compress_kv_strides")
        if _CHECK_STATUS:
            _check_status(ws, dt, B, Hq, Hkv, Lk, D, window, "dropkv_compress")
    if return_scores:
        return idx, Kc, Vc, sc
    return idx, Kc, Vc


def compress_workspace_size(B: int, Hq: int, Hkv: int, Lk: int, D: int, window: int) -> int:
    """Scratch bytes of compress / compress_strided for this problem."""
    return int(_lib.load().dropkv_compress_workspace_size(B, Hq, Hkv, Lk, D, int(window)))


def compress_strided(Q: torch.Tensor, K_buf: torch.Tensor, V_buf: torch.Tensor, Lk: int, window: int,
                     kernel_size: int, keep_len: int, K_out: torch.Tensor, V_out: torch.Tensor,
                     protect_window: int | None = None, eps: float = 1e-6, round_p: bool = True,
                     workspace: torch.Tensor | None = None, idx_out: torch.Tensor | None = None) -> torch.Tensor:
    """``compress`` over row buffers: scores the first ``Lk`` rows of ``K_buf`` /
    ``V_buf`` ([B, Hkv, capacity, D], contiguous) and writes the kept rows to rows
    ``[0, keep_len)`` of ``K_out`` / ``V_out`` ([B, Hkv, capacity', D], contiguous,
    not the input buffers).  Returns keep_idx [B, Hkv, keep_len] (ascending).
    Same results as ``compress`` on the same rows; nothing is concatenated.
    ``workspace`` (uint8, large enough) and ``idx_out`` (int64, at least
    B * Hkv * keep_len elements) are used instead of allocating when given."""
    _require_cuda(Q, K_buf, V_buf, K_out, V_out)
    B, Hq, Lq, D = Q.shape
    Bk, Hkv, cap, Dk = K_buf.shape
    dt = _DTYPE_CODE.get(Q.dtype)
    if dt is None or K_buf.dtype != Q.dtype or V_buf.dtype != Q.dtype or K_out.dtype != Q.dtype:
        raise TypeError("Q, K/V buffers and outputs must share one of fp32/fp16/bf16")
    for t in (K_buf, V_buf, K_out, V_out):
        if not t.is_contiguous():
            raise ValueError("row buffers must be contiguous [B, Hkv, capacity, D]")
    if K_buf.shape != V_buf.shape or K_out.shape != V_out.shape or Bk != B or Dk != D:
        raise ValueError("buffer shapes disagree")
    if not 1 <= Lk <= cap or keep_len > K_out.shape[2]:
        raise ValueError(f"Lk={Lk} must fit the input buffer ({cap} rows) and keep_len={keep_len} the "
                         f"output buffer ({K_out.shape[2]} rows)")
    if K_out.data_ptr() == K_buf.data_ptr():
        raise ValueError("K_out must not be the input buffer")
    pw = window if protect_window is None else protect_window
    lib = _lib.load()
    dev = Q.device
    with torch.cuda.device(dev):
        n_idx = B * Hkv * keep_len
        if idx_out is not None and idx_out.dtype == torch.int64 and idx_out.numel() >= n_idx and idx_out.is_contiguous():
            idx = idx_out.view(-1)[:n_idx].view(B, Hkv, keep_len)
        else:
            idx = torch.empty(B, Hkv, keep_len, dtype=torch.int64, device=dev)
        need = lib.dropkv_compress_workspace_size(B, Hq, Hkv, Lk, D, int(window))
        ws = workspace if workspace is not None and workspace.numel() >= need else _workspace(need, dev)
        rc = lib.dropkv_compress_strided(Q.data_ptr(), *Q.stride(), Lq, K_buf.data_ptr(), V_buf.data_ptr(),
                                         cap * D, dt, B, Hq, Hkv, int(Lk), D, int(window), float(eps),
                                         _ROUND_CODE[Q.dtype] if round_p else _lib.ROUND_NONE,
                                         int(kernel_size), int(pw), int(keep_len), None, idx.data_ptr(),
                                         K_out.data_ptr(), V_out.data_ptr(), K_out.shape[2] * D,
                                         ws.data_ptr(), ws.numel(), _stream(dev))
        _lib.check(rc, "dropkv_compress_strided")
        if _CHECK_STATUS:
            _check_status(ws, dt, B, Hq, Hkv, Lk, D, window, "dropkv_compress_strided")
    return idx


_DA_WS: dict = {}  # per device: zero-initialised decode-attention workspace (kept zeroed by the library)


def decode_attention_workspace(B: int, Hq: int, Hkv: int, Lq: int, L: int, D: int, device) -> torch.Tensor:
    """A zero-filled workspace for ``decode_attention`` of this shape (fresh)."""
    n = _lib.load().dropkv_decode_attention_workspace_size(B, Hq, Hkv, Lq, L, D)
    return torch.zeros(max(int(n), 1), dtype=torch.uint8, device=device)


def decode_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of the Lq query rows over the cached keys: [B, Hq, Lq, D] ->
    [B, Hq, Lq, D], softmax(scale Q K^T) V per KV-head group, the query rows
    tail-aligned to the L keys (row i sees keys j <= L - Lq + i).

    This is what the model computes over the K/V that ``DropKVCache.update``
    returns during decode (dropkv_cache.py:609-617 append the token; the model's
    SDPA attends). K and V may be views into row buffers with spare capacity
    (rows of D contiguous elements, any head and batch stride), as
    ``DropKVCache(storage="buffer")`` hands out. ``workspace`` must be zero-filled
    before its first use (``decode_attention_workspace``); the library leaves it
    zeroed, so it can be reused, but not by calls running concurrently on two
    streams. Without one, a per-device workspace is kept here.
    """
    _require_cuda(Q, K, V)
    if Q.dim() != 4 or K.dim() != 4 or K.shape != V.shape:
        raise ValueError("expected Q [B,Hq,Lq,D] and K, V [B,Hkv,L,D] of one shape")
    if not (Q.dtype == K.dtype == V.dtype) or Q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("decode attention takes bf16 or fp16 Q, K and V of one dtype")
    B, Hq, Lq, D = Q.shape
    _, Hkv, L, _ = K.shape
    if K.shape[0] != B or K.shape[3] != D or Hq % Hkv:
        raise ValueError(f"shape mismatch: Q {tuple(Q.shape)}, K {tuple(K.shape)}")
    if K.stride() != V.stride() or K.stride(3) != 1 or K.stride(2) != D:
        raise ValueError("K and V need rows of D contiguous elements and equal strides")
    scale = float(D ** -0.5 if scale is None else scale)
    lib = _lib.load()
    dev = Q.device
    need = lib.dropkv_decode_attention_workspace_size(B, Hq, Hkv, Lq, L, D)
    if workspace is None:
        workspace = _DA_WS.get(dev)
        if workspace is None or workspace.numel() < need:
            workspace = torch.zeros(max(int(need), 1), dtype=torch.uint8, device=dev)
            _DA_WS[dev] = workspace
    out = torch.empty(B, Hq, Lq, D, dtype=Q.dtype, device=dev)
    with torch.cuda.device(dev):
        rc = lib.dropkv_decode_attention(Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(), K.stride(0),
                                         K.stride(1), _DTYPE_CODE[Q.dtype], B, Hq, Hkv, L, D, scale,
                                         out.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream(dev))
        _lib.check(rc, "dropkv_decode_attention")
    return out


def decode_append_attention(Q: torch.Tensor, K_new: torch.Tensor, V_new: torch.Tensor, K_buf: torch.Tensor,
                            V_buf: torch.Tensor, pos: int, scale: float | None = None,
                            workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Append the decode rows and attend over the cache in one launch.

    K_new, V_new [B, Hkv, n, D] are stored into the row buffers K_buf, V_buf
    [B, Hkv, cap, D] at rows [pos, pos + n) and Q [B, Hq, Lq, D] attends over rows
    [0, pos + n) -- the same output, bit for bit, as writing the rows and then
    calling ``decode_attention(Q, K_buf[:, :, :pos + n], V_buf[:, :, :pos + n])``
    (dropkv_cache.py:609-617 concatenate the token; the model's SDPA attends). The
    buffers need rows of D contiguous elements and cap >= pos + n; the workspace
    rules are those of ``decode_attention``.
    """
    _require_cuda(Q, K_new, V_new, K_buf, V_buf)
    if Q.dim() != 4 or K_new.dim() != 4 or K_buf.dim() != 4 or K_new.shape != V_new.shape \
            or K_buf.shape != V_buf.shape:
        raise ValueError("expected Q [B,Hq,Lq,D], K_new, V_new [B,Hkv,n,D] and K_buf, V_buf [B,Hkv,cap,D]")
    if not (Q.dtype == K_new.dtype == V_new.dtype == K_buf.dtype == V_buf.dtype) \
            or Q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("decode attention takes bf16 or fp16 tensors of one dtype")
    B, Hq, Lq, D = Q.shape
    _, Hkv, n, _ = K_new.shape
    cap = K_buf.shape[2]
    pos = int(pos)
    if K_new.shape[0] != B or K_new.shape[3] != D or K_buf.shape[0] != B or K_buf.shape[1] != Hkv \
            or K_buf.shape[3] != D or Hq % Hkv:
        raise ValueError(f"shape mismatch: Q {tuple(Q.shape)}, K_new {tuple(K_new.shape)}, "
                         f"K_buf {tuple(K_buf.shape)}")
    if pos < 0 or pos + n > cap:
        raise ValueError(f"rows [{pos}, {pos + n}) do not fit a buffer of {cap} rows")
    for name, t, u in (("K_buf", K_buf, V_buf), ("K_new", K_new, V_new)):
        if t.stride() != u.stride() or t.stride(3) != 1 or (t.stride(2) != D and t.shape[2] > 1):
            raise ValueError(f"{name} and its V need rows of D contiguous elements and equal strides")
    scale = float(D ** -0.5 if scale is None else scale)
    lib = _lib.load()
    dev = Q.device
    L = pos + n
    need = lib.dropkv_decode_attention_workspace_size(B, Hq, Hkv, Lq, L, D)
    if workspace is None:
        workspace = _DA_WS.get(dev)
        if workspace is None or workspace.numel() < need:
            workspace = torch.zeros(max(int(need), 1), dtype=torch.uint8, device=dev)
            _DA_WS[dev] = workspace
    out = torch.empty(B, Hq, Lq, D, dtype=Q.dtype, device=dev)
    with torch.cuda.device(dev):
        rc = lib.dropkv_decode_append_attention(Q.data_ptr(), *Q.stride(), Lq, K_new.data_ptr(), V_new.data_ptr(),
                                                K_new.stride(0), K_new.stride(1), n, K_buf.data_ptr(),
                                                V_buf.data_ptr(), K_buf.stride(0), K_buf.stride(1), pos,
                                                _DTYPE_CODE[Q.dtype], B, Hq, Hkv, D, scale, out.data_ptr(),
                                                workspace.data_ptr(), workspace.numel(), _stream(dev))
        _lib.check(rc, "dropkv_decode_append_attention")
    return out


def inv_sqrt_d(D: int) -> float:
    return 1.0 / math.sqrt(D)


class Compressor:
    """Pre-planned ``compress`` for a fixed problem shape.

    Holds the outputs (keep_idx, K_c, V_c, optionally scores) and the scratch
    workspace, so ``run`` issues exactly one C-ABI call and allocates nothing --
    suitable for timing loops and CUDA-graph capture.
    """

    def __init__(self, B: int, Hq: int, Hkv: int, Lq: int, Lk: int, D: int, dtype: torch.dtype,
                 window: int, kernel_size: int, keep_len: int, protect_window: int | None = None,
                 eps: float = 1e-6, round_p: bool = True, keep_scores: bool = False,
                 device="cuda"):
        self.shape = (B, Hq, Hkv, Lq, Lk, D)
        self.dtype = dtype
        self.window = int(window)
        self.kernel_size = int(kernel_size)
        self.keep_len = int(keep_len)
        self.protect = int(window if protect_window is None else protect_window)
        self.eps = float(eps)
        self.round = _ROUND_CODE[dtype] if round_p else _lib.ROUND_NONE
        self.device = torch.device(device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            self.keep_idx = torch.empty(B, Hkv, keep_len, dtype=torch.int64, device=self.device)
            self.k_out = torch.empty(B, Hkv, keep_len, D, dtype=dtype, device=self.device)
            self.v_out = torch.empty_like(self.k_out)
            self.scores = (torch.empty(B, Hkv, Lk, dtype=torch.float32, device=self.device)
                           if keep_scores else None)
            self.workspace = _workspace(
                lib.dropkv_compress_workspace_size(B, Hq, Hkv, Lk, D, self.window), self.device)

    def run(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, stream: int | None = None):
        B, Hq, Hkv, Lq, Lk, D = self.shape
        if tuple(Q.shape) != (B, Hq, Lq, D) or tuple(K.shape) != (B, Hkv, Lk, D) or K.shape != V.shape:
            raise ValueError("input shapes do not match this Compressor")
        if not (K.is_contiguous() and V.is_contiguous()):
            raise ValueError("K and V must be contiguous")
        lib = _lib.load()
        st = _stream(self.device) if stream is None else stream
        rc = lib.dropkv_compress(Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(),
                                 _DTYPE_CODE[self.dtype], B, Hq, Hkv, Lk, D, self.window, self.eps,
                                 self.round, self.kernel_size, self.protect, self.keep_len,
                                 self.scores.data_ptr() if self.scores is not None else None,
                                 self.keep_idx.data_ptr(), self.k_out.data_ptr(),
                                 self.v_out.data_ptr(), self.workspace.data_ptr(),
                                 self.workspace.numel(), st)
        _lib.check(rc, "dropkv_compress")
        return self.keep_idx, self.k_out, self.v_out

    def capture(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> int:
        """Capture one ``run`` on these (fixed-address) inputs into a CUDA graph that
        ``replay`` launches again: the same kernels and copies, without the host's
        per-call work. Returns the number of kernel launches in the graph."""
        cur = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            self.run(Q, K, V)  # first use of every kernel and launch attribute off the capture
        cur.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        n0 = _lib.launch_count()
        # thread_local: CUDA calls other threads make meanwhile (a communication
        # library's watchdog, say) do not invalidate this capture
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            self.run(Q, K, V)
        self.graph = graph
        self.graph_launches = _lib.launch_count() - n0
        return self.graph_launches

    def replay(self):
        """Launch the graph ``capture`` recorded (on the current stream)."""
        self.graph.replay()
        return self.keep_idx, self.k_out, self.v_out


class HostPipeline:
    """Compress a sequence of layers whose Q/K/V live in (pinned) host memory and
    whose outputs go back to host memory, as for a KV cache offloaded to the host.

    Two device slots, each with its input buffers and a ``Compressor``, and one
    CUDA stream per stage: the host-to-device copy of layer i + 1 runs while layer
    i is compressed and its outputs copied back, so the PCIe link stays busy in
    both directions. Every layer's copies and compression are done; only their
    order in time overlaps. Host tensors should be pinned for the copies to be
    asynchronous.
    """

    def __init__(self, B: int, Hq: int, Hkv: int, Lq: int, Lk: int, D: int, dtype: torch.dtype,
                 window: int, kernel_size: int, keep_len: int, device="cuda", **kw):
        self.device = torch.device(device)
        self.shape = (B, Hq, Hkv, Lq, Lk, D)
        with torch.cuda.device(self.device):
            self.comps = [Compressor(B, Hq, Hkv, Lq, Lk, D, dtype, window, kernel_size, keep_len,
                                     device=self.device, **kw) for _ in range(2)]
            self.inputs = [(torch.empty(B, Hq, Lq, D, dtype=dtype, device=self.device),
                            torch.empty(B, Hkv, Lk, D, dtype=dtype, device=self.device),
                            torch.empty(B, Hkv, Lk, D, dtype=dtype, device=self.device)) for _ in range(2)]
            self.h2d = torch.cuda.Stream(self.device)
            self.work = torch.cuda.Stream(self.device)
            self.d2h = torch.cuda.Stream(self.device)
        self.loaded = [torch.cuda.Event() for _ in range(2)]
        self.computed = [torch.cuda.Event() for _ in range(2)]
        self.returned = [torch.cuda.Event() for _ in range(2)]
        self.used = [False, False]

    def run(self, layers):
        """``layers``: iterable of (Qh, Kh, Vh, idx_out, kc_out, vc_out) host tensors;
        inputs [B,Hq,Lq,D] / [B,Hkv,Lk,D], outputs [B,Hkv,keep_len] int64 and
        [B,Hkv,keep_len,D]. Enqueues everything and returns the event that
        completes when the last output has reached the host (the caller
        synchronises on it before reading the outputs)."""
        last = None
        for i, (Qh, Kh, Vh, idx_o, kc_o, vc_o) in enumerate(layers):
            s = i % 2
            Qd, Kd, Vd = self.inputs[s]
            comp = self.comps[s]
            with torch.cuda.stream(self.h2d):
                if self.used[s]:  # the slot's inputs were read by its previous compression
                    self.h2d.wait_event(self.computed[s])
                Qd.copy_(Qh, non_blocking=True)
                Kd.copy_(Kh, non_blocking=True)
                Vd.copy_(Vh, non_blocking=True)
                self.loaded[s].record(self.h2d)
            self.work.wait_event(self.loaded[s])
            if self.used[s]:  # the slot's outputs were copied out
                self.work.wait_event(self.returned[s])
            comp.run(Qd, Kd, Vd, stream=self.work.cuda_stream)
            self.computed[s].record(self.work)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.computed[s])
                idx_o.copy_(comp.keep_idx, non_blocking=True)
                kc_o.copy_(comp.k_out, non_blocking=True)
                vc_o.copy_(comp.v_out, non_blocking=True)
                self.returned[s].record(self.d2h)
            self.used[s] = True
            last = self.returned[s]
        if last is None:  # nothing enqueued: an event that completes at once
            last = torch.cuda.Event()
            last.record(self.d2h)
        return last


def _device_i64(x, n: int, device, what: str):
    """None, a device int64 tensor [n], or a sequence of n ints (None -> -1)."""
    if x is None:
        return None
    if isinstance(x, torch.Tensor):
        if x.dtype != torch.int64 or x.numel() != n or not x.is_cuda:
            raise ValueError(f"{what} must be an int64 CUDA tensor of {n} entries")
        return x.contiguous()
    vals = [-1 if v is None else int(v) for v in x]
    if len(vals) != n:
        raise ValueError(f"{what} needs {n} entries, got {len(vals)}")
    return torch.tensor(vals, dtype=torch.int64, device=device)


class VarlenCompressor:
    """Pre-planned ``dropkv_compress_varlen`` for a fixed ragged batch.

    ``shapes``: per sequence (B, Lq, Lk) -- B rows of the sequence's batch (its
    layers stacked, say), Lq query rows, Lk keys -- at most ``VARLEN_MAX_SEQS``
    sequences. Holds per sequence the outputs keep_idx [B, Hkv, cap] and
    K_c / V_c [B, Hkv, cap, D] (``cap``: rows of room, default Lk), the device
    vector ``keep_len`` [n] (int32) and the workspace, so ``run`` issues exactly one
    C-ABI call and allocates nothing (CUDA-graph capturable). Rows of an output
    past its sequence's keep_len are left as they were.
    """

    def __init__(self, shapes, Hq: int, Hkv: int, D: int, dtype: torch.dtype, window: int, kernel_size: int,
                 keep_ratio: float, caps=None, keep_window: int | None = None, protect_window: int | None = None,
                 eps: float = 1e-6, round_p: bool = True, device="cuda"):
        n = len(shapes)
        if not 1 <= n <= _lib.VARLEN_MAX_SEQS:
            raise ValueError(f"1..{_lib.VARLEN_MAX_SEQS} sequences per VarlenCompressor, got {n}")
        if dtype not in _DTYPE_CODE:
            raise TypeError(f"unsupported dtype {dtype}")
        self.shapes = [tuple(int(x) for x in sh) for sh in shapes]
        self.caps = [lk for (_, _, lk) in self.shapes] if caps is None else [int(c) for c in caps]
        if len(self.caps) != n:
            raise ValueError(f"caps needs {n} entries")
        self.Hq, self.Hkv, self.D, self.dtype = int(Hq), int(Hkv), int(D), dtype
        self.window, self.kernel_size = int(window), int(kernel_size)
        self.keep_ratio = float(keep_ratio)
        self.keep_window = int(window if keep_window is None else keep_window)
        self.protect = int(window if protect_window is None else protect_window)
        self.eps = float(eps)
        self.round = _ROUND_CODE[dtype] if round_p else _lib.ROUND_NONE
        self.device = torch.device(device)
        lib = _lib.load()
        self._seqs = (_lib.VarlenSeq * n)()
        with torch.cuda.device(self.device):
            self.outputs = []
            for i, ((B, Lq, Lk), cap) in enumerate(zip(self.shapes, self.caps)):
                idx = torch.empty(B, Hkv, cap, dtype=torch.int64, device=self.device)
                kc = torch.empty(B, Hkv, cap, D, dtype=dtype, device=self.device)
                vc = torch.empty_like(kc)
                self.outputs.append((idx, kc, vc))
                sq = self._seqs[i]
                sq.Lq, sq.B, sq.Lk, sq.cap = Lq, B, Lk, cap
                sq.keep_idx, sq.k_out, sq.v_out = idx.data_ptr(), kc.data_ptr(), vc.data_ptr()
            self.keep_len = torch.zeros(n, dtype=torch.int32, device=self.device)
            nbytes = lib.dropkv_compress_varlen_workspace_size(n, self._seqs, self.Hq, self.Hkv, self.D, self.window)
            if nbytes == 0:
                raise ValueError("invalid ragged batch shapes")
            self.workspace = _workspace(nbytes, self.device)

    def run(self, Qs, Ks, Vs, total_tokens=None, max_keep_len=None, stream: int | None = None):
        """Compress sequence i from Qs[i] [B, Hq, Lq, D] (any strides) and Ks[i], Vs[i]
        [B, Hkv, Lk, D] (contiguous). ``total_tokens`` / ``max_keep_len``: None, an
        int64 CUDA tensor [n] or n ints (a None / negative max_keep_len entry sets no
        cap). Returns (keep_len [n] int32 on the device, outputs)."""
        n = len(self.shapes)
        if not (len(Qs) == len(Ks) == len(Vs) == n):
            raise ValueError(f"expected {n} sequences")
        _require_cuda(*Qs, *Ks, *Vs)
        for i, (Q, K, V) in enumerate(zip(Qs, Ks, Vs)):
            B, Lq, Lk = self.shapes[i]
            if tuple(Q.shape) != (B, self.Hq, Lq, self.D) or tuple(K.shape) != (B, self.Hkv, Lk, self.D) \
                    or K.shape != V.shape:
                raise ValueError(f"sequence {i}: shapes do not match this VarlenCompressor")
            if Q.dtype != self.dtype or K.dtype != self.dtype or V.dtype != self.dtype:
                raise TypeError(f"sequence {i}: expected {self.dtype}")
            if not (K.is_contiguous() and V.is_contiguous()):
                raise ValueError(f"sequence {i}: K and V must be contiguous")
            sq = self._seqs[i]
            sq.q = Q.data_ptr()
            sq.q_sb, sq.q_sh, sq.q_ss, sq.q_sd = Q.stride()
            sq.k, sq.v = K.data_ptr(), V.data_ptr()
        tt = _device_i64(total_tokens, n, self.device, "total_tokens")
        mk = _device_i64(max_keep_len, n, self.device, "max_keep_len")
        lib = _lib.load()
        st = _stream(self.device) if stream is None else stream
        rc = lib.dropkv_compress_varlen(n, self._seqs, _DTYPE_CODE[self.dtype], self.Hq, self.Hkv, self.D,
                                        self.window, self.eps, self.round, self.kernel_size, self.protect,
                                        self.keep_ratio, self.keep_window,
                                        tt.data_ptr() if tt is not None else None,
                                        mk.data_ptr() if mk is not None else None,
                                        self.keep_len.data_ptr(), self.workspace.data_ptr(),
                                        self.workspace.numel(), st)
        _lib.check(rc, "dropkv_compress_varlen")
        if _CHECK_STATUS and not torch.cuda.is_current_stream_capturing():
            s = int(self.workspace[:4].view(torch.int32).item())
            if s != 0:
                raise _lib.DropKVError(_lib.ERR_DEVICE, f"dropkv_compress_varlen: device status {s} "
                                                        "(a bounded wait timed out)")
        return self.keep_len, self.outputs


def compress_varlen(Qs, Ks, Vs, window: int, kernel_size: int, keep_ratio: float, total_tokens=None,
                    max_keep_len=None, caps=None, keep_window: int | None = None,
                    protect_window: int | None = None, eps: float = 1e-6, round_p: bool = True):
    """A ragged batch of sequences (lists Qs, Ks, Vs: [B_i, Hq, Lq_i, D] and
    [B_i, Hkv, Lk_i, D]) compressed with one C call per ``VARLEN_MAX_SEQS``
    sequences; keep_len per sequence is evaluated on the device. Returns
    (keep_len [n] int32 on the device, [(keep_idx, K_c, V_c)] with cap rows each,
    the rows past keep_len unspecified)."""
    n = len(Qs)
    if n == 0:
        raise ValueError("empty batch")
    _, Hq, _, D = Qs[0].shape
    Hkv = Ks[0].shape[1]
    dev = Qs[0].device
    tt = _device_i64(total_tokens, n, dev, "total_tokens")
    mk = _device_i64(max_keep_len, n, dev, "max_keep_len")
    lens, outs = [], []
    step = _lib.VARLEN_MAX_SEQS
    for a in range(0, n, step):
        b = min(n, a + step)
        shapes = [(Q.shape[0], Q.shape[2], K.shape[2]) for Q, K in zip(Qs[a:b], Ks[a:b])]
        comp = VarlenCompressor(shapes, Hq, Hkv, D, Qs[0].dtype, window, kernel_size, keep_ratio,
                                caps=None if caps is None else caps[a:b], keep_window=keep_window,
                                protect_window=protect_window, eps=eps, round_p=round_p, device=dev)
        kl, o = comp.run([Q for Q in Qs[a:b]], [K.contiguous() for K in Ks[a:b]], [V.contiguous() for V in Vs[a:b]],
                         total_tokens=None if tt is None else tt[a:b],
                         max_keep_len=None if mk is None else mk[a:b])
        lens.append(kl)
        outs.extend(o)
    return torch.cat(lens), outs
