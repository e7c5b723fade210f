"""DropKV KV cache with the CUDA eviction backend.

Keeps the reference's interface and state machine (dropkv_cache.py:310-807) so it
drops in: ``DropKVCache(keep_ratio, window_size, kernel_size, use_triton)``,
``update`` (5-argument form and the HF 4-argument form), ``_compute_keep_indices``,
``_gather_compressed``, ``get_seq_length``, ``get_mask_sizes`` and the
``prefill_chunked`` helper with its three eviction strategies.

What changes is the backend: every eviction runs ``dropkv_b200.ops`` (the C ABI of
libdropkv_b200.so).  ``use_triton`` is accepted for signature compatibility and
both values select the CUDA kernels -- there is no PyTorch or CPU scoring branch.
The reference's PyTorch branch also served queries shorter than the window
(dropkv_cache.py:399-407, scoring window min(window, Lq)); here the CUDA scorer
takes that shorter window directly, and protection still covers ``window_size``
positions (dropkv_cache.py:466-467).
"""

from __future__ import annotations

import logging
from typing import Any, Optional

import torch

from . import _lib, ops

logger = logging.getLogger(__name__)

__all__ = ["DropKVCache", "prefill_chunked"]


class _KVStore:
    """Per-layer K/V storage under DropKVCache's state machine.

    ``key_cache[i]`` / ``value_cache[i]`` hold layer i's retained K and V
    ([B, Hkv, L_i, D]); ``_seen_tokens`` counts the tokens layer 0 has received
    (the logical sequence length that positions continue from after an eviction).
    Layers are indexed by ``cache[i]`` -> (K, V), iterated in order and counted by
    ``len``.  Only what DropKVCache and its callers use is here: no beam-search or
    legacy-format conversions.
    """

    def __init__(self) -> None:
        self._seen_tokens = 0
        self.key_cache: list[torch.Tensor] = []
        self.value_cache: list[torch.Tensor] = []

    def __len__(self) -> int:
        return len(self.key_cache)

    def __getitem__(self, layer_idx: int):
        if not 0 <= layer_idx < len(self.key_cache):
            raise KeyError(f"layer {layer_idx} is not in this cache ({len(self.key_cache)} layers)")
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    def __iter__(self):
        return iter(list(zip(self.key_cache, self.value_cache)))

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        raise NotImplementedError

    def crop(self, max_length: int) -> None:
        """Truncate every layer to its first ``max_length`` positions (a negative
        value drops that many from the end) when the cache's length exceeds it;
        the length is ``get_seq_length()``, as in the reference's base cache
        (dropkv_cache.py:255-269), so for DropKVCache it is the tokens seen."""
        if max_length < 0:
            max_length = self.get_seq_length() - abs(max_length)
        if self.get_seq_length() <= max_length:
            return
        self._seen_tokens = max_length
        for i, k in enumerate(self.key_cache):
            if k.numel():
                self.key_cache[i] = k[..., :max_length, :]
                self.value_cache[i] = self.value_cache[i][..., :max_length, :]


_VALID_MODES = ("single_pass", "accumulate", "evict_accumulated")


class _LayerRows:
    """One layer's K/V for ``DropKVCache(storage="buffer")``: two [B, Hkv, capacity, D]
    buffer pairs used in turn.  Rows [0, n) of the current pair are the layer's
    cache.  New tokens are copied in place after them (the reference concatenates
    stored and new K/V into fresh tensors for every chunk and decode step,
    dropkv_cache.py:581-617).  An eviction scores the current pair's rows and writes
    the kept rows to the other pair, which becomes current; the evicted-from rows
    stay intact until the pair is written again, so the full K/V returned for the
    chunk's attention remains valid until the layer's next update.  Each pair grows
    (doubling, one copy of its live rows) only when it must hold more rows."""

    def __init__(self, like: torch.Tensor):
        self.shape = (like.shape[0], like.shape[1], like.shape[3])
        self.dtype, self.device = like.dtype, like.device
        self.bufs: list = [None, None]
        self.cur = 0
        self.n = 0
        self.last_m = 0  # rows of the last append: an eviction target keeps room for the next one
        self.ws = torch.empty(0, dtype=torch.uint8, device=self.device)    # reused scratch
        self.idx = torch.empty(0, dtype=torch.int64, device=self.device)   # reused keep indices

    def _alloc(self, rows: int):
        B, H, D = self.shape
        return (torch.empty(B, H, rows, D, dtype=self.dtype, device=self.device),
                torch.empty(B, H, rows, D, dtype=self.dtype, device=self.device))

    def _reserve(self, which: int, rows: int, keep_live: bool):
        buf = self.bufs[which]
        have = 0 if buf is None else buf[0].shape[2]
        if rows <= have:
            return
        new = self._alloc(-(-max(rows, 2 * have) // 1024) * 1024)
        if keep_live and buf is not None and self.n:
            new[0][:, :, :self.n].copy_(buf[0][:, :, :self.n])
            new[1][:, :, :self.n].copy_(buf[1][:, :, :self.n])
        self.bufs[which] = new

    def views(self):
        k, v = self.bufs[self.cur]
        return k[:, :, :self.n], v[:, :, :self.n]

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor):
        m = k_new.shape[2]
        self.last_m = max(self.last_m, m)
        self._reserve(self.cur, self.n + m, keep_live=True)
        k, v = self.bufs[self.cur]
        if k.is_cuda and k_new.is_cuda and k_new.is_contiguous() and v_new.is_contiguous() and \
                k_new.dtype == k.dtype and v_new.dtype == k.dtype:
            B, H, D = self.shape
            with torch.cuda.device(self.device):
                rc = _lib.load().dropkv_append_rows(
                    k.data_ptr(), v.data_ptr(), k.shape[2] * D, self.n, k_new.data_ptr(), v_new.data_ptr(),
                    m * D, m, D, k.element_size(), B * H, torch.cuda.current_stream(self.device).cuda_stream)
            _lib.check(rc, "dropkv_append_rows")
        else:  # CPU tensors or non-contiguous chunks
            k[:, :, self.n:self.n + m].copy_(k_new)
            v[:, :, self.n:self.n + m].copy_(v_new)
        self.n += m

    def _compress(self, q, k, v, lk, window, kernel_size, keep_len, ko, vo, protect):
        """dropkv_compress_strided on these buffers (shapes are guaranteed by the
        cache, so the call skips the generic wrapper's checks and allocations)."""
        B, H, D = self.shape
        lib = _lib.load()
        need = lib.dropkv_compress_workspace_size(B, q.shape[1], H, lk, D, window)
        if self.ws.numel() < need:
            self.ws = torch.empty(max(need, 2 * self.ws.numel()), dtype=torch.uint8, device=self.device)
        if self.idx.numel() < B * H * keep_len:
            self.idx = torch.empty(max(B * H * keep_len, 2 * self.idx.numel()), dtype=torch.int64,
                                   device=self.device)
        if q.dtype != self.dtype or not q.is_cuda:
            raise TypeError("query_states must be a CUDA tensor of the cache's dtype")
        with torch.cuda.device(self.device):
            rc = lib.dropkv_compress_strided(
                q.data_ptr(), *q.stride(), q.shape[2], k.data_ptr(), v.data_ptr(), k.shape[2] * D,
                ops._DTYPE_CODE[self.dtype], B, q.shape[1], H, lk, D, window, 1e-6, ops._ROUND_CODE[self.dtype],
                kernel_size, protect, keep_len, None, self.idx.data_ptr(), ko.data_ptr(), vo.data_ptr(),
                ko.shape[2] * D, self.ws.data_ptr(), self.ws.numel(),
                torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "dropkv_compress_strided")

    def evict(self, q: torch.Tensor, window: int, kernel_size: int, keep_len: int, protect: int):
        other = 1 - self.cur
        self._reserve(other, keep_len + self.last_m, keep_live=False)
        (k, v), (ko, vo) = self.bufs[self.cur], self.bufs[other]
        self._compress(q, k, v, self.n, window, kernel_size, keep_len, ko, vo, protect)
        self.cur, self.n = other, keep_len

    def load_evicted(self, q, k, v, window: int, kernel_size: int, keep_len: int, protect: int):
        """First eviction of a layer, straight from the model's contiguous K/V."""
        self._reserve(self.cur, keep_len, keep_live=False)
        ko, vo = self.bufs[self.cur]
        self._compress(q, k, v, k.shape[2], window, kernel_size, keep_len, ko, vo, protect)
        self.n = keep_len


class DropKVCache(_KVStore):
    """KV cache that evicts at prefill with the DropKV score (CUDA backend)."""

    def __init__(self, keep_ratio: float = 0.1, window_size: int = 8, kernel_size: int = 11,
                 use_triton: bool = True, storage: str = "cat") -> None:
        """``storage``: ``"cat"`` (default) keeps the reference's storage, a fresh
        tensor per layer after every update; ``"buffer"`` keeps each layer in
        preallocated row buffers (no copy of the stored cache per chunk or decode
        step).  With ``"buffer"`` the tensors in key_cache / value_cache and those
        update returns are views that stay valid until that layer's next update."""
        super().__init__()
        if storage not in ("cat", "buffer"):
            raise ValueError(f"storage must be 'cat' or 'buffer', got {storage!r}")
        self.storage = storage
        self._rows: list[_LayerRows] = []
        if not 0 < keep_ratio <= 1.0:
            raise ValueError(f"keep_ratio must be in (0, 1], got {keep_ratio}")
        if window_size <= 0:
            raise ValueError(f"window_size must be positive, got {window_size}")
        if kernel_size < 1 or kernel_size % 2 == 0:
            raise ValueError(f"kernel_size must be a positive odd integer, got {kernel_size}")
        self.keep_ratio = keep_ratio
        self.window_size = window_size
        self.kernel_size = kernel_size
        self.use_triton = use_triton  # accepted for compatibility; CUDA either way
        # "single_pass" | "accumulate" | "evict_accumulated" (set by prefill_chunked)
        self._prefill_mode = "single_pass"
        self._evict_use_seen_tokens = False
        self._budget_max_kv_tokens: Optional[int] = None

    def _rebuild_rows(self):
        """Row buffers again from key_cache / value_cache after they were replaced
        by a whole-cache operation (crop)."""
        if self.storage != "buffer":
            return
        self._rows = []
        for i in range(len(self.key_cache)):
            rows = _LayerRows(self.key_cache[i])
            rows.append(self.key_cache[i], self.value_cache[i])
            self._rows.append(rows)
            self.key_cache[i], self.value_cache[i] = rows.views()

    def crop(self, max_length: int):
        super().crop(max_length)
        self._rebuild_rows()

    def batch_split(self, full_batch_size: int, split_size: int):
        raise NotImplementedError(
            "DropKVCache does not support batch_split (beam search). "
            "Use DynamicCache for beam search or implement DropKV-aware splitting.")

    @classmethod
    def from_batch_splits(cls, splits, **kwargs):
        raise NotImplementedError(
            "DropKVCache does not support from_batch_splits (beam search). "
            "Use DynamicCache for beam search or implement DropKV-aware merging.")

    # -- eviction ---------------------------------------------------------------
    def _keep_len(self, seq_len: int, total_tokens: Optional[int], max_keep_len: Optional[int]) -> int:
        """dropkv_cache.py:470-473."""
        base = total_tokens if total_tokens is not None else seq_len
        kl = min(seq_len, max(int(self.keep_ratio * base), self.window_size, 1))
        if max_keep_len is not None:
            kl = min(kl, max_keep_len)
        return kl

    def _check_heads(self, query_states, key_states):
        hq, hkv = query_states.shape[1], key_states.shape[1]
        if hq % hkv != 0:
            raise ValueError(f"Query heads {hq} must be divisible by KV heads {hkv}")

    def _compute_keep_indices(self, query_states: torch.Tensor, key_states: torch.Tensor,
                              value_states: torch.Tensor, total_tokens: Optional[int] = None,
                              max_keep_len: Optional[int] = None) -> torch.Tensor:
        """Sorted kept positions [B, Hkv, keep_len] int64 (dropkv_cache.py:355-477)."""
        self._check_heads(query_states, key_states)
        seq_len = key_states.shape[2]
        W = min(self.window_size, query_states.shape[2])
        sc = ops.scores(query_states, key_states.contiguous(), value_states.contiguous(), W)
        kl = self._keep_len(seq_len, total_tokens, max_keep_len)
        return ops.select_keep_indices(sc, self.kernel_size, self.window_size, kl)

    @staticmethod
    def _gather_compressed(key_states: torch.Tensor, value_states: torch.Tensor,
                           keep_idx: torch.Tensor):
        """dropkv_cache.py:479-491."""
        return ops.gather_compressed(key_states, value_states, keep_idx)

    def _evict_keep_len(self, seq_len: int) -> int:
        total = self._seen_tokens if self._evict_use_seen_tokens else None
        return self._keep_len(seq_len, total, self._budget_max_kv_tokens)

    def _store_new(self, key_states, value_states):
        """A layer's first K/V, kept without eviction."""
        if self.storage == "buffer":
            rows = _LayerRows(key_states)
            rows.append(key_states, value_states)
            self._rows.append(rows)
            key_states, value_states = rows.views()
        self.key_cache.append(key_states)
        self.value_cache.append(value_states)

    def _update_rows(self, query_states, key_states, value_states, layer_idx):
        """The continuation branches of update (dropkv_cache.py:576-622) over row
        buffers: same decisions, same kept rows, no concatenation."""
        rows = self._rows[layer_idx]
        mode = self._prefill_mode
        if mode not in _VALID_MODES:
            raise ValueError(f"Invalid _prefill_mode {mode!r} in decode path")
        rows.append(key_states, value_states)
        full_k, full_v = rows.views()
        if mode == "evict_accumulated" and query_states is not None and rows.n >= self.window_size:
            self._check_heads(query_states, full_k)
            W = min(self.window_size, query_states.shape[2])
            rows.evict(query_states, W, self.kernel_size, self._evict_keep_len(rows.n), self.window_size)
        self.key_cache[layer_idx], self.value_cache[layer_idx] = rows.views()
        return full_k, full_v

    def _evict(self, query_states, key_states, value_states):
        """Fused _compute_keep_indices + _gather_compressed: one C-ABI call."""
        self._check_heads(query_states, key_states)
        kl = self._evict_keep_len(key_states.shape[2])
        W = min(self.window_size, query_states.shape[2])
        _, kc, vc = ops.compress(query_states, key_states, value_states, W, self.kernel_size, kl,
                                 protect_window=self.window_size)
        return kc, vc

    # -- state machine (dropkv_cache.py:493-622) --------------------------------
    def update(self, query_states, key_states, value_states, layer_idx, cache_kwargs: Optional[dict[str, Any]] = None):
        # HF calls update(key, value, layer_idx, cache_kwargs): shift the arguments.
        if isinstance(value_states, int) and isinstance(layer_idx, dict):
            cache_kwargs = layer_idx
            layer_idx = value_states
            value_states = key_states
            key_states = query_states
            query_states = cache_kwargs.get("query_states") if cache_kwargs else None
            if query_states is None:
                logger.warning(
                    "DropKVCache.update() called without query_states — eviction disabled for this "
                    "layer. Patch your transformers to pass query_states in cache_kwargs.")

        if layer_idx == 0:
            self._seen_tokens += key_states.shape[-2]

        n_layers = len(self.key_cache)
        if n_layers < layer_idx:
            raise ValueError("Use DynamicCache.")

        if n_layers == layer_idx:  # first time this layer is seen: prefill
            if query_states is None:
                if self._prefill_mode != "single_pass":
                    logger.warning("query_states is None at layer %d — storing full KV without eviction.", layer_idx)
                self._store_new(key_states, value_states)
                return key_states, value_states
            if self._prefill_mode not in _VALID_MODES:
                raise ValueError(f"Invalid _prefill_mode: {self._prefill_mode!r}")
            if self._prefill_mode == "accumulate" or key_states.shape[2] < self.window_size:
                self._store_new(key_states, value_states)
                return key_states, value_states
            if self.storage == "buffer":
                rows = _LayerRows(key_states)
                kl = self._evict_keep_len(key_states.shape[2])
                W = min(self.window_size, query_states.shape[2])
                self._check_heads(query_states, key_states)
                rows.load_evicted(query_states, key_states.contiguous(), value_states.contiguous(), W,
                                  self.kernel_size, kl, self.window_size)
                self._rows.append(rows)
                kv, vv = rows.views()
                self.key_cache.append(kv)
                self.value_cache.append(vv)
                return key_states, value_states
            kc, vc = self._evict(query_states, key_states, value_states)
            self.key_cache.append(kc)
            self.value_cache.append(vc)
            return key_states, value_states
        if self.storage == "buffer":
            return self._update_rows(query_states, key_states, value_states, layer_idx)

        # continuation: decode or chunked prefill
        mode = self._prefill_mode
        if mode == "accumulate" or mode == "single_pass":
            self.key_cache[layer_idx] = torch.cat([self.key_cache[layer_idx], key_states], dim=-2)
            self.value_cache[layer_idx] = torch.cat([self.value_cache[layer_idx], value_states], dim=-2)
            return self.key_cache[layer_idx], self.value_cache[layer_idx]
        if mode == "evict_accumulated":
            full_k = torch.cat([self.key_cache[layer_idx], key_states], dim=-2)
            full_v = torch.cat([self.value_cache[layer_idx], value_states], dim=-2)
            if query_states is not None and full_k.shape[2] >= self.window_size:
                kc, vc = self._evict(query_states, full_k, full_v)
                self.key_cache[layer_idx] = kc
                self.value_cache[layer_idx] = vc
            else:
                self.key_cache[layer_idx] = full_k
                self.value_cache[layer_idx] = full_v
            return full_k, full_v
        raise ValueError(f"Invalid _prefill_mode {mode!r} in decode path")

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        """Logical length (tokens seen), used for RoPE positions after eviction."""
        if len(self.key_cache) <= layer_idx:
            return 0
        return self._seen_tokens

    def get_mask_sizes(self, cache_position: torch.Tensor, layer_idx: int = 0) -> tuple[int, int]:
        """(stored KV length + query length, 0): the mask must match stored tensors."""
        q = cache_position.shape[0]
        empty = len(self.key_cache) <= layer_idx or not self.key_cache[layer_idx].numel()
        stored = 0 if empty else self.key_cache[layer_idx].shape[-2]
        return stored + q, 0


def prefill_chunked(model, input_ids, cache, chunk_size=4096, evict_strategy="last_chunk",
                    max_kv_tokens=32768, **forward_kwargs):
    """Chunked prefill with DropKV eviction (dropkv_cache.py:651-807).

    ``evict_strategy``: ``"last_chunk"`` (accumulate, evict on the last chunk),
    ``"budget"`` (evict to keep_ratio * tokens seen whenever the stored KV would
    exceed ``max_kv_tokens``, which also caps keep_len) or ``"every_chunk"``.
    On any exception the cache is cleared; its mode flags are always restored.
    """
    if not isinstance(cache, DropKVCache):
        raise TypeError(f"cache must be DropKVCache, got {type(cache).__name__}")
    if len(cache.key_cache) > 0:
        raise ValueError("prefill_chunked() requires a fresh (empty) cache. Create a new DropKVCache instance.")
    if chunk_size < cache.window_size:
        raise ValueError(f"chunk_size ({chunk_size}) must be >= window_size ({cache.window_size})")
    bad = {"attention_mask", "position_ids", "cache_position"} & forward_kwargs.keys()
    if bad:
        raise ValueError(
            f"prefill_chunked() does not support sequence-shaped kwargs {bad} — the model computes "
            f"these internally per chunk. Remove them from forward_kwargs.")
    strategies = ("last_chunk", "budget", "every_chunk")
    if evict_strategy not in strategies:
        raise ValueError(f"evict_strategy must be one of {strategies}, got {evict_strategy!r}")
    if evict_strategy == "budget":
        if max_kv_tokens is None:
            raise ValueError("max_kv_tokens is required when evict_strategy='budget'")
        if max_kv_tokens < cache.window_size:
            raise ValueError(
                f"max_kv_tokens ({max_kv_tokens}) must be >= window_size ({cache.window_size}) "
                f"to preserve protected tail tokens")

    B, L = input_ids.shape
    if L <= chunk_size and evict_strategy == "last_chunk":
        with torch.no_grad():
            return model(input_ids, past_key_values=cache, use_cache=True, **forward_kwargs)

    starts = list(range(0, L, chunk_size))
    try:
        cache._evict_use_seen_tokens = evict_strategy in ("budget", "every_chunk")
        if evict_strategy == "budget":
            cache._budget_max_kv_tokens = max_kv_tokens
        with torch.no_grad():
            output = None
            for i, start in enumerate(starts):
                end = min(start + chunk_size, L)
                last = i == len(starts) - 1
                if evict_strategy == "last_chunk":
                    cache._prefill_mode = "evict_accumulated" if last else "accumulate"
                elif evict_strategy == "every_chunk":
                    cache._prefill_mode = "single_pass" if i == 0 else "evict_accumulated"
                else:  # budget
                    if last:
                        cache._prefill_mode = "evict_accumulated"
                    else:
                        stored = cache.key_cache[0].shape[2] if cache.key_cache else 0
                        cache._prefill_mode = ("evict_accumulated" if stored + (end - start) > max_kv_tokens
                                               else "accumulate")
                output = model(input_ids[:, start:end], past_key_values=cache, use_cache=True,
                               **forward_kwargs)
            return output
    except BaseException:
        cache.key_cache.clear()
        cache.value_cache.clear()
        cache._rows.clear()
        cache._seen_tokens = 0
        raise
    finally:
        cache._prefill_mode = "single_pass"
        cache._evict_use_seen_tokens = False
        cache._budget_max_kv_tokens = None
