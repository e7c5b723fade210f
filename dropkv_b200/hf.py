"""Transformers integration of the CUDA eviction path.

The reference ships this layer as a patch against Transformers
(patches/dropkv_transformers.patch); here it is a module that works with the
Transformers release installed beside this package (the layered ``Cache`` API of
5.x), with no edit to Transformers itself:

* ``DropKVLayer`` / ``DropKVCache``: the eviction cache of patch:59-264
  (``cache_utils.DropKVLayer``, ``cache_utils.DropKVCache``). At the first update
  that carries ``query_states`` a layer scores its keys, keeps the top
  ``keep_ratio`` fraction per KV head and stores the compacted K/V (one
  ``dropkv_compress`` call: scores -> max-pool -> protect -> top-k -> gather); it
  returns the full K/V for that step's attention. Later updates append.
* ``enable_query_states``: the query plumbing of patch:321-344 (Llama and Qwen2
  attention pass ``query_states`` in ``cache_kwargs``), installed on a model's
  attention modules at run time.
* ``register_attention``: an attention function (``attn_implementation="dropkv"``)
  that runs decode steps over the cache with ``dropkv_decode_attention`` and
  everything else with Transformers' SDPA path.
* ``make_cache`` / ``generate``: the generate wiring of patch:282-319
  (``cache_implementation="quantized", backend="DropKV"`` plus the DropKV keys in
  the generation kwargs).
"""

from __future__ import annotations

import logging
import sys
import types
from typing import Any, Optional

import torch

from . import ops

logger = logging.getLogger(__name__)

try:  # Transformers is optional for the rest of the package
    from transformers.cache_utils import Cache, DynamicLayer
except ImportError as _e:  # pragma: no cover - exercised only without transformers
    raise ImportError("dropkv_b200.hf needs the transformers package") from _e


class DropKVLayer(DynamicLayer):
    """One layer of the eviction cache (patch:59-233 ``DropKVLayer``).

    ``use_triton`` is accepted for drop-in compatibility; the CUDA library is the
    only backend. ``cumulative_length`` counts every token seen (the logical
    length RoPE positions come from), the stored K/V may be shorter.
    """

    def __init__(self, keep_ratio: float = 0.1, window_size: int = 8, kernel_size: int = 11,
                 use_triton: bool = True):
        super().__init__()
        if not 0 < keep_ratio <= 1.0:
            raise ValueError(f"keep_ratio must be in (0, 1], got {keep_ratio}")
        if window_size <= 0:
            raise ValueError(f"window_size must be positive, got {window_size}")
        if kernel_size < 1 or kernel_size % 2 == 0:
            raise ValueError(f"kernel_size must be a positive odd integer, got {kernel_size}")
        self.keep_ratio = keep_ratio
        self.window_size = window_size
        self.kernel_size = kernel_size
        self.use_triton = use_triton
        self._prefilled = False
        self.cumulative_length = 0
        self._warned_no_query = False
        self.timer: Optional[list] = None  # (start, end) CUDA events of each eviction when set

    def reset(self) -> None:
        super().reset()
        self._prefilled = False
        self._warned_no_query = False
        if self.is_initialized:
            self.keys = torch.tensor([], dtype=self.dtype, device=self.device)
            self.values = torch.tensor([], dtype=self.dtype, device=self.device)

    def crop(self, max_length: int) -> None:
        super().crop(max_length)
        self.cumulative_length = self._stored()

    def _stored(self) -> int:
        return 0 if (not self.is_initialized or self.keys.numel() == 0) else self.keys.shape[-2]

    def keep_len(self, seq_len: int) -> int:
        """Kept positions per KV head (patch:190; no cap at seq_len is needed
        because seq_len >= window_size and keep_ratio <= 1 here)."""
        return max(int(self.keep_ratio * seq_len), self.window_size, 1)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor,
               cache_kwargs: Optional[dict[str, Any]] = None) -> tuple[torch.Tensor, torch.Tensor]:
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.cumulative_length += key_states.shape[-2]
        query_states = cache_kwargs.get("query_states") if cache_kwargs is not None else None
        if query_states is None and not self._prefilled and not self._warned_no_query:
            self._warned_no_query = True
            logger.warning("DropKVLayer received no query_states in cache_kwargs; eviction will not occur. "
                           "Call dropkv_b200.hf.enable_query_states(model) first.")
        if not self._prefilled and query_states is not None:
            self._prefilled = True
            bsz, num_kv_heads, seq_len, head_dim = key_states.shape
            if seq_len < self.window_size:  # too short to score: keep everything
                self.keys, self.values = key_states, value_states
                return key_states, value_states
            if query_states.shape[1] % num_kv_heads != 0:
                raise ValueError(f"Query heads {query_states.shape[1]} must be divisible by KV heads {num_kv_heads}")
            keep = self.keep_len(seq_len)
            ev = None
            if self.timer is not None and key_states.is_cuda:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            _, kc, vc = ops.compress(query_states, key_states, value_states, self.window_size,
                                     self.kernel_size, keep)
            if ev is not None:
                ev[1].record()
                self.timer.append(ev)
            self.keys, self.values = kc, vc
            return key_states, value_states
        # decode / later chunks: append (once appended, a late query_states no longer evicts)
        self._prefilled = True
        self.keys = torch.cat([self.keys, key_states], dim=-2)
        self.values = torch.cat([self.values, value_states], dim=-2)
        return self.keys, self.values

    def get_seq_length(self) -> int:
        """The logical length (tokens seen), which RoPE positions follow."""
        return self.cumulative_length if self.is_initialized else 0

    def get_mask_sizes(self, query_length) -> tuple[int, int]:
        """(kv_length, kv_offset) of the STORED K/V plus the new tokens.
        Accepts the query length or, as older Transformers pass, cache_position."""
        q = query_length if isinstance(query_length, int) else int(query_length.shape[0])
        return self._stored() + q, 0


class DropKVCache(Cache):
    """KV cache with DropKV eviction at prefill (patch:236-264 ``DropKVCache``):
    one ``DropKVLayer`` per decoder layer of ``config``."""

    def __init__(self, config=None, keep_ratio: float = 0.1, window_size: int = 8, kernel_size: int = 11,
                 use_triton: bool = True, num_layers: Optional[int] = None):
        if config is not None:
            num_layers = config.get_text_config(decoder=True).num_hidden_layers
        if num_layers is None:
            raise ValueError("DropKVCache needs a model config or num_layers")
        layers = [DropKVLayer(keep_ratio=keep_ratio, window_size=window_size, kernel_size=kernel_size,
                              use_triton=use_triton) for _ in range(num_layers)]
        super().__init__(layers=layers)

    def record_timing(self, on: bool = True) -> None:
        """Record CUDA events around every eviction (see ``compression_ms``)."""
        for layer in self.layers:
            layer.timer = [] if on else None

    def compression_ms(self) -> float:
        """Device time of the evictions recorded so far, summed over layers
        (synchronises on the recorded events)."""
        total = 0.0
        for layer in self.layers:
            for a, b in (layer.timer or []):
                b.synchronize()
                total += a.elapsed_time(b)
        return total


# ---------------------------------------------------------------------------
# query_states plumbing (patch:321-344)
# ---------------------------------------------------------------------------
def _attention_forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None, **kwargs):
    """Llama / Qwen2 decoder attention that also hands ``query_states`` to the
    cache (the one line patch:330 and patch:343 change), otherwise the same
    projections, RoPE, cache update and attention call as the installed model."""
    input_shape = hidden_states.shape[:-1]
    hidden_shape = (*input_shape, -1, self.head_dim)
    query_states = self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    key_states = self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    value_states = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    cos, sin = position_embeddings
    query_states, key_states = self._dropkv_rope(query_states, key_states, cos, sin)
    if past_key_values is not None:
        cache_kwargs = {"sin": sin, "cos": cos, "query_states": query_states}
        key_states, value_states = past_key_values.update(key_states, value_states, self.layer_idx, cache_kwargs)
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    attention_interface = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation,
                                                                self._dropkv_eager)
    attn_output, attn_weights = attention_interface(
        self, query_states, key_states, value_states, attention_mask,
        dropout=0.0 if not self.training else self.attention_dropout, scaling=self.scaling,
        sliding_window=getattr(self, "sliding_window", None), **kwargs)
    attn_output = attn_output.reshape(*input_shape, -1).contiguous()
    return self.o_proj(attn_output), attn_weights


def enable_query_states(model) -> int:
    """Make every Llama/Qwen2-style attention module of ``model`` pass its query
    states to the cache. Returns the number of modules changed."""
    n = 0
    for m in model.modules():
        if not all(hasattr(m, a) for a in ("q_proj", "k_proj", "v_proj", "o_proj", "layer_idx", "head_dim")):
            continue
        mod = sys.modules[type(m).__module__]
        rope = getattr(mod, "apply_rotary_pos_emb", None)
        eager = getattr(mod, "eager_attention_forward", None)
        if rope is None or eager is None:
            continue
        m._dropkv_rope = rope
        m._dropkv_eager = eager
        m.forward = types.MethodType(_attention_forward, m)
        n += 1
    return n


# ---------------------------------------------------------------------------
# attention over the compressed cache
# ---------------------------------------------------------------------------
def dropkv_attention_forward(module, query, key, value, attention_mask, dropout: float = 0.0,
                             scaling: Optional[float] = None, is_causal: Optional[bool] = None, **kwargs):
    """Decode steps (at most 8 new query rows, no padding mask, bf16/fp16,
    head_dim 64 or 128) attend over the cache with ``dropkv_decode_attention``;
    every other call goes to Transformers' SDPA attention. Returns
    ([B, Lq, Hq, D], None) as Transformers' attention functions do."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    Lq, L, D = query.shape[2], key.shape[2], query.shape[3]
    if (query.is_cuda and attention_mask is None and dropout == 0.0 and 1 <= Lq <= 8 and Lq < L
            and query.dtype in (torch.bfloat16, torch.float16) and key.dtype == query.dtype and D in (64, 128)
            and key.stride(3) == 1 and key.stride(2) == D and key.stride() == value.stride()):
        out = ops.decode_attention(query, key, value, scale=scaling)
        return out.transpose(1, 2).contiguous(), None
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  is_causal=is_causal, **kwargs)


def register_attention(name: str = "dropkv") -> str:
    """Register ``dropkv_attention_forward`` (and SDPA's mask builder) under
    ``name`` for ``attn_implementation``."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register(name, dropkv_attention_forward)
    AttentionMaskInterface.register(name, sdpa_mask)
    return name


# ---------------------------------------------------------------------------
# generate wiring (patch:282-319)
# ---------------------------------------------------------------------------
_DROPKV_KEYS = ("backend", "keep_ratio", "window_size", "kernel_size", "use_triton")


def make_cache(config, **cache_config) -> DropKVCache:
    """A ``DropKVCache`` from generation-style settings, parsed as patch:1892-1905
    does: numbers may be strings, ``use_triton`` "0"/"false"/"no" means off."""
    cache_config = dict(cache_config)
    backend = cache_config.pop("backend", "DropKV")
    if backend != "DropKV":
        raise ValueError(f"backend must be 'DropKV', got {backend!r}")
    use_triton = cache_config.pop("use_triton", "1")
    if isinstance(use_triton, str):
        use_triton = use_triton.lower() not in ("0", "false", "no")
    return DropKVCache(config=config,
                       keep_ratio=float(cache_config.pop("keep_ratio", 0.1)),
                       window_size=int(cache_config.pop("window_size", 8)),
                       kernel_size=int(cache_config.pop("kernel_size", 11)),
                       use_triton=bool(use_triton))


def generate(model, input_ids, **kwargs):
    """``model.generate`` with a DropKV cache: the DropKV keys (backend,
    keep_ratio, window_size, kernel_size, use_triton) are taken out of the
    generation kwargs (patch:2368-2374), the cache is built from them and the
    model's attention modules pass their query states."""
    dropkv = {k: kwargs.pop(k) for k in _DROPKV_KEYS if k in kwargs}
    kwargs.pop("cache_implementation", None)
    enable_query_states(model)
    cache = make_cache(model.config, **dropkv)
    return model.generate(input_ids, past_key_values=cache, **kwargs)
