"""dropkv_b200: B200-native (sm_100a) DropKV prefill eviction path.

Public API (the reference's names and semantics):

* ``dropkv_scores_cuda(Q, K, V, window_size=8, eps=1e-6, allow_tf32=True,
  match_pytorch_precision=True)`` -- drop-in for ``dropkv_scores_triton``; also
  exported under that name.
* ``DropKVCache(keep_ratio=0.1, window_size=8, kernel_size=11, use_triton=True)``
  and ``prefill_chunked(model, input_ids, cache, ...)``.
* ``compress`` / ``scores`` / ``select_keep_indices`` / ``gather_compressed``:
  the stages as tensor functions over the C ABI (include/dropkv_b200.h);
  ``Compressor`` (pre-planned, allocation-free calls) and ``HostPipeline``
  (host-resident layers with overlapped copies).
* ``compress_varlen`` / ``VarlenCompressor``: a ragged batch of sequences in one
  call, keep_len per sequence evaluated on the device (total_tokens /
  max_keep_len per sequence).
* ``dropkv_b200.hf`` (imported on demand, needs transformers): the
  Transformers integration -- ``DropKVCache(config, ...)``, query-state
  plumbing, decode attention over the compressed cache, generate wiring.
"""

from ._lib import DropKVError, version
from .cache import DropKVCache, prefill_chunked
from .ops import (Compressor, HostPipeline, VarlenCompressor, compress, compress_varlen, decode_append_attention,
                  decode_attention, dropkv_scores_cuda, gather_compressed, scores, select_keep_indices)

# Name of the reference entry point (dropkv_triton.py:643) for drop-in imports.
dropkv_scores_triton = dropkv_scores_cuda

__all__ = [
    "DropKVCache", "prefill_chunked", "DropKVError", "version",
    "compress", "decode_attention", "decode_append_attention", "dropkv_scores_cuda", "dropkv_scores_triton", "gather_compressed",
    "scores", "select_keep_indices", "Compressor", "HostPipeline", "VarlenCompressor", "compress_varlen",
]
