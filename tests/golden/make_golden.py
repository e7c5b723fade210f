"""Generate the golden fixtures for the eviction path from the reference itself.

Run in a container where the reference checkout is present (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/DropKV

For every case it regenerates the seeded inputs with
``dropkv_b200.workloads.make_qkv`` (CPU generator, bit-reproducible for a given
torch build), runs the reference's own functions on them and stores the outputs:

* ``scores_exact`` -- ``dropkv_scores_reference(..., match_pytorch_precision=False)``
  (dropkv_triton.py:29-109)
* ``scores_round`` -- the same with ``match_pytorch_precision=True`` (p rounded to
  the input dtype, dropkv_triton.py:88-92)
* ``keep_idx_cache`` -- ``DropKVCache(use_triton=False)._compute_keep_indices`` on the
  same inputs (dropkv_cache.py:355-477, the reference's PyTorch eviction path)
* ``kc_sum`` / ``vc_sum`` -- float64 sums of ``_gather_compressed`` outputs
  (dropkv_cache.py:479-491) as a compact check of the gather.
* ``keep_idx_round`` / ``keep_idx_exact`` -- the reference's own selection
  (``_compute_keep_indices`` with ``use_triton=True``: max_pool1d, protection,
  topk, sort, dropkv_cache.py:462-477) applied to the scores of
  ``dropkv_scores_reference`` with and without p rounded to the input dtype, i.e.
  the kept sets the reference's Triton branch produces when its kernel returns
  the reference formula's values (its tests hold the kernel to that function,
  tests/test_dropkv_triton.py:122-137).  The scorer is put in place of
  ``dropkv_scores_triton`` for the call, since the Triton kernel needs a GPU.
  Where attention saturates (p ~ 1 in some window row) these sets and
  ``keep_idx_cache`` differ: the score there is fp32 cancellation noise, and
  each of the reference's paths keeps or evicts such a key by the sign of its
  own noise.

Inputs are not stored; their SHA-256 is, so a test can detect generator drift.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from dropkv_b200.workloads import Workload, make_qkv  # noqa: E402

# name -> (Workload, keep_ratio for the cache path)
CASES = {
    "cfg1_fp32_heavy": Workload(B=1, Hq=8, Hkv=2, D=64, Lq=64, Lk=1024, dtype=torch.float32,
                                dist="heavy", seed=1, extra={"n_heavy": 4, "boost": 3.0}),
    "llama_small_bf16": Workload(B=1, Hq=8, Hkv=2, D=128, Lq=256, Lk=256, dtype=torch.bfloat16,
                                 keep_ratio=0.3, seed=11),
    "qwen_m56_bf16_lq64": Workload(B=1, Hq=14, Hkv=2, D=64, Lq=64, Lk=512, dtype=torch.bfloat16,
                                   keep_ratio=0.1, seed=12),
    "mha_bf16": Workload(B=1, Hq=4, Hkv=4, D=128, Lq=128, Lk=128, dtype=torch.bfloat16,
                         keep_ratio=0.3, seed=13),
    "w65_bf16": Workload(B=1, Hq=4, Hkv=2, D=128, Lq=1344, Lk=1344, dtype=torch.bfloat16,
                         window_size=65, keep_ratio=0.1, seed=14),
    "l_eq_w_bf16": Workload(B=1, Hq=8, Hkv=2, D=128, Lq=8, Lk=8, dtype=torch.bfloat16,
                            keep_ratio=0.5, seed=15),
    "l100_bf16": Workload(B=1, Hq=8, Hkv=2, D=128, Lq=100, Lk=100, dtype=torch.bfloat16,
                          keep_ratio=0.3, seed=16),
    "batch2_bf16": Workload(B=2, Hq=8, Hkv=2, D=64, Lq=64, Lk=384, dtype=torch.bfloat16,
                            keep_ratio=0.25, seed=17),
    "fp16_small": Workload(B=1, Hq=8, Hkv=2, D=64, Lq=32, Lk=640, dtype=torch.float16,
                           keep_ratio=0.2, seed=18),
    "sink_bf16_4k": Workload(B=1, Hq=32, Hkv=8, D=128, Lq=8, Lk=4096, dtype=torch.bfloat16,
                             keep_ratio=0.1, dist="llama_sink", seed=19,
                             extra={"n_outlier": 2, "outlier_scale": 8.0, "sink_alpha": 64.0}),
    "short_chunk_lq4_bf16": Workload(B=1, Hq=8, Hkv=2, D=128, Lq=4, Lk=256, dtype=torch.bfloat16,
                                     keep_ratio=0.3, seed=20),
}


def input_digest(Q, K, V) -> str:
    h = hashlib.sha256()
    for t in (Q, K, V):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def workload_to_json(wl: Workload) -> str:
    d = dict(B=wl.B, Hq=wl.Hq, Hkv=wl.Hkv, D=wl.D, Lq=wl.Lq, Lk=wl.Lk,
             dtype=str(wl.dtype).replace("torch.", ""), window_size=wl.window_size,
             kernel_size=wl.kernel_size, keep_ratio=wl.keep_ratio, dist=wl.dist,
             seed=wl.seed, extra=wl.extra)
    return json.dumps(d, sort_keys=True)


def workload_from_json(s: str) -> Workload:
    d = json.loads(s)
    d["dtype"] = getattr(torch, d["dtype"])
    return Workload(**d)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DROPKV_REFERENCE", ""),
                    help="path of the reference checkout (contains dropkv_triton.py)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if not args.reference or not os.path.isfile(os.path.join(args.reference, "dropkv_triton.py")):
        raise SystemExit("pass --reference <checkout of the reference>")
    sys.path.insert(0, args.reference)
    import dropkv_cache  # noqa: E402  (reference module)
    import dropkv_triton  # noqa: E402  (reference module)

    torch.manual_seed(0)
    for name, wl in CASES.items():
        Q, K, V = make_qkv(wl, "cpu")
        W = wl.window_size
        rec = {"workload": workload_to_json(wl), "digest": input_digest(Q, K, V)}
        if wl.Lq >= W:
            s_exact = dropkv_triton.dropkv_scores_reference(Q, K, V, window_size=W,
                                                            match_pytorch_precision=False)
            s_round = dropkv_triton.dropkv_scores_reference(Q, K, V, window_size=W,
                                                            match_pytorch_precision=True)
            rec["scores_exact"] = s_exact.numpy()
            rec["scores_round"] = s_round.numpy()
        cache = dropkv_cache.DropKVCache(keep_ratio=wl.keep_ratio, window_size=W,
                                         kernel_size=wl.kernel_size, use_triton=False)
        idx = cache._compute_keep_indices(Q, K, V)
        if wl.Lq >= W:
            orig = dropkv_triton.dropkv_scores_triton
            for field, rnd in (("keep_idx_round", True), ("keep_idx_exact", False)):
                dropkv_triton.dropkv_scores_triton = (
                    lambda q, k, v, window_size=8, _r=rnd: dropkv_triton.dropkv_scores_reference(
                        q, k, v, window_size=window_size, match_pytorch_precision=_r))
                try:
                    sel = dropkv_cache.DropKVCache(keep_ratio=wl.keep_ratio, window_size=W,
                                                   kernel_size=wl.kernel_size, use_triton=True)
                    rec[field] = sel._compute_keep_indices(Q, K, V).numpy()
                finally:
                    dropkv_triton.dropkv_scores_triton = orig
        kc, vc = dropkv_cache.DropKVCache._gather_compressed(K, V, idx)
        rec["keep_idx_cache"] = idx.numpy()
        rec["kc_sum"] = np.float64(kc.double().sum().item())
        rec["vc_sum"] = np.float64(vc.double().sum().item())
        path = os.path.join(args.out, f"{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"{name}: wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
