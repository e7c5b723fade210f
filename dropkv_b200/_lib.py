"""ctypes binding of libdropkv_b200.so (the C ABI declared in include/dropkv_b200.h).

The library is the only compute path of this package: if it is missing the
first call raises, there is no Python or CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdropkv_b200.so")

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
ROUND_NONE, ROUND_BF16, ROUND_F16 = 0, 1, 2
OK, ERR_ARG, ERR_WORKSPACE, ERR_CUDA, ERR_UNSUPPORTED, ERR_DEVICE = range(6)

_c_int, _c_i64, _c_f, _c_sz, _c_p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p

VARLEN_MAX_SEQS = 32


class VarlenSeq(ctypes.Structure):
    """``dropkv_varlen_seq``: one sequence of a ragged batch (include/dropkv_b200.h)."""
    _fields_ = [("q", _c_p), ("q_sb", _c_i64), ("q_sh", _c_i64), ("q_ss", _c_i64), ("q_sd", _c_i64),
                ("Lq", _c_int), ("B", _c_int), ("Lk", _c_int), ("cap", _c_int),
                ("k", _c_p), ("v", _c_p), ("keep_idx", _c_p), ("k_out", _c_p), ("v_out", _c_p)]


# name -> (restype, argtypes)
SIGNATURES = {
    "dropkv_version": (ctypes.c_char_p, []),
    "dropkv_last_error": (ctypes.c_char_p, []),
    "dropkv_launch_count": (ctypes.c_uint64, []),
    "dropkv_scores_workspace_size": (_c_sz, [_c_int] * 6),
    "dropkv_scores": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_int,
                               _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _c_int, _c_p,
                               _c_p, _c_sz, _c_p]),
    "dropkv_scores_static": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_int,
                                      _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _c_int,
                                      _c_p, _c_p]),
    "dropkv_scores_static_status": (_c_int, [_c_int] * 7 + [_c_p, _c_p]),
    "dropkv_scorer_for": (_c_int, [_c_int] * 7),
    "dropkv_set_scorer": (_c_int, [_c_int]),
    "dropkv_test_scorer_waits": (_c_int, [ctypes.c_uint64, _c_int]),
    "dropkv_scores_status_offset": (_c_sz, [_c_int] * 7),
    "dropkv_selftest_tcgen05": (_c_int, [_c_int, _c_p, _c_p, _c_int, _c_p, _c_p, _c_p]),
    "dropkv_select_workspace_size": (_c_sz, [_c_int] * 3),
    "dropkv_select": (_c_int, [_c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p, _c_p,
                               _c_sz, _c_p]),
    "dropkv_gather": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p, _c_int,
                               _c_p, _c_p, _c_p]),
    "dropkv_compress_workspace_size": (_c_sz, [_c_int] * 6),
    "dropkv_compress_strided": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_i64,
                                         _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f,
                                         _c_int, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_i64,
                                         _c_p, _c_sz, _c_p]),
    "dropkv_append_rows": (_c_int, [_c_p, _c_p, _c_i64, _c_int, _c_p, _c_p, _c_i64, _c_int, _c_int, _c_int,
                                    _c_int, _c_p]),
    "dropkv_decode_attention_workspace_size": (_c_sz, [_c_int] * 6),
    "dropkv_decode_attention": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_i64,
                                         _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _c_p,
                                         _c_p, _c_sz, _c_p]),
    "dropkv_compress": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_int,
                                 _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _c_int,
                                 _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p, _c_sz,
                                 _c_p]),
    "dropkv_decode_append_attention": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_i64,
                                                _c_i64, _c_int, _c_p, _c_p, _c_i64, _c_i64, _c_int, _c_int, _c_int,
                                                _c_int, _c_int, _c_int, _c_f, _c_p, _c_p, _c_sz, _c_p]),
    "dropkv_compress_kv_strides": (_c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_i64,
                                            _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                            _c_f, _c_int, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p,
                                            _c_sz, _c_p]),
    "dropkv_compress_varlen_workspace_size": (_c_sz, [_c_int, ctypes.POINTER(VarlenSeq), _c_int, _c_int, _c_int,
                                                      _c_int]),
    "dropkv_compress_varlen": (_c_int, [_c_int, ctypes.POINTER(VarlenSeq), _c_int, _c_int, _c_int, _c_int, _c_int,
                                        _c_f, _c_int, _c_int, _c_int, ctypes.c_double, _c_int, _c_p, _c_p, _c_p,
                                        _c_p, _c_sz, _c_p]),
}


class DropKVError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[dropkv_b200 status {code}] {message}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"dropkv_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -m dropkv_b200.build` (there is no fallback path)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != OK:
        msg = load().dropkv_last_error().decode(errors="replace")
        raise DropKVError(rc, f"{what}: {msg}" if what else msg)


SCORER_AUTO, SCORER_CUDA_CORES, SCORER_TENSOR_CORES = 0, 1, 2
NO_STATUS = ctypes.c_size_t(-1).value


scorer_mode = SCORER_AUTO  # the mode last set through set_scorer (keys cached per-shape plans)


def set_scorer(mode: int) -> None:
    """Process-wide scorer choice (0 auto, 1 CUDA cores, 2 tensor cores)."""
    global scorer_mode
    check(load().dropkv_set_scorer(int(mode)), "dropkv_set_scorer")
    scorer_mode = int(mode)


def launch_count() -> int:
    """Kernel launches issued by the library so far in this process."""
    return int(load().dropkv_launch_count())


def version() -> str:
    return load().dropkv_version().decode()
