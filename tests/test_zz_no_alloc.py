"""dropkv_scores_static -- the scoring call whose scratch is a static device
buffer inside the library -- against dropkv_scores with a caller workspace.

It exists for callers that cannot allocate device memory while they score (an
engine that reserved all of its memory up front, a thread that must not enter an
allocator).  The tests check that it gives the workspace entry's scores, that its
device status word (read through dropkv_scores_static_status) stays zero, and
that a warm call allocates nothing: neither torch's caching allocator nor the
device's free memory moves across it.

This file is collected last on purpose: the static entry must give the same
scores in a fresh process (first call looks the buffer up) and after every other
test has run in the same process.
"""

import pytest
import torch

from dropkv_b200 import _lib, ops
from dropkv_b200.workloads import Workload, llama_layer, make_qkv
from parity import assert_scores_close

STATIC_BYTES = 16 << 20
DT = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}
RND = {torch.float32: _lib.ROUND_NONE, torch.float16: _lib.ROUND_F16, torch.bfloat16: _lib.ROUND_BF16}
# same kernels as the workspace entry: the bf16/fp16 kernel tolerance of the parity tests
TOL = {torch.float32: (1e-5, 1e-6), torch.float16: (1e-3, 1e-4), torch.bfloat16: (1e-3, 1e-4)}


def _call_static(Q, K, V, window, round_p, out, stream=None):
    B, Hq, Lq, D = Q.shape
    _, Hkv, Lk, _ = K.shape
    st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    return _lib.load().dropkv_scores_static(
        Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(), DT[Q.dtype], B, Hq, Hkv, Lk, D,
        int(window), 1e-6, RND[Q.dtype] if round_p else _lib.ROUND_NONE, out.data_ptr(), st)


def _static_status(Q, K, window):
    """The status word of the last static call for this problem (0 = no wait timed out)."""
    B, Hq, Lq, D = Q.shape
    _, Hkv, Lk, _ = K.shape
    st = torch.zeros(1, dtype=torch.int32, device=Q.device)
    _lib.check(_lib.load().dropkv_scores_static_status(DT[Q.dtype], B, Hq, Hkv, Lk, D, int(window),
                                                       st.data_ptr(), torch.cuda.current_stream().cuda_stream),
               "dropkv_scores_static_status")
    return int(st.item())


CASES = [
    ("llama_32k_bf16", llama_layer(32768)),                                              # tensor-core scorer
    ("qwen_d64_bf16", Workload(B=1, Hq=14, Hkv=2, D=64, Lq=64, Lk=20000, seed=11)),      # M = 56
    ("fp16_mha", Workload(B=2, Hq=8, Hkv=8, D=128, Lq=16, Lk=4096, dtype=torch.float16, seed=12)),
    ("fp32_simt", Workload(B=1, Hq=32, Hkv=8, D=128, Lq=64, Lk=3000, dtype=torch.float32, seed=13)),
]


@pytest.mark.gpu
@pytest.mark.parametrize("name,wl", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("round_p", [False, True])
def test_static_scratch_matches_workspace_entry(name, wl, round_p):
    Q, K, V = make_qkv(wl, "cuda")
    W = wl.window_size
    assert _lib.load().dropkv_scores_workspace_size(wl.B, wl.Hq, wl.Hkv, wl.Lk, wl.D, W) <= STATIC_BYTES
    want = ops.scores(Q, K, V, W, round_p=round_p).cpu().numpy()
    for call in range(2):  # two calls in a row reuse the same static buffer
        out = torch.full((wl.B, wl.Hkv, wl.Lk), float("nan"), device="cuda")
        _lib.check(_call_static(Q, K, V, W, round_p, out), "dropkv_scores_static")
        assert _static_status(Q, K, W) == 0, f"{name} call {call}: a bounded wait timed out"
        torch.cuda.synchronize()
        assert_scores_close(out.cpu().numpy(), want, *TOL[wl.dtype], what=f"{name} call {call}")


@pytest.mark.gpu
def test_static_scratch_headline_layer_two_calls():
    """The 128K-token Llama layer fits the static buffer."""
    wl = llama_layer(131072)
    Q, K, V = make_qkv(wl, "cuda")
    want = ops.dropkv_scores_cuda(Q, K, V).cpu().numpy()
    outs = [torch.empty(1, 8, 131072, device="cuda") for _ in range(2)]
    for o in outs:
        _lib.check(_call_static(Q, K, V, 8, True, o), "dropkv_scores_static")
        assert _static_status(Q, K, 8) == 0
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert_scores_close(o.cpu().numpy(), want, *TOL[torch.bfloat16], what=f"128K call {i}")


@pytest.mark.gpu
@pytest.mark.parametrize("name,wl", [CASES[0], CASES[3]], ids=[CASES[0][0], CASES[3][0]])
def test_static_scratch_allocates_nothing(name, wl):
    """A warm static call leaves torch's allocator counters and the device's free
    memory unchanged (the first call may load kernels; it runs before the check)."""
    Q, K, V = make_qkv(wl, "cuda")
    out = torch.empty(wl.B, wl.Hkv, wl.Lk, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    args = (DT[wl.dtype], wl.B, wl.Hq, wl.Hkv, wl.Lk, wl.D, wl.window_size)
    _lib.check(_call_static(Q, K, V, wl.window_size, True, out), "dropkv_scores_static")  # warm-up
    _lib.check(lib.dropkv_scores_static_status(*args, status.data_ptr(), st), "status")
    torch.cuda.synchronize()
    keys = ("allocation.all.allocated", "segment.all.allocated", "reserved_bytes.all.current")
    stats0 = {k: torch.cuda.memory_stats().get(k, 0) for k in keys}
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        _lib.check(_call_static(Q, K, V, wl.window_size, True, out), "dropkv_scores_static")
        _lib.check(lib.dropkv_scores_static_status(*args, status.data_ptr(), st), "status")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    stats1 = {k: torch.cuda.memory_stats().get(k, 0) for k in keys}
    assert stats1 == stats0, f"torch allocator moved: {stats0} -> {stats1}"
    assert free1 == free0, f"device free memory moved: {free0} -> {free1}"
    assert int(status.item()) == 0


def test_static_scratch_rejects_oversized_problem():
    """Eight 128K sequences need ~80 MB of partials: refused before any launch
    (argument checks only read the shapes, so this runs without a GPU)."""
    lib = _lib.load()
    before = lib.dropkv_launch_count()
    fake = 1 << 20  # never dereferenced: the call fails its size check first
    rc = lib.dropkv_scores_static(fake, 0, 0, 0, 0, 8, fake, fake, _lib.DTYPE_BF16, 8, 32, 8, 131072, 128,
                                  8, 1e-6, _lib.ROUND_BF16, fake, None)
    assert rc == _lib.ERR_WORKSPACE
    msg = lib.dropkv_last_error().decode()
    assert "static buffer" in msg and str(STATIC_BYTES) in msg
    assert lib.dropkv_launch_count() == before
