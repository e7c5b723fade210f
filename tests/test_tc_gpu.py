"""The tensor-core scorer: hardware self-test of its MMA building blocks, and
parity of the fused tcgen05 kernel with the CUDA-core kernels and the oracle."""

import numpy as np
import pytest
import torch

from dropkv_b200 import _lib, ops
from dropkv_b200.workloads import Workload, llama_layer, make_qkv
from oracle import dropkv_oracle as O
from parity import assert_scores_close, well_conditioned

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4, 5])
@pytest.mark.parametrize("n", [16, 32, 64, 128])
def test_tcgen05_selftest(mode, n):
    if mode == 4 and n == 128:
        pytest.skip("MN-major B rows hold at most 64 elements")
    if mode == 5 and n == 16:
        pytest.skip("two MN-major atoms need n >= 32")
    D = 64 if mode in (2, 3) else 128
    g = torch.Generator().manual_seed(mode * 1000 + n)
    A = torch.randn(128, D, generator=g).to(torch.bfloat16)
    kb = D if mode in (0, 2) else 128
    Bm = torch.randn(n, kb, generator=g).to(torch.bfloat16)
    out = torch.full((128, n), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    Ad, Bd = A.cuda(), Bm.cuda()
    rc = _lib.load().dropkv_selftest_tcgen05(mode, Ad.data_ptr(), Bd.data_ptr(), n, out.data_ptr(),
                                             status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "selftest")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    if mode in (0, 2):
        want = A.double() @ Bm.double().T                       # [128, n]
    else:
        Af = A.double()
        if D == 64:
            Af = torch.cat([Af, Af], dim=1)                     # second slab repeats the first
        want = Af.T @ Bm.double().T                             # [128 (d), n]
    torch.testing.assert_close(out.double().cpu(), want, rtol=1e-5, atol=1e-4)


def _scores_with(mode, Q, K, V, W, round_p):
    _lib.set_scorer(mode)
    try:
        return ops.scores(Q, K, V, W, round_p=round_p)
    finally:
        _lib.set_scorer(_lib.SCORER_AUTO)


CASES = [
    dict(B=1, Hq=32, Hkv=8, D=128, Lq=64, Lk=1000),    # Llama M=32
    dict(B=1, Hq=14, Hkv=2, D=64, Lq=64, Lk=777),      # Qwen M=56 -> N 64
    dict(B=1, Hq=8, Hkv=8, D=128, Lq=32, Lk=300),      # MHA M=8 -> N 16
    dict(B=2, Hq=8, Hkv=2, D=64, Lq=16, Lk=4097),      # batch 2, ragged last tile
    dict(B=1, Hq=4, Hkv=1, D=128, Lq=8, Lk=8),         # L = W: one partial tile
    dict(B=1, Hq=4, Hkv=2, D=128, Lq=8, Lk=129),       # a CTA whose keys are all masked for some rows
]


@pytest.mark.parametrize("cfg", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_scorer_matches_oracle(cfg, dtype):
    wl = Workload(dtype=dtype, seed=17, **cfg)
    Q, K, V = make_qkv(wl, "cpu")
    assert ops.scorer_for(dtype, wl.B, wl.Hq, wl.Hkv, wl.Lk, wl.D, 8) == "tensor_cores"
    Qn, Kn, Vn = (t.float().numpy() for t in (Q, K, V))
    cond = well_conditioned(O.max_attention(Qn, Kn, 8))
    Qd, Kd, Vd = Q.cuda(), K.cuda(), V.cuda()
    got = _scores_with(_lib.SCORER_TENSOR_CORES, Qd, Kd, Vd, 8, False).cpu().numpy()
    assert_scores_close(got, O.scores_reference(Qn, Kn, Vn, 8), 1e-3, 1e-4, mask=cond)
    name = "bf16" if dtype == torch.bfloat16 else "fp16"
    got_r = _scores_with(_lib.SCORER_TENSOR_CORES, Qd, Kd, Vd, 8, True).cpu().numpy()
    assert_scores_close(got_r, O.scores_reference(Qn, Kn, Vn, 8, round_p=name), 1e-2, 1e-3, mask=cond)
    simt = _scores_with(_lib.SCORER_CUDA_CORES, Qd, Kd, Vd, 8, False).cpu().numpy()
    assert_scores_close(got, simt, 1e-3, 1e-4, mask=cond, what="tensor vs CUDA cores")


@pytest.mark.parametrize("Lk", [32768, 131072])
def test_tensor_core_scorer_full_size(Lk):
    wl = llama_layer(Lk)
    Q, K, V = make_qkv(wl, "cuda")
    assert ops.scorer_for(wl.dtype, 1, 32, 8, Lk, 128, 8) == "tensor_cores"
    tc = _scores_with(_lib.SCORER_TENSOR_CORES, Q, K, V, 8, True)
    simt = _scores_with(_lib.SCORER_CUDA_CORES, Q, K, V, 8, True)
    assert torch.isfinite(tc).all()
    Qa, Ka = Q.float().cpu().numpy(), K.float().cpu().numpy()
    full_cond = well_conditioned(O.max_attention(Qa, Ka, 8))
    assert_scores_close(tc.cpu().numpy(), simt.cpu().numpy(), 1e-2, 1e-3, mask=full_cond,
                        what="tensor vs CUDA cores")
    h = 5
    Qn = Qa[:, 4 * h:4 * h + 4]
    Kn = Ka[:, h:h + 1]
    cond = full_cond[:, h:h + 1]
    Vn = V[:, h:h + 1].float().cpu().numpy()
    want = O.scores_reference(Qn, Kn, Vn, 8, round_p="bf16")
    assert_scores_close(tc[:, h:h + 1].cpu().numpy(), want, 1e-2, 1e-3, mask=cond)


def test_tensor_core_scorer_repeatable():
    wl = llama_layer(20000)
    Q, K, V = make_qkv(wl, "cuda")
    a = ops.scores(Q, K, V, 8)
    b = ops.scores(Q, K, V, 8)
    assert torch.equal(a, b)


def test_bounded_wait_timeout_sets_status_and_next_call_is_correct():
    """The scorer's failure path, driven without any fault: the test hook shortens
    the wait limit to 1 ms and makes head 0's first group barrier unreachable.
    The barrier wait runs out, the kernel records a non-zero status word and ends
    (the call itself returns DROPKV_OK); the Python layer turns the status into
    DropKVError(ERR_DEVICE).  The next call, hook off, on the same GPU and
    workspace sizes, gives the oracle's scores."""
    wl = llama_layer(8192)
    Q, K, V = (t.cuda() for t in make_qkv(wl, "cpu"))
    lib = _lib.load()
    B, Hq, Lq, D = Q.shape
    Hkv, Lk = K.shape[1], K.shape[2]
    ws = torch.zeros(lib.dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, 8), dtype=torch.uint8, device="cuda")
    out = torch.empty(B, Hkv, Lk, device="cuda")
    off = lib.dropkv_scores_status_offset(_lib.DTYPE_BF16, B, Hq, Hkv, Lk, D, 8)
    assert off != _lib.NO_STATUS, "the tensor-core scorer serves this shape"

    def call():
        return lib.dropkv_scores(Q.data_ptr(), *Q.stride(), Lq, K.data_ptr(), V.data_ptr(), _lib.DTYPE_BF16,
                                 B, Hq, Hkv, Lk, D, 8, 1e-6, _lib.ROUND_BF16, out.data_ptr(), ws.data_ptr(),
                                 ws.numel(), torch.cuda.current_stream().cuda_stream)

    _lib.check(lib.dropkv_test_scorer_waits(1_000_000, 1), "test hook")
    try:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        assert call() == _lib.OK
        t1.record()
        torch.cuda.synchronize()
        status = int(ws[off:off + 4].view(torch.int32).item())
        assert status != 0, "the blocked barrier's wait must run out and set the status word"
        assert t0.elapsed_time(t1) < 1000.0, "every wait gave up within its 1 ms limit"
        with pytest.raises(_lib.DropKVError) as err:
            ops.scores(Q, K, V, 8)  # DROPKV_CHECK_STATUS=1 (tests/conftest.py) reads the status
        assert err.value.code == _lib.ERR_DEVICE
    finally:
        _lib.check(lib.dropkv_test_scorer_waits(0, 0), "test hook off")
    assert call() == _lib.OK
    torch.cuda.synchronize()
    assert int(ws[off:off + 4].view(torch.int32).item()) == 0
    Qn, Kn, Vn = (t.float().cpu().numpy() for t in (Q, K, V))
    want = O.scores_reference(Qn, Kn, Vn, 8, round_p="bf16")
    cond = well_conditioned(O.max_attention(Qn, Kn, 8))
    assert_scores_close(out.cpu().numpy(), want, rtol=1e-2, atol=1e-3, mask=cond, what="after the timeout")
