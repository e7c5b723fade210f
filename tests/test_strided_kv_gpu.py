"""K/V read in place from a model's layout: the [B, L, Hkv, D] projections that
an attention module hands over as [B, Hkv, L, D] views. ``dropkv_compress_kv_strides``
(through ``ops.compress``) must give exactly what ``dropkv_compress`` gives on the
packed copy: the same scorer arithmetic, with only the addresses of the K/V tiles
and gathered rows changed."""

import pytest
import torch

from dropkv_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _model_views(B, L, Hq, Hkv, D, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, L, Hq, D, device="cuda", generator=g).to(dtype).transpose(1, 2)
    k = (torch.randn(B, L, Hkv, D, device="cuda", generator=g) * 1.5).to(dtype).transpose(1, 2)
    v = torch.randn(B, L, Hkv, D, device="cuda", generator=g).to(dtype).transpose(1, 2)
    return q, k, v


@pytest.mark.parametrize("B,L,Hq,Hkv,D", [
    (1, 8192, 14, 2, 64),     # Qwen2-0.5B prefill (config 3)
    (2, 3000, 32, 8, 128),    # batch 2: the sequence stride is not Hkv * head stride
    (1, 777, 8, 8, 128),      # MHA, a ragged last tile
    (1, 20000, 32, 8, 128),
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_model_layout_equals_packed_copy(B, L, Hq, Hkv, D, dtype):
    q, k, v = _model_views(B, L, Hq, Hkv, D, dtype, seed=L + D)
    assert not k.is_contiguous() and ops._kv_strides(k, v) is not None
    keep = max(8, L // 10)
    n0 = _lib.launch_count()
    idx, kc, vc, sc = ops.compress(q, k, v, 8, 11, keep, return_scores=True)
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 4, "memset, scorer, select, gather: no copy kernels of this library"
    idx_p, kc_p, vc_p, sc_p = ops.compress(q, k.contiguous(), v.contiguous(), 8, 11, keep, return_scores=True)
    assert torch.equal(sc, sc_p)
    assert torch.equal(idx, idx_p)
    assert torch.equal(kc, kc_p) and torch.equal(vc, vc_p)


def test_layouts_the_tensor_core_scorer_does_not_serve_are_packed_first():
    # fp32 goes to the CUDA-core scorer, which needs packed rows: ops.compress
    # copies, and the C entry itself refuses the strided layout
    q, k, v = _model_views(1, 1000, 8, 2, 64, torch.float32, seed=4)
    idx, kc, vc = ops.compress(q, k, v, 8, 11, 100)
    idx_p, kc_p, vc_p = ops.compress(q, k.contiguous(), v.contiguous(), 8, 11, 100)
    assert torch.equal(idx, idx_p) and torch.equal(kc, kc_p) and torch.equal(vc, vc_p)
    lib = _lib.load()
    sb, sh, ss = ops._kv_strides(k, v)
    ws = torch.empty(lib.dropkv_compress_workspace_size(1, 8, 2, 1000, 64, 8), dtype=torch.uint8, device="cuda")
    out_i = torch.empty(1, 2, 100, dtype=torch.int64, device="cuda")
    out_k = torch.empty(1, 2, 100, 64, device="cuda")
    out_v = torch.empty_like(out_k)
    rc = lib.dropkv_compress_kv_strides(q.data_ptr(), *q.stride(), 1000, k.data_ptr(), v.data_ptr(), sb, sh, ss,
                                        _lib.DTYPE_F32, 1, 8, 2, 1000, 64, 8, 1e-6, _lib.ROUND_NONE, 11, 8, 100,
                                        None, out_i.data_ptr(), out_k.data_ptr(), out_v.data_ptr(), ws.data_ptr(),
                                        ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_UNSUPPORTED
    assert "packed" in lib.dropkv_last_error().decode()
