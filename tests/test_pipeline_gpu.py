"""ops.HostPipeline: layers in pinned host memory compressed with overlapped
copies give the same outputs as one compress call per layer on the device."""

import pytest
import torch

from dropkv_b200 import ops
from dropkv_b200.workloads import llama_layer, make_qkv

pytestmark = pytest.mark.gpu


def test_host_pipeline_matches_per_layer_compress():
    dev = torch.device("cuda")
    layers = []
    for seed in (3, 4, 5):
        wl = llama_layer(4096, seed=seed)
        Q, K, V = make_qkv(wl, dev)
        kl = wl.keep_len()
        want = ops.compress(Q, K, V, 8, 11, kl)
        outs = (torch.empty(1, 8, kl, dtype=torch.int64).pin_memory(),
                torch.empty(1, 8, kl, 128, dtype=torch.bfloat16).pin_memory(),
                torch.empty(1, 8, kl, 128, dtype=torch.bfloat16).pin_memory())
        layers.append(((Q.cpu().pin_memory(), K.cpu().pin_memory(), V.cpu().pin_memory()) + outs, want))
    pipe = ops.HostPipeline(1, 32, 8, 8, 4096, 128, torch.bfloat16, 8, 11, layers[0][1][0].shape[-1], device=dev)
    for rep in range(2):  # the slots are reused across runs
        pipe.run([item for item, _ in layers]).synchronize()
        for item, (idx, kc, vc) in layers:
            assert torch.equal(item[3], idx.cpu())
            assert torch.equal(item[4], kc.cpu())
            assert torch.equal(item[5], vc.cpu())


def test_compressor_graph_replay_matches_run():
    dev = torch.device("cuda")
    wl = llama_layer(32768, seed=6)
    Q, K, V = make_qkv(wl, dev)
    kl = wl.keep_len()
    comp = ops.Compressor(1, 32, 8, 8, 32768, 128, torch.bfloat16, 8, 11, kl, device=dev)
    idx, kc, vc = (t.clone() for t in comp.run(Q, K, V))
    assert comp.capture(Q, K, V) >= 3  # scorer, selection, gather
    for t in (comp.keep_idx, comp.k_out, comp.v_out):
        t.zero_()
    for _ in range(2):
        comp.replay()
    torch.cuda.synchronize()
    assert torch.equal(comp.keep_idx, idx) and torch.equal(comp.k_out, kc) and torch.equal(comp.v_out, vc)
