"""The allocation-free forward (llmoc_moe_forward_noalloc), on the GPU.

It exists for callers that cannot give the library device memory for a
workspace (their device memory belongs to another allocator, their serving
loop must not call cudaMalloc/cudaFree, or they call through an FFI with no
device allocator).  It must give the same result as llmoc_moe_forward with a
caller-provided workspace, call after call (the static scratch keeps the
previous call's contents), and refuse token counts whose workspace would not
fit its fixed 8 MiB scratch.  This file is collected last on purpose.
"""
import numpy as np
import pytest

import llmoc_b200 as L
import moe_gpu as G
import orc

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_noalloc_forward_matches_workspace_forward(oracle):
    assert torch.cuda.is_available()
    rng = np.random.default_rng(2026)
    layer = orc.make_layer(oracle, rng, H=512, I=256, E=32, topk=8, gs=128)
    dl = G.DevLayer(layer, 48)
    cap = L.lib.llmoc_moe_noalloc_capacity()
    assert cap == 8 << 20
    stream = torch.cuda.current_stream()
    for T in (37, 12, 1):  # calls in a row, different sizes (stale scratch must not matter; T = 1: one launch)
        X = orc.make_tokens(rng, T, layer.H)
        Xd = G.bf16_dev(X)
        Y_ref, _ = dl.forward(X)  # caller-provided workspace
        Y = torch.empty((T, layer.H), dtype=torch.bfloat16, device="cuda")
        st = L.lib.llmoc_moe_forward_noalloc(dl.dev.handle, Xd.data_ptr(), T, Y.data_ptr(),
                                             stream.cuda_stream)
        assert st == 0, L.last_error()
        # the forward's device error word lives in the static array: read through the status query
        assert L.lib.llmoc_moe_noalloc_status(dl.dev.handle, T, stream.cuda_stream) == 0, L.last_error()
        torch.cuda.synchronize()
        mre, cos = G.quality(G.bf16_to_f32(Y), G.bf16_to_f32(Y_ref))
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (T, mre, cos)
        Yo, _, _, _ = oracle.moe_layer_forward(layer, X)
        mre, cos = G.quality(G.bf16_to_f32(Y), Yo)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (T, mre, cos)
    dl.close()


def test_noalloc_refuses_sizes_beyond_capacity(oracle):
    rng = np.random.default_rng(7)
    layer = orc.make_layer(oracle, rng, H=512, I=256, E=32, topk=8, gs=128)
    dev = L.MoeLayer.from_host(layer, 0)
    cap = L.lib.llmoc_moe_noalloc_capacity()
    T = 1
    while dev.workspace_bytes(T) <= cap:
        T *= 2
    X = torch.zeros((T, layer.H), dtype=torch.bfloat16, device="cuda")
    Y = torch.empty((T, layer.H), dtype=torch.bfloat16, device="cuda")
    st = L.lib.llmoc_moe_forward_noalloc(dev.handle, X.data_ptr(), T, Y.data_ptr(), None)
    assert st == 7 and "static scratch" in L.last_error()
    assert L.lib.llmoc_moe_noalloc_status(dev.handle, T, None) == 1  # no such forward fits
    dev.close()
