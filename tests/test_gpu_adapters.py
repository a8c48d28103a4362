"""contracts::IExpertRuntime over an expert-parallel shard, on the GPU.

ExpertRuntimeB200 (llm-on-cpu_b200/adapters/contracts_b200.cpp, built against
the reference's src/contracts headers into libllmoc_adapters.so) runs
prefetch / pin / gemm_swiglu / release for one expert of this rank's shard.
Its output for n rows is compared with the oracle's expert FFN of each row
(down(silu(gate x) * up x), the reference's moe_cpu_experts arithmetic),
within the layer tolerance; an expert another rank owns gives an invalid
handle and runs nothing.  Skipped when the adapter library was not built
(it needs the reference tree at build time)."""
import ctypes as C
import os

import numpy as np
import pytest

import llmoc_b200 as L
import moe_gpu as G
import orc

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
ADAPTER = os.path.join(os.path.dirname(L.LIB_PATH), "adapters", "libllmoc_adapters.so")


@pytest.fixture(scope="module")
def adapter():
    if not os.path.exists(ADAPTER):
        pytest.skip("libllmoc_adapters.so not built")
    lib = C.CDLL(ADAPTER)
    fn = lib.llmoc_adapter_expert_runtime_run
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_int,
                   C.c_int, C.c_void_p, C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    return fn


@pytest.mark.parametrize("world,rank", [(1, 0), (2, 0), (2, 1)])
def test_expert_runtime_gemm_swiglu(oracle, adapter, world, rank):
    layer = orc.make_layer(oracle, np.random.default_rng(21), H=512, I=256, E=16, topk=4, gs=128)
    shard = L.EpLayerShard.from_host_ep(layer, rank, world)
    nbytes = L.lib.llmoc_expert_storage_bytes(512, 256, 128, 0)
    n = 13
    X = orc.make_tokens(np.random.default_rng(22), n, 512)
    Xd = G.bf16_dev(X)
    st = torch.cuda.current_stream()
    for expert in (3, 6, 11):
        Y = torch.zeros((n, 512), dtype=torch.bfloat16, device="cuda")
        owns, valid = C.c_int(-1), C.c_int(-1)
        rc = adapter(shard.handle, rank, world, 0, nbytes, 5, expert, Xd.data_ptr(), n, 512, Y.data_ptr(),
                     st.cuda_stream, C.byref(owns), C.byref(valid))
        torch.cuda.synchronize()
        assert rc == 0
        assert owns.value == int(expert % world == rank) and valid.value == owns.value
        if not owns.value:
            assert float(Y.float().abs().max()) == 0.0  # another rank's expert: nothing ran
            continue
        ref = np.stack([oracle.moe_ffn_routed(X[i], 512, 256, [layer.experts[expert]], np.ones(1, np.float32),
                                              None, 0.0) for i in range(n)])
        mre, cos = G.quality(G.bf16_to_f32(Y), ref)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (expert, mre, cos)
    shard.close()
