"""The C-ABI library on a CPU-only host: it loads, exports exactly what the
header declares, and its host-side logic (argument checks, byte geometry,
error reporting) behaves without touching a GPU."""
import ctypes as C
import subprocess

import numpy as np
import pytest

import llmoc_b200 as L


def test_exports_match_header():
    declared = L.header_symbols()
    assert len(declared) >= 30
    out = subprocess.check_output(["nm", "-D", "--defined-only", L.LIB_PATH]).decode()
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported, sorted(set(declared) - exported)
    assert {s for s in exported if s.startswith("llmoc_")} == set(declared)


def test_struct_layouts_match_reference_types():
    """sizeof/offsetof of the reference's qlwc::Int4View and hal::cuda::MoeExpertInt4
    on x86-64 (g++ over src/weights/qlwc_store.h, src/hal/cuda_backend.h):
    Int4View 56 bytes, M at 32, scheme at 44, awq_zp at 48; MoeExpertInt4 32, weight at 24."""
    assert C.sizeof(L.Int4View) == 56
    assert (L.Int4View.M.offset, L.Int4View.scheme.offset, L.Int4View.awq_zp.offset) == (32, 44, 48)
    assert C.sizeof(L.MoeExpertInt4) == 32 and L.MoeExpertInt4.weight.offset == 24


@pytest.mark.parametrize("H,I,gs,z,expect", [
    (2048, 768, 128, 0, 2_433_024),     # Qwen3-30B-A3B expert
    (4096, 1408, 128, 0, 8_921_088),    # GLM-4.5-Air expert
    (7168, 2048, 32, 0, 24_772_608),    # Kimi-K2 expert, gs 32
    (2048, 768, 128, 1, 2_433_024 + 2 * (768 * 16 * 2) + 2048 * 6 * 2),
])
def test_expert_storage_bytes(H, I, gs, z, expect):
    """src/moe/qlwc_expert_bytes.h:43-48 (test_moe_offload_cache.cpp:10-20 checks the same)."""
    assert L.lib.llmoc_expert_storage_bytes(H, I, gs, z) == expect


def test_no_gpu_paths_fail_cleanly():
    if L.lib.llmoc_cuda_probe_available():
        pytest.skip("a GPU is present")
    assert L.lib.llmoc_cuda_enable(0) == 0
    assert L.lib.llmoc_cuda_enabled() == 0
    assert L.lib.llmoc_cuda_status()
    x = np.zeros(64, np.float32)
    y = np.zeros(16, np.float32)
    q = np.zeros((16, 32), np.uint8)
    s = np.zeros((16, 1), np.uint16)
    v = L.view(q, s, None, 16, 64, 64)
    assert L.lib.llmoc_try_gemm_int4(L.ptr(x), C.byref(v), L.ptr(y)) == 0
    assert "not enabled" in L.last_error()


def _desc(**kw):
    d = dict(hidden=256, inter=128, n_experts=8, topk=2, group_size=64, scheme=2, awq_zp=7,
             router=0, routed_scaling=1.0, has_shared=0, shared_scale=1.0)
    d.update(kw)
    return L.LayerDesc(*[d[f[0]] for f in L.LayerDesc._fields_])


@pytest.mark.parametrize("kw,code", [
    (dict(topk=0), 1), (dict(topk=65, n_experts=100), 1), (dict(topk=9, n_experts=8), 1),
    (dict(n_experts=600), 6), (dict(group_size=48), 6), (dict(hidden=100), 6),
    (dict(router=7), 1), (dict(scheme=3), 1),
])
def test_layer_desc_validation(kw, code):
    """Bad layer shapes are rejected before any device work."""
    h = C.c_void_p()
    rw = np.zeros(1, np.uint16)
    views = (L.Int4View * 3)()
    st = L.lib.llmoc_moe_layer_create(C.byref(_desc(**kw)), L.ptr(rw), None, views, None, 0, C.byref(h))
    assert st == code, (st, L.last_error())
    assert h.value is None


def test_layer_view_mismatch_rejected():
    """Views whose shapes disagree with the layer are refused (no upload)."""
    h = C.c_void_p()
    rw = np.zeros(8 * 256, np.uint16)
    q = np.zeros((128, 128), np.uint8)
    s = np.zeros((128, 4), np.uint16)
    good = L.view(q, s, None, 128, 256, 64)
    bad = L.view(q, s, None, 128, 192, 64)
    views = (L.Int4View * 24)(*([good, good, L.view(q, s, None, 256, 128, 64)] * 7 + [good, bad, good]))
    st = L.lib.llmoc_moe_layer_create(C.byref(_desc()), L.ptr(rw), None, views, None, 0, C.byref(h))
    assert st == 1 and "expert 7" in L.last_error()


def test_null_arguments():
    assert L.lib.llmoc_moe_forward(None, None, 1, None, None, 0, None) == 1
    assert L.lib.llmoc_moe_workspace_bytes(None, 4) == 0
    assert L.lib.llmoc_try_moe_ffn_int4(None, 1, 1, None, 0, None, None, None, 0.0, None) == 0
