"""The C-ABI library on a CPU-only host: it loads, exports exactly what the
header declares, and its host-side logic (argument checks, byte geometry,
error reporting) behaves without touching a GPU."""
import ctypes as C
import os
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


def test_ctypes_structs_match_the_c_header(tmp_path):
    """The binding's structs and include/llmoc_b200.h, both read by compilers
    (the header's layouts against the reference's own types are pinned by
    tests/test_boundary.py)."""
    src = tmp_path / "h.c"
    src.write_text("""
#include <stddef.h>
#include <stdio.h>
#include "llmoc_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(llmoc_int4_view), offsetof(llmoc_int4_view, qweight),
         offsetof(llmoc_int4_view, scales), offsetof(llmoc_int4_view, zeros), offsetof(llmoc_int4_view, scales_f32),
         offsetof(llmoc_int4_view, M), offsetof(llmoc_int4_view, K), offsetof(llmoc_int4_view, group_size),
         offsetof(llmoc_int4_view, scheme), offsetof(llmoc_int4_view, awq_zp));
  printf("%zu %zu %zu %zu %zu\\n", sizeof(llmoc_moe_expert_int4), offsetof(llmoc_moe_expert_int4, gate),
         offsetof(llmoc_moe_expert_int4, up), offsetof(llmoc_moe_expert_int4, down),
         offsetof(llmoc_moe_expert_int4, weight));
  return 0;
}
""")
    exe = tmp_path / "h"
    subprocess.check_call(["gcc", f"-I{os.path.dirname(L.HEADER)}", str(src), "-o", str(exe)])
    view, moe = [list(map(int, ln.split())) for ln in subprocess.check_output([str(exe)]).decode().splitlines()]
    V, E = L.Int4View, L.MoeExpertInt4
    assert view == [C.sizeof(V), V.qweight.offset, V.scales.offset, V.zeros.offset, V.scales_f32.offset,
                    V.M.offset, V.K.offset, V.group_size.offset, V.scheme.offset, V.awq_zp.offset]
    assert moe == [C.sizeof(E), E.gate.offset, E.up.offset, E.down.offset, E.weight.offset]


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
