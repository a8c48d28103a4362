"""The drop-in boundary against the reference's own headers (CPU only).

The adapters under llm-on-cpu_b200/adapters are the files a maintainer adds
to the reference's build: the hal::cuda INT4/MoE entry points
(src/hal/cuda_backend.h) on this library's C ABI, contracts::ICollective and
contracts::IExpertRuntime (src/contracts/), and the Qwen3.6 MoE model whose
moe_ffn_token runs on the device (src/model/qwen3_6_moe_int4_model.h).  They
are compiled here against the reference tree, so a change of the
reference's types or of include/llmoc_b200.h that breaks the byte-for-byte
struct layouts stops the build (static_asserts in cuda_backend_b200.cpp).
Skipped when the reference tree is not on this machine (it is not needed at
run time)."""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ADAPTERS = os.path.join(REPO, "llm-on-cpu_b200", "adapters")


def reference_tree():
    t = os.environ.get("LLMOC_REFERENCE_TREE") or os.path.join(os.path.dirname(REPO), "reference")
    return t if os.path.isfile(os.path.join(t, "src", "hal", "cuda_backend.h")) else None


@pytest.fixture(scope="module")
def ref():
    t = reference_tree()
    if t is None:
        pytest.skip("the reference tree is not on this machine")
    return t


def test_adapters_build_against_reference_headers(ref, tmp_path):
    out = tmp_path / "adapters"
    out.mkdir()
    for src in ("cuda_backend_b200.cpp", "contracts_b200.cpp", "qwen36_moe_b200.cpp"):
        subprocess.check_call(["/usr/bin/g++", "-std=gnu++20", "-O1", "-fPIC", f"-I{ref}/src",
                               f"-I{REPO}/include", "-I/usr/local/cuda/include", "-c",
                               os.path.join(ADAPTERS, src), "-o", str(out / (src + ".o"))])


def test_layout_drift_stops_the_build(ref, tmp_path):
    """A copy of the C header with one member moved must fail the adapter's static_asserts."""
    hdr = open(os.path.join(REPO, "include", "llmoc_b200.h")).read()
    moved = hdr.replace("  int32_t M, K;\n  int32_t group_size;", "  int32_t group_size;\n  int32_t M, K;", 1)
    assert moved != hdr
    (tmp_path / "llmoc_b200.h").write_text(moved)
    r = subprocess.run(["/usr/bin/g++", "-std=gnu++20", "-fsyntax-only", f"-I{ref}/src", f"-I{tmp_path}",
                        os.path.join(ADAPTERS, "cuda_backend_b200.cpp")], capture_output=True, text=True)
    assert r.returncode != 0 and "static assertion failed" in r.stderr


def _layout_program(tmp_path, ref):
    src = tmp_path / "layout.cpp"
    src.write_text('''
#include <cstddef>
#include <cstdio>
#include "hal/cuda_backend.h"
int main() {
  using llmoc::qlwc::Int4View;
  using llmoc::hal::cuda::MoeExpertInt4;
  std::printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(Int4View), offsetof(Int4View, qweight),
              offsetof(Int4View, scales), offsetof(Int4View, zeros), offsetof(Int4View, scales_f32),
              offsetof(Int4View, M), offsetof(Int4View, K), offsetof(Int4View, group_size),
              offsetof(Int4View, scheme), offsetof(Int4View, awq_zp));
  std::printf("%zu %zu %zu %zu %zu\\n", sizeof(MoeExpertInt4), offsetof(MoeExpertInt4, gate),
              offsetof(MoeExpertInt4, up), offsetof(MoeExpertInt4, down), offsetof(MoeExpertInt4, weight));
}
''')
    exe = tmp_path / "layout"
    subprocess.check_call(["/usr/bin/g++", "-std=gnu++20", f"-I{ref}/src", str(src), "-o", str(exe)])
    return [list(map(int, ln.split())) for ln in subprocess.check_output([str(exe)]).decode().splitlines()]


def test_ctypes_binding_matches_reference_layouts(ref, tmp_path):
    """The Python binding's structs (what the tests and bench pass) have the
    reference's sizes and offsets, read from the reference headers by g++."""
    import ctypes as C

    import llmoc_b200 as L

    view, moe = _layout_program(tmp_path, ref)
    V = L.Int4View
    assert view == [C.sizeof(V), V.qweight.offset, V.scales.offset, V.zeros.offset, V.scales_f32.offset,
                    V.M.offset, V.K.offset, V.group_size.offset, V.scheme.offset, V.awq_zp.offset]
    E = L.MoeExpertInt4
    assert moe == [C.sizeof(E), E.gate.offset, E.up.offset, E.down.offset, E.weight.offset]
