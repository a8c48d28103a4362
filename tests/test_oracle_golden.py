"""The CPU oracle against golden fixtures produced by the reference itself.

The fixtures in tests/golden/ were made by tests/golden/make_golden.py from the
reference's own compiled ``src/hal`` operators and its ``tools/quantize_int4.py``.
Every check here is bit-exact: the oracle restates the reference's fp32
operation order, so equality is the bar.
"""
import numpy as np
import pytest

import make_golden as mg
import orc

GOLD = {}


def gold(name):
    if name not in GOLD:
        GOLD[name] = np.load(f"{mg.HERE}/{name}.npz")
    return GOLD[name]


def cases(g):
    return sorted({k.split("/")[0] for k in g.files})


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("case", ["awq_scalar", "awq_batch", "gptq_batch", "awq_gemv", "gptq_gemv"])
def test_reference_unit_cases(oracle, case):
    """Known-answer cases of the reference's tests/unit/test_int4_gemm.cpp and
    test_gpu_quant_gemm.cpp: oracle == reference bits, and within the
    reference tests' own tolerance (1e-3 rel) of the scalar formula."""
    g = gold("unit_cases")
    d = {k.split("/")[1]: g[k] for k in g.files if k.startswith(case + "/")}
    M, K, gs, scheme = int(d["M"]), int(d["K"]), int(d["gs"]), int(d["scheme"])
    W = orc.Int4Weight(d["q"], d["s"], d.get("z"), M, K, gs, scheme, 7 if scheme == 2 else 0)
    assert bits_equal(oracle.dequant_matrix(W), d["dq"])
    if "x" in d:
        y = oracle.gemm_int4(d["x"], W)
        assert bits_equal(y, d["y"])
        ref_scalar = d["dq"].astype(np.float64) @ d["x"].astype(np.float64)
        assert np.all(np.abs(y - ref_scalar) < 1e-3 * (1 + np.abs(ref_scalar)))
    else:
        Y = oracle.gemm_int4_batch(d["X"], W)
        assert bits_equal(Y, d["Y"])
        for t in range(d["X"].shape[0]):
            assert np.all(np.abs(oracle.gemm_int4(d["X"][t], W) - Y[t]) < 1e-4 * (1 + np.abs(Y[t])))


ARGMAX = ["awq", "gptq", "awq_tie", "awq_nan", "awq_large", "gptq_neg"]


@pytest.mark.parametrize("case", ARGMAX)
def test_argmax_cases(oracle, case):
    """hal::gemm_int4_argmax (greedy lm_head): the oracle's (index, value)
    equal the reference's bits on every case -- AWQ and GPTQ rows, equal
    largest rows (the first wins), a NaN input (every row non-finite: value
    -1e30, index 0), M >= 4096, all rows negative."""
    import make_golden as mg

    g = gold("argmax_cases")
    x, W = mg.argmax_weight(case)
    assert bits_equal(x, g[f"{case}/x"])
    i, v = oracle.gemm_int4_argmax(x, W)
    assert i == int(g[f"{case}/index"])
    assert bits_equal(v, g[f"{case}/value"])


@pytest.mark.parametrize("gs", [32, 128])
def test_quantizers_match_reference_tool(oracle, gs):
    """quant_awq_sym / quant_gptq_asym of tools/quantize_int4.py, byte for byte."""
    g = gold("quant_cases")
    p = f"quant_gs{gs}/"
    W = g[p + "W"]
    a = oracle.quant_awq_sym(W, gs)
    assert np.array_equal(a.q.reshape(-1), g[p + "awq_q"])
    assert np.array_equal(a.scales.reshape(-1), g[p + "awq_s"])
    q = oracle.quant_gptq_asym(W, gs)
    assert np.array_equal(q.q.reshape(-1), g[p + "gptq_q"])
    assert np.array_equal(q.scales.reshape(-1), g[p + "gptq_s"])
    assert np.array_equal(q.zeros.reshape(-1), g[p + "gptq_z"])


@pytest.mark.parametrize("case", list(mg.ROUTER_CASES))
def test_router_logits(oracle, case):
    """gemm_bias_free (cpu_ops.cpp:57-95) logits, bit-exact (ids depend on them)."""
    g = gold("router_cases")
    Wb, X = mg.router_inputs(case)
    assert mg.digest(Wb, X) == str(g[case + "/input_sha256"])
    logits = np.stack([oracle.gemm_bias_free(X[t], Wb) for t in range(X.shape[0])])
    assert bits_equal(logits, g[case + "/logits"])


def test_silu_and_mul(oracle):
    g = gold("router_cases")
    assert bits_equal(oracle.silu_and_mul(g["silu/g"], g["silu/u"]), g["silu/out"])


@pytest.mark.parametrize("case", list(mg.LAYER_CASES))
def test_layer_forward(oracle, case):
    """Full per-token MoE layer: ids, weights and fp32 outputs, bit-exact."""
    g = gold("layer_cases")
    L, X, h = mg.layer_inputs(oracle, case)
    assert h == str(g[f"layer_{case}/input_sha256"])
    Y, ids, w, ties = oracle.moe_layer_forward(L, X)
    assert not ties.any()
    assert np.array_equal(ids, g[f"layer_{case}/ids"])
    assert bits_equal(w, g[f"layer_{case}/w"])
    assert bits_equal(Y, g[f"layer_{case}/Y"])


def test_permutation_is_canonical(oracle):
    rng = np.random.default_rng(5)
    T, k, E = 37, 8, 20
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    off, srt, inv = oracle.permute(ids, E)
    pairs = [(int(ids.reshape(-1)[p]), p // k, p % k) for p in range(T * k)]
    expect = sorted(range(T * k), key=lambda p: pairs[p])
    assert list(srt) == expect
    assert np.array_equal(inv[srt], np.arange(T * k))
    assert np.array_equal(np.diff(off), np.bincount(ids.reshape(-1), minlength=E))


def test_oracle_vs_reference_random(oracle, reference):
    """Random shapes through both libraries (skipped when oracle/_ref is absent)."""
    rng = np.random.default_rng(99)
    for _ in range(40):
        M = int(rng.choice([1, 3, 8, 17, 64, 4096, 4097]))
        K = int(rng.choice([32, 96, 100, 256, 2048]))
        gs = int(rng.choice([32, 64, 128]))
        sc = int(rng.choice([1, 2]))
        rb, ng = (K + 1) // 2, (K + gs - 1) // gs
        W = orc.Int4Weight(rng.integers(0, 256, (M, rb), dtype=np.uint8),
                           rng.integers(0x2000, 0x2400, (M, ng)).astype(np.uint16),
                           rng.integers(0xA000, 0xA400, (M, ng)).astype(np.uint16) if sc == 1 else None,
                           M, K, gs, sc, 7 if sc == 2 else 0)
        x = rng.standard_normal(K, dtype=np.float32)
        X = rng.standard_normal((3, K), dtype=np.float32)
        assert bits_equal(oracle.gemm_int4(x, W), reference.gemm_int4(x, W))
        assert bits_equal(oracle.gemm_int4_batch(X, W), reference.gemm_int4_batch(X, W))
