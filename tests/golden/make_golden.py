#!/usr/bin/env python3
"""Generate the golden fixtures in this folder from the reference itself.

Run in a container that has the reference tree (read-only) and the compiled
reference operators (``make -C oracle ref``):

    python tests/golden/make_golden.py [--ref /path/to/llm-on-cpu]

Sources of truth, all from appolloqin/llm-on-cpu:
* ``tools/quantize_int4.py`` (imported from the reference tree):
  ``quant_awq_sym`` (:150-166), ``quant_gptq_asym`` (:127-147), ``pack_int4`` (:115-124);
* ``oracle/_ref/libllmoc_ref.so``: the reference's own ``src/hal`` sources
  (``hal::gemm_int4``, ``gemm_int4_batch``, ``dequant_int4_row``,
  ``gemm_bias_free``, ``silu_and_mul``) plus the per-token MoE loop restated
  in ``oracle/ref_shim.cpp`` from ``src/model/qwen3_6_moe_int4_model.cpp:184-232,377-404``,
  run single-threaded so the expert combine has one defined order;
* the known-answer cases of ``tests/unit/test_int4_gemm.cpp:40-149`` and
  ``tests/unit/test_gpu_quant_gemm.cpp:130-245`` (same patterns, same sizes);
* ``write_qlwc`` of ``tools/quantize_int4.py`` (:183-260): a one-layer QLWC
  file (``qlwc_cases.npz``) for the library's QLWC loader.
* ``hal::gemm_int4_argmax`` (``src/hal/int4_ops.cpp:344-446``) through the
  compiled reference: (index, value) of six cases whose weights come from
  numpy seeds (``argmax_cases.npz``; ``argmax_weight`` rebuilds them).

Inputs that are large are not stored: they are regenerated from the seed by
``oracle/orc.py`` (whose quantizer is itself pinned here against the Python
reference), and the fixture stores a hash of them next to the outputs.
The golden files are read by tests/test_oracle_golden.py.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

os.environ.setdefault("OMP_NUM_THREADS", "1")

import numpy as np  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
import orc  # noqa: E402


def f32_to_f16bits_trunc(x: float) -> int:
    """The truncating converter of tests/unit/test_int4_gemm.cpp:25-37."""
    u = int(np.array([x], np.float32).view(np.uint32)[0])
    sign = (u >> 16) & 0x8000
    exp = ((u >> 23) & 0xFF) - 127 + 15
    man = u & 0x7FFFFF
    if exp <= 0:
        return sign
    if exp >= 31:
        return sign | 0x7C00
    return sign | (exp << 10) | (man >> 13)


def pack(q: np.ndarray) -> np.ndarray:
    M, K = q.shape
    out = np.zeros((M, (K + 1) // 2), np.uint8)
    for k in range(0, K, 2):
        lo = q[:, k]
        hi = q[:, k + 1] if k + 1 < K else 0
        out[:, k // 2] = (lo | (hi << 4)).astype(np.uint8)
    return out


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def unit_cases(R: orc.Reference) -> dict:
    out = {}
    # GemmAwqMatchesScalarRef (test_int4_gemm.cpp:40-78)
    M, K, gs = 17, 128, 128
    q = np.array([(i * 3) % 16 for i in range(M * K)], np.uint8).reshape(M, K)
    sc = np.array([f32_to_f16bits_trunc(0.01 + 0.001 * m) for m in range(M)], np.uint16).reshape(M, 1)
    x = np.array([0.02 * ((k % 7) - 3) for k in range(K)], np.float32)
    W = orc.Int4Weight(pack(q), sc, None, M, K, gs, orc.SCHEME_AWQ_SYM, 7)
    out["awq_scalar"] = dict(q=W.q, s=W.scales, x=x, M=M, K=K, gs=gs, scheme=2, y=R.gemm_int4(x, W))
    # GemmBatchMatchesSingle (:80-113)
    M, K, gs, n = 64, 128, 128, 7
    q = np.array([(i * 5 + 1) % 16 for i in range(M * K)], np.uint8).reshape(M, K)
    sc = np.full((M, 1), f32_to_f16bits_trunc(0.02), np.uint16)
    X = np.array([0.01 * ((i % 11) - 5) for i in range(n * K)], np.float32).reshape(n, K)
    W = orc.Int4Weight(pack(q), sc, None, M, K, gs, orc.SCHEME_AWQ_SYM, 7)
    out["awq_batch"] = dict(q=W.q, s=W.scales, X=X, M=M, K=K, gs=gs, scheme=2, Y=R.gemm_int4_batch(X, W))
    # GptqGemmBatchMatchesSingle (:115-149)
    M, K, gs, n = 64, 128, 128, 9
    q = np.array([(i * 7 + 3) % 16 for i in range(M * K)], np.uint8).reshape(M, K)
    sc = np.array([f32_to_f16bits_trunc(0.015 + 0.0001 * (i % 17)) for i in range(M)], np.uint16).reshape(M, 1)
    z = np.array([f32_to_f16bits_trunc(-0.05 + 0.001 * (i % 7)) for i in range(M)], np.uint16).reshape(M, 1)
    X = np.array([0.01 * ((i % 13) - 6) for i in range(n * K)], np.float32).reshape(n, K)
    W = orc.Int4Weight(pack(q), sc, z, M, K, gs, orc.SCHEME_GPTQ_ASYM, 0)
    out["gptq_batch"] = dict(q=W.q, s=W.scales, z=z, X=X, M=M, K=K, gs=gs, scheme=1, Y=R.gemm_int4_batch(X, W))
    # AwqGemvJitMatchesCpu (test_gpu_quant_gemm.cpp:130-183)
    M, K, gs = 24, 256, 128
    ng = K // gs
    q = np.array([(i * 7 + 3) % 16 for i in range(M * K)], np.uint8).reshape(M, K)
    sc = np.array([f32_to_f16bits_trunc(0.01 * ((i % 5) + 1)) for i in range(M * ng)], np.uint16).reshape(M, ng)
    x = np.array([0.02 * ((k % 11) - 5) for k in range(K)], np.float32)
    W = orc.Int4Weight(pack(q), sc, None, M, K, gs, orc.SCHEME_AWQ_SYM, 7)
    out["awq_gemv"] = dict(q=W.q, s=W.scales, x=x, M=M, K=K, gs=gs, scheme=2, y=R.gemm_int4(x, W))
    # GptqGemvJitMatchesCpu (:186-245)
    M, K, gs = 16, 256, 128
    ng = K // gs
    q = np.array([(i * 5 + 1) % 16 for i in range(M * K)], np.uint8).reshape(M, K)
    sc = np.array([f32_to_f16bits_trunc(0.02 * ((i % 3) + 1)) for i in range(M * ng)], np.uint16).reshape(M, ng)
    z = np.array([f32_to_f16bits_trunc(-0.1 * (i % 4)) for i in range(M * ng)], np.uint16).reshape(M, ng)
    x = np.array([0.03 * ((k % 7) - 3) for k in range(K)], np.float32)
    W = orc.Int4Weight(pack(q), sc, z, M, K, gs, orc.SCHEME_GPTQ_ASYM, 0)
    out["gptq_gemv"] = dict(q=W.q, s=W.scales, z=z, x=x, M=M, K=K, gs=gs, scheme=1, y=R.gemm_int4(x, W))
    for v in out.values():
        v["dq"] = R.dequant_matrix(orc.Int4Weight(v["q"], v["s"], v.get("z"), v["M"], v["K"], v["gs"],
                                                  v["scheme"], 7 if v["scheme"] == 2 else 0))
    return out


def quant_cases(qi) -> dict:
    out = {}
    rng = np.random.default_rng(2024)
    for gs in (32, 128):
        W = orc.bf16_round(rng.standard_normal((32, 512), dtype=np.float32) * np.float32(0.02))
        aq, asc, _ = qi.quant_awq_sym(W, gs)
        gq, gsc, gz = qi.quant_gptq_asym(W, gs)
        out[f"quant_gs{gs}"] = dict(W=W, awq_q=np.frombuffer(aq, np.uint8), awq_s=asc,
                                    gptq_q=np.frombuffer(gq, np.uint8), gptq_s=gsc, gptq_z=gz, gs=gs)
    return out


ROUTER_CASES = {
    # name: (seed, E, H, T)
    "router_128x2048": (77, 128, 2048, 4),
    "router_384x7168": (78, 384, 7168, 2),
    "router_7x100": (79, 7, 100, 3),
    "router_129x4096": (80, 129, 4096, 2),
}


def router_inputs(name: str):
    seed, E, H, T = ROUTER_CASES[name]
    rng = np.random.default_rng(seed)
    Wb = orc.bf16_bits(rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02))
    X = orc.make_tokens(rng, T, H)
    return Wb, X


def router_cases(R: orc.Reference) -> dict:
    out = {}
    for name in ROUTER_CASES:
        Wb, X = router_inputs(name)
        logits = np.stack([R.gemm_bias_free(X[t], Wb) for t in range(X.shape[0])])
        out[name] = dict(logits=logits, input_sha256=np.array(digest(Wb, X)))
    rng = np.random.default_rng(81)
    g = (rng.standard_normal(4096, dtype=np.float32) * 4).astype(np.float32)
    u = rng.standard_normal(4096, dtype=np.float32)
    out["silu"] = dict(g=g, u=u, out=R.silu_and_mul(g, u))
    return out


LAYER_CASES = {
    # name: (seed, make_layer kwargs, T)
    "qwen_small_softmax": (11, dict(H=512, I=256, E=32, topk=8, gs=128), 6),
    "glm_small_sigmoid_shared": (12, dict(H=512, I=128, E=32, topk=8, gs=128, router=1,
                                          routed_scaling=1.0, shared=True, shared_scale=1.0), 5),
    "kimi_small_gs32": (13, dict(H=448, I=128, E=48, topk=8, gs=32, router=1,
                                 routed_scaling=2.827, shared=True), 4),
    "gptq_small": (14, dict(H=256, I=128, E=16, topk=4, gs=64, scheme=1, shared=True, shared_scale=0.5), 5),
    # Qwen3.6-style shared expert with its per-token sigmoid gate (qwen3_6_moe_int4_model.cpp:365-371)
    "gptq_shared_gate": (15, dict(H=256, I=128, E=16, topk=4, gs=64, scheme=1, shared=True,
                                  shared_gate=True), 6),
}


def layer_inputs(O: orc.Oracle, name: str):
    seed, kw, T = LAYER_CASES[name]
    rng = np.random.default_rng(seed)
    L = orc.make_layer(O, rng, **kw)
    X = orc.make_tokens(rng, T, kw["H"])
    arrays = [L.router_w, X] + [a for e in L.experts for w in (e.gate, e.up, e.down)
                                for a in (w.q, w.scales) + ((w.zeros,) if w.zeros is not None else ())]
    if L.bias is not None:
        arrays.append(L.bias)
    if L.shared is not None:
        arrays += [L.shared.gate.q, L.shared.up.q, L.shared.down.q]
    if L.shared_gate_w is not None:
        arrays.append(L.shared_gate_w)
    return L, X, digest(*arrays)


def layer_cases(O: orc.Oracle, R: orc.Reference) -> dict:
    out = {}
    for name in LAYER_CASES:
        L, X, h = layer_inputs(O, name)
        Y, ids, w, _ = R.moe_layer_forward(L, X)
        out[f"layer_{name}"] = dict(Y=Y, ids=ids, w=w, input_sha256=np.array(h))
    return out


# One MoE layer as the reference's tools write it: GPTQ experts, a shared
# expert with its per-token gate, bf16 router; layer index 3 under "model.".
# hal::gemm_int4_argmax (int4_ops.cpp:344-446) cases: weights drawn from
# numpy seeds (rebuilt by the tests with argmax_weight), the reference's
# (index, value) stored.  tie: rows 10 and 40 equal and largest; nan: a NaN in
# x makes every row non-finite; large: M >= 4096 (the reference's OpenMP
# branch, serial with one thread); neg: every row negative.
ARGMAX_CASES = {
    "awq": dict(seed=31, M=300, K=512, gs=128, scheme=2),
    "gptq": dict(seed=32, M=200, K=256, gs=64, scheme=1),
    "awq_tie": dict(seed=33, M=64, K=128, gs=64, scheme=2, tie=(10, 40)),
    "awq_nan": dict(seed=34, M=48, K=128, gs=128, scheme=2, nan=True),
    "awq_large": dict(seed=35, M=4099, K=64, gs=32, scheme=2),
    "gptq_neg": dict(seed=36, M=96, K=128, gs=64, scheme=1, neg=True),
}


def argmax_weight(name: str):
    """(x, Int4Weight) of an argmax case, from its seed alone."""
    c = ARGMAX_CASES[name]
    rng = np.random.default_rng(c["seed"])
    M, K, gs = c["M"], c["K"], c["gs"]
    ng = K // gs
    q = rng.integers(0, 16, size=(M, K), dtype=np.uint8)
    s = orc.bf16_round(rng.uniform(0.005, 0.02, size=(M, ng)).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    if c.get("tie"):  # rows a and b equal, with q - 7 = 7 sign(x): the largest rows
        a, b = c["tie"]
        q[a] = np.where(x > 0, 14, 0).astype(np.uint8)
        q[b], s[b] = q[a], s[a]
    s16 = np.array([f32_to_f16bits_trunc(v) for v in s.reshape(-1)], np.uint16).reshape(M, ng)
    z16 = None
    if c["scheme"] == 1:
        z = rng.uniform(0.0, 0.05, size=(M, ng)).astype(np.float32)
        z16 = np.array([f32_to_f16bits_trunc(v) for v in z.reshape(-1)], np.uint16).reshape(M, ng)
    if c.get("neg"):
        x = -np.abs(x)
    if c.get("nan"):
        x[K // 3] = np.float32(np.nan)
    W = orc.Int4Weight(pack(q), s16, z16, M, K, gs, c["scheme"], 7 if c["scheme"] == 2 else 0)
    return x, W


def argmax_cases(R: orc.Reference) -> dict:
    out = {}
    for name in ARGMAX_CASES:
        x, W = argmax_weight(name)
        i, v = R.gemm_int4_argmax(x, W)
        out[name] = dict(index=np.int32(i), value=np.float32(v), x=x)
    return out


QLWC_CASE = dict(seed=21, layer=3, prefix="model.",
                 kw=dict(H=256, I=64, E=8, topk=2, gs=64, scheme=1, shared=True, shared_gate=True))


def qlwc_layer(O: orc.Oracle) -> orc.MoeLayer:
    return orc.make_layer(O, np.random.default_rng(QLWC_CASE["seed"]), **QLWC_CASE["kw"])


def qlwc_cases(O: orc.Oracle, qi) -> dict:
    import tempfile
    from pathlib import Path

    L = qlwc_layer(O)
    base = f"{QLWC_CASE['prefix']}layers.{QLWC_CASE['layer']}.mlp."
    items = []

    def int4(name, w):
        # flat arrays, as the reference's own quantizer hands them to write_qlwc
        items.append(dict(name=name, kind=1, shape=[w.M, w.K], q=w.q.tobytes(), scales=w.scales.reshape(-1),
                          zeros=None if w.zeros is None else w.zeros.reshape(-1)))

    for e, ex in enumerate(L.experts):
        for pn, w in (("gate_proj", ex.gate), ("up_proj", ex.up), ("down_proj", ex.down)):
            int4(f"{base}experts.{e}.{pn}.weight", w)
    for pn, w in (("gate_proj", L.shared.gate), ("up_proj", L.shared.up), ("down_proj", L.shared.down)):
        int4(f"{base}shared_expert.{pn}.weight", w)
    items.append(dict(name=base + "gate.weight", kind=0, shape=[L.E, L.H], pass_dtype=1, data=L.router_w.tobytes()))
    items.append(dict(name=base + "shared_expert_gate.weight", kind=0, shape=[1, L.H], pass_dtype=1,
                      data=L.shared_gate_w.tobytes()))
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "layer.qlwc"
        qi.write_qlwc(path, 1, QLWC_CASE["kw"]["gs"], items)  # scheme 1 = GPTQ-asym
        blob = np.frombuffer(path.read_bytes(), dtype=np.uint8).copy()
    return {"qlwc_gptq_shared_gate": dict(file=blob, input_sha256=np.array(digest(L.router_w, L.shared_gate_w)))}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("LLMOC_REFERENCE_TREE")
                    or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference"),
                    help="the reference tree (default: $LLMOC_REFERENCE_TREE, else a 'reference' folder "
                         "beside this repository)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "tools"))
    import quantize_int4 as qi  # the reference's quantizer, imported unmodified

    R = orc.Reference()
    O = orc.Oracle()
    assert R.max_threads() == 1, "run with OMP_NUM_THREADS=1 so the combine order is defined"
    groups = {"unit_cases": unit_cases(R), "quant_cases": quant_cases(qi),
              "router_cases": router_cases(R), "layer_cases": layer_cases(O, R),
              "qlwc_cases": qlwc_cases(O, qi), "argmax_cases": argmax_cases(R)}
    for gname, cases in groups.items():
        flat = {}
        for cname, d in cases.items():
            for k, v in d.items():
                flat[f"{cname}/{k}"] = np.asarray(v)
        path = os.path.join(HERE, f"{gname}.npz")
        np.savez_compressed(path, **flat)
        print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(cases)} cases)")


if __name__ == "__main__":
    main()
