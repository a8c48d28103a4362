"""ctypes front-end for the CPU checkers (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this
module.  It wraps two shared libraries built by ``oracle/Makefile``:

* ``oracle/libmoe_oracle.so`` — the plain-C restatement (``moe_oracle.c``) of
  llm-on-cpu's INT4 MoE expert-FFN arithmetic (file:line citations live there);
* ``oracle/_ref/libllmoc_ref.so`` — the reference's own ``src/hal`` CPU operators
  compiled from its sources plus ``ref_shim.cpp`` (optional: present when the
  reference tree was available at build time).

All arrays are numpy; nothing here touches a GPU.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_SO = os.path.join(HERE, "libmoe_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libllmoc_ref.so")

SCHEME_GPTQ_ASYM = 1
SCHEME_AWQ_SYM = 2
ROUTER_SOFTMAX = 0
ROUTER_SIGMOID_BIAS = 1

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


class Int4ViewC(C.Structure):
    """Field-for-field qlwc::Int4View (src/weights/qlwc_store.h:17-27), minus scales_f32."""

    _fields_ = [
        ("qweight", C.c_void_p),
        ("scales", C.c_void_p),
        ("zeros", C.c_void_p),
        ("M", C.c_int),
        ("K", C.c_int),
        ("group_size", C.c_int),
        ("scheme", C.c_int),
        ("awq_zp", C.c_int),
    ]


class ExpertC(C.Structure):
    _fields_ = [("gate", Int4ViewC), ("up", Int4ViewC), ("down", Int4ViewC)]


class LayerC(C.Structure):
    _fields_ = [
        ("H", C.c_int),
        ("I", C.c_int),
        ("E", C.c_int),
        ("topk", C.c_int),
        ("router", C.c_int),
        ("router_w", C.c_void_p),
        ("bias", C.c_void_p),
        ("routed_scaling", C.c_float),
        ("experts", C.POINTER(ExpertC)),
        ("shared", C.POINTER(ExpertC)),
        ("shared_scale", C.c_float),
        ("shared_gate_w", C.c_void_p),
    ]


@dataclass
class Int4Weight:
    """Host INT4 tensor in the QLWC layout (q | fp16 scales | fp16 zeros)."""

    q: np.ndarray  # uint8 [M, ceil(K/2)]
    scales: np.ndarray  # uint16 [M, ng]
    zeros: Optional[np.ndarray]  # uint16 [M, ng] or None
    M: int
    K: int
    group_size: int
    scheme: int = SCHEME_AWQ_SYM
    awq_zp: int = 7

    def view(self) -> Int4ViewC:
        return Int4ViewC(
            self.q.ctypes.data,
            self.scales.ctypes.data,
            self.zeros.ctypes.data if self.zeros is not None else None,
            self.M,
            self.K,
            self.group_size,
            self.scheme,
            self.awq_zp,
        )


@dataclass
class Expert:
    gate: Int4Weight
    up: Int4Weight
    down: Int4Weight

    def c(self) -> ExpertC:
        return ExpertC(self.gate.view(), self.up.view(), self.down.view())


@dataclass
class MoeLayer:
    """One MoE layer's host weights (router bf16 [E,H], E experts, optional shared)."""

    H: int
    I: int
    E: int
    topk: int
    router_w: np.ndarray  # uint16 bf16 bits [E, H]
    experts: List[Expert]
    router: int = ROUTER_SOFTMAX
    bias: Optional[np.ndarray] = None  # float32 [E]
    routed_scaling: float = 1.0
    shared: Optional[Expert] = None
    shared_scale: float = 1.0
    shared_gate_w: Optional[np.ndarray] = None  # uint16 bf16 bits [H]: per-token sigmoid shared weight
    _keep: list = field(default_factory=list, repr=False)

    def c(self) -> LayerC:
        arr = (ExpertC * self.E)(*[e.c() for e in self.experts])
        sh = C.pointer(self.shared.c()) if self.shared is not None else None
        self._keep = [arr, sh]
        return LayerC(
            self.H,
            self.I,
            self.E,
            self.topk,
            self.router,
            self.router_w.ctypes.data,
            self.bias.ctypes.data if self.bias is not None else None,
            float(self.routed_scaling),
            C.cast(arr, C.POINTER(ExpertC)),
            sh,
            float(self.shared_scale),
            self.shared_gate_w.ctypes.data if self.shared_gate_w is not None else None,
        )


def _load(path: str) -> C.CDLL:
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built (run `make -C oracle liborc ref`)")
    return C.CDLL(path)


class Oracle:
    """The plain-C restatement (libmoe_oracle.so)."""

    prefix = "orc_"

    def __init__(self, path: str = ORC_SO):
        self.lib = _load(path)
        L, p = self.lib, self.prefix
        g = lambda n: getattr(L, p + n)  # noqa: E731
        self._gemm_int4 = g("gemm_int4")
        self._gemm_int4.argtypes = [_f32p, C.POINTER(Int4ViewC), _f32p]
        self._gemm_int4.restype = None
        self._argmax = g("gemm_int4_argmax")
        self._argmax.argtypes = [_f32p, C.POINTER(Int4ViewC), C.POINTER(C.c_int32), C.POINTER(C.c_float)]
        self._argmax.restype = None
        self._gemm_int4_batch = g("gemm_int4_batch")
        self._gemm_int4_batch.argtypes = [_f32p, C.c_int, C.POINTER(Int4ViewC), _f32p]
        self._gemm_int4_batch.restype = None
        self._dequant_row = g("dequant_int4_row")
        self._dequant_row.argtypes = [C.POINTER(Int4ViewC), C.c_int, _f32p]
        self._dequant_row.restype = C.c_int
        self._gemm_bias_free = g("gemm_bias_free")
        self._gemm_bias_free.argtypes = [_f32p, _u16p, _f32p, C.c_int, C.c_int, C.c_int]
        self._gemm_bias_free.restype = None
        self._silu = g("silu_and_mul")
        self._silu.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        self._silu.restype = None
        self._layer = g("moe_layer_forward")
        self._layer.restype = None
        if p == "orc_":
            self._layer.argtypes = [C.POINTER(LayerC), _f32p, C.c_int, _f32p, _i32p, _f32p, C.c_void_p]
            self._route_softmax = L.orc_route_softmax
            self._route_softmax.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p, C.c_void_p]
            self._route_softmax.restype = C.c_int
            self._route_sig = L.orc_route_sigmoid_bias
            self._route_sig.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_float, _i32p, _f32p]
            self._route_sig.restype = None
            self._permute = L.orc_permute
            self._permute.argtypes = [_i32p, C.c_int, C.c_int, C.c_int, _i32p, _i32p, _i32p]
            self._permute.restype = None
            self._qawq = L.orc_quant_awq_sym
            self._qawq.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _u8p, _u16p]
            self._qawq.restype = None
            self._qgptq = L.orc_quant_gptq_asym
            self._qgptq.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _u8p, _u16p, _u16p]
            self._qgptq.restype = None
            self._route_all = L.orc_moe_route
            self._route_all.argtypes = [C.POINTER(LayerC), _f32p, C.c_int, _f32p, _i32p, _f32p]
            self._route_all.restype = None
            self._routed = L.orc_moe_ffn_routed
            self._routed.argtypes = [_f32p, C.c_int, C.c_int, C.POINTER(ExpertC), _f32p, C.c_int,
                                     C.c_void_p, C.c_float, _f32p]
            self._routed.restype = None
            for n in ("f16_to_f32", "bf16_to_f32"):
                fn = getattr(L, "orc_" + n)
                fn.argtypes = [C.c_uint16]
                fn.restype = C.c_float
            L.orc_f32_to_f16_rne.argtypes = [C.c_float]
            L.orc_f32_to_f16_rne.restype = C.c_uint16
            L.orc_f32_to_bf16.argtypes = [C.c_float]
            L.orc_f32_to_bf16.restype = C.c_uint16
        else:
            self._layer.argtypes = [C.POINTER(LayerC), _f32p, C.c_int, _f32p, _i32p, _f32p]

    # --- INT4 operators -------------------------------------------------
    def gemm_int4(self, x: np.ndarray, W: Int4Weight) -> np.ndarray:
        y = np.empty(W.M, np.float32)
        v = W.view()
        self._gemm_int4(np.ascontiguousarray(x, np.float32), C.byref(v), y)
        return y

    def gemm_int4_argmax(self, x: np.ndarray, W: Int4Weight):
        """hal::gemm_int4_argmax: (index, value) of the largest row of W . x."""
        i, v = C.c_int32(), C.c_float()
        wv = W.view()
        self._argmax(np.ascontiguousarray(x, np.float32), C.byref(wv), C.byref(i), C.byref(v))
        return int(i.value), np.float32(v.value)

    def gemm_int4_batch(self, X: np.ndarray, W: Int4Weight) -> np.ndarray:
        X = np.ascontiguousarray(X, np.float32)
        Y = np.empty((X.shape[0], W.M), np.float32)
        v = W.view()
        self._gemm_int4_batch(X, X.shape[0], C.byref(v), Y)
        return Y

    def dequant_matrix(self, W: Int4Weight) -> np.ndarray:
        out = np.empty((W.M, W.K), np.float32)
        v = W.view()
        for r in range(W.M):
            row = np.empty(W.K, np.float32)
            assert self._dequant_row(C.byref(v), r, row) == 0
            out[r] = row
        return out

    def gemm_bias_free(self, x: np.ndarray, Wbits: np.ndarray, is_f16: bool = False) -> np.ndarray:
        M, K = Wbits.shape
        y = np.empty(M, np.float32)
        self._gemm_bias_free(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(Wbits), y, M, K,
                             int(is_f16))
        return y

    def silu_and_mul(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        out = np.empty_like(g, dtype=np.float32)
        self._silu(np.ascontiguousarray(g, np.float32), np.ascontiguousarray(u, np.float32), out, g.size)
        return out

    # --- the layer --------------------------------------------------------
    def moe_layer_forward(self, layer: MoeLayer, X: np.ndarray):
        X = np.ascontiguousarray(X, np.float32)
        T = X.shape[0]
        Y = np.empty((T, layer.H), np.float32)
        ids = np.empty((T, layer.topk), np.int32)
        w = np.empty((T, layer.topk), np.float32)
        lc = layer.c()
        if self.prefix == "orc_":
            ties = np.zeros(T, np.int32)
            self._layer(C.byref(lc), X, T, Y, ids, w, ties.ctypes.data)
            return Y, ids, w, ties
        self._layer(C.byref(lc), X, T, Y, ids, w)
        return Y, ids, w, None

    # --- oracle-only helpers --------------------------------------------
    def moe_route(self, layer: MoeLayer, X: np.ndarray):
        """Router logits [T,E], ids and weights [T,topk] of every token (the
        routing of moe_layer_forward; tokens in parallel, no expert reads)."""
        X = np.ascontiguousarray(X, np.float32)
        T = X.shape[0]
        logits = np.empty((T, layer.E), np.float32)
        ids = np.empty((T, layer.topk), np.int32)
        w = np.empty((T, layer.topk), np.float32)
        lc = layer.c()
        self._route_all(C.byref(lc), X, T, logits, ids, w)
        return logits, ids, w


    def route_softmax(self, logits: np.ndarray, k: int):
        E = logits.size
        ids = np.empty(k, np.int32)
        w = np.empty(k, np.float32)
        tie = self._route_softmax(np.ascontiguousarray(logits, np.float32), E, k, ids, w, None)
        return ids, w, bool(tie)

    def route_sigmoid_bias(self, logits: np.ndarray, bias: np.ndarray, k: int, scaling: float):
        E = logits.size
        ids = np.empty(k, np.int32)
        w = np.empty(k, np.float32)
        self._route_sig(np.ascontiguousarray(logits, np.float32), np.ascontiguousarray(bias, np.float32),
                        E, k, float(scaling), ids, w)
        return ids, w

    def permute(self, ids: np.ndarray, n_exp: int):
        ids = np.ascontiguousarray(ids, np.int32)
        T, kk = ids.shape
        off = np.empty(n_exp + 1, np.int32)
        srt = np.empty(T * kk, np.int32)
        inv = np.empty(T * kk, np.int32)
        self._permute(ids, T, kk, n_exp, off, srt, inv)
        return off, srt, inv

    def quant_awq_sym(self, W: np.ndarray, gs: int, bf16_scale: bool = False) -> Int4Weight:
        W = np.ascontiguousarray(W, np.float32)
        M, K = W.shape
        assert K % gs == 0, "quant_awq_sym needs K % group_size == 0 (quantize_int4.py:153)"
        q = np.empty((M, K // 2), np.uint8)
        s = np.empty((M, K // gs), np.uint16)
        self._qawq(W, M, K, gs, int(bf16_scale), q, s)
        return Int4Weight(q, s, None, M, K, gs, SCHEME_AWQ_SYM, 7)

    def quant_gptq_asym(self, W: np.ndarray, gs: int) -> Int4Weight:
        W = np.ascontiguousarray(W, np.float32)
        M, K = W.shape
        assert K % gs == 0, "quant_gptq_asym needs K % group_size == 0 (quantize_int4.py:130)"
        q = np.empty((M, K // 2), np.uint8)
        s = np.empty((M, K // gs), np.uint16)
        z = np.empty((M, K // gs), np.uint16)
        self._qgptq(W, M, K, gs, q, s, z)
        return Int4Weight(q, s, z, M, K, gs, SCHEME_GPTQ_ASYM, 0)

    def moe_ffn_routed(self, x, H, I, experts: List[Expert], w, shared: Optional[Expert], shared_scale):
        arr = (ExpertC * len(experts))(*[e.c() for e in experts])
        y = np.empty(H, np.float32)
        sh = C.pointer(shared.c()) if shared is not None else None
        self._routed(np.ascontiguousarray(x, np.float32), H, I, arr, np.ascontiguousarray(w, np.float32),
                     len(experts), C.cast(sh, C.c_void_p) if sh is not None else None, float(shared_scale), y)
        return y


class Reference(Oracle):
    """The reference's own CPU operators (oracle/_ref/libllmoc_ref.so)."""

    prefix = "ref_"

    def __init__(self, path: str = REF_SO):
        super().__init__(path)
        self.lib.ref_max_threads.restype = C.c_int

    def max_threads(self) -> int:
        return int(self.lib.ref_max_threads())


def ref_available() -> bool:
    return os.path.exists(REF_SO)


# ---------------------------------------------------------------------------
# seeded synthetic inputs (the BASELINE configs' shapes and distributions)
# ---------------------------------------------------------------------------

def bf16_round(a: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16, returned as fp32 values."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def make_layer(orc: Oracle, rng: np.random.Generator, H: int, I: int, E: int, topk: int, gs: int,
               router: int = ROUTER_SOFTMAX, routed_scaling: float = 1.0, shared: bool = False,
               shared_scale: float = 1.0, scheme: int = SCHEME_AWQ_SYM, wstd: float = 0.02,
               n_real: Optional[int] = None, shared_gate: bool = False) -> MoeLayer:
    """Seeded synthetic MoE layer: W ~ N(0, wstd^2) rounded to bf16, quantized
    per expert with quant_awq_sym semantics (bf16-valued scales) or GPTQ-asym.
    ``n_real`` < E makes only the first n_real experts distinct and re-uses
    them cyclically for the rest (keeps big-E layers cheap to build)."""
    def q(M, K):
        W = bf16_round(rng.standard_normal((M, K), dtype=np.float32) * np.float32(wstd))
        if scheme == SCHEME_AWQ_SYM:
            return orc.quant_awq_sym(W, gs, bf16_scale=True)
        return orc.quant_gptq_asym(W, gs)

    nr = E if n_real is None else n_real
    base = [Expert(q(I, H), q(I, H), q(H, I)) for _ in range(nr)]
    experts = [base[e % nr] for e in range(E)]
    rw = bf16_bits(rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02))
    bias = None
    if router == ROUTER_SIGMOID_BIAS:
        bias = (rng.standard_normal(E, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    sh = Expert(q(I, H), q(I, H), q(H, I)) if shared else None
    sg = bf16_bits(rng.standard_normal(H, dtype=np.float32) * np.float32(0.05)) if shared and shared_gate else None
    return MoeLayer(H, I, E, topk, rw, experts, router, bias, routed_scaling, sh, shared_scale, sg)


def make_tokens(rng: np.random.Generator, T: int, H: int) -> np.ndarray:
    """Hidden states N(0,1) rounded to bf16 (returned as fp32 values)."""
    return bf16_round(rng.standard_normal((T, H), dtype=np.float32))
