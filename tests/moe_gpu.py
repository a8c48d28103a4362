"""Helpers for the GPU parity tests: oracle-built layers on the device.

The CUDA path is always reached through the C ABI (llmoc_b200.py); torch only
allocates device buffers and moves bytes.
"""
from __future__ import annotations

import numpy as np

import llmoc_b200 as L
import orc


def torch():
    import torch as _t

    return _t


def bf16_dev(x: np.ndarray):
    """fp32 values that are exactly bf16 -> a cuda bf16 tensor (bit-preserving)."""
    t = torch()
    bits = orc.bf16_bits(x)
    assert np.array_equal(orc.bits_to_f32(bits), np.asarray(x, np.float32)), "not bf16-exact"
    return t.from_numpy(bits.view(np.int16).copy()).view(t.bfloat16).cuda()


def bf16_to_f32(y) -> np.ndarray:
    t = torch()
    return y.float().cpu().numpy().astype(np.float32)


def quality(y: np.ndarray, ref: np.ndarray):
    """(normwise max relative error, cosine similarity) of y against ref."""
    y = np.asarray(y, np.float64).reshape(-1)
    r = np.asarray(ref, np.float64).reshape(-1)
    denom = np.max(np.abs(r))
    mre = float(np.max(np.abs(y - r)) / denom) if denom > 0 else float(np.max(np.abs(y)))
    nr, ny = np.linalg.norm(r), np.linalg.norm(y)
    cos = float(np.dot(y, r) / (nr * ny)) if nr > 0 and ny > 0 else (1.0 if nr == ny else 0.0)
    return mre, cos


# Tolerance for bf16 layer outputs against the fp32 oracle:
MAX_REL = 1e-2
MIN_COS = 0.9999


class DevLayer:
    """An oracle layer uploaded through llmoc_moe_layer_create, with a workspace."""

    def __init__(self, layer: orc.MoeLayer, max_tokens: int):
        t = torch()
        self.host = layer
        self.dev = L.MoeLayer.from_host(layer, 0)
        self.max_tokens = max_tokens
        self.ws_bytes = self.dev.workspace_bytes(max_tokens)
        self.ws = t.empty(self.ws_bytes, dtype=t.uint8, device="cuda")

    def forward(self, X: np.ndarray):
        t = torch()
        T = X.shape[0]
        Xd = bf16_dev(X)
        Y = t.empty((T, self.host.H), dtype=t.bfloat16, device="cuda")
        ws_bytes = self.dev.workspace_bytes(T)
        self.dev.forward(Xd, T, Y, self.ws, ws_bytes, t.cuda.current_stream())
        t.cuda.synchronize()
        return Y, ws_bytes

    def route(self, X: np.ndarray):
        t = torch()
        T = X.shape[0]
        Xd = bf16_dev(X)
        ws_bytes = self.dev.workspace_bytes(T)
        self.dev.route(Xd, T, self.ws, ws_bytes, t.cuda.current_stream())
        t.cuda.synchronize()
        return self.views(T, ws_bytes)

    def views(self, T: int, ws_bytes: int) -> dict:
        """Routing outputs in the workspace, copied to numpy."""
        t = torch()
        v = self.dev.route_views(T, self.ws, ws_bytes)
        base = self.ws.data_ptr()
        kk, E, n_exp = self.dev.kk, self.host.E, self.dev.n_exp
        ld = E + (1 if getattr(self.host, "shared_gate_w", None) is not None else 0)  # + the shared gate's logit

        def grab(addr, n, dt):
            off = addr - base
            nbytes = n * 4
            return self.ws[off:off + nbytes].cpu().numpy().view(dt).copy()

        return dict(
            logits=grab(v.logits, T * ld, np.float32).reshape(T, ld),
            ids=grab(v.ids, T * kk, np.int32).reshape(T, kk),
            weights=grab(v.weights, T * kk, np.float32).reshape(T, kk),
            offsets=grab(v.offsets, n_exp + 1, np.int32),
            sorted=grab(v.sorted, T * kk, np.int32),
            inverse=grab(v.inverse, T * kk, np.int32),
            n_active=int(grab(v.n_active, 1, np.int32)[0]),
            error_flag=int(grab(v.error_flag, 1, np.int32)[0]),
        )

    def close(self):
        self.dev.close()


# ------------------------------------------------ full-size layers in HBM

class DeviceBuiltLayer:
    """A full-size layer whose experts are all distinct, drawn and quantized
    on the device (torch RNG, then llmoc_quantize_awq_sym: quant_awq_sym
    semantics with bf16-valued scales, the same quantizer the CPU tests pin to
    the reference's) and uploaded with llmoc_moe_layer_create_device.  The
    QLWC tensors stay on the device, so the oracle can be handed any expert's
    exact bytes (host_layer) without building every expert on the CPU."""

    def __init__(self, H, I, E, topk, gs, router=0, routed_scaling=1.0, shared=False, seed=0,
                 rw_add=None):
        t = torch()
        self.H, self.I, self.E, self.topk, self.gs = H, I, E, topk, gs
        self.router, self.routed_scaling, self.has_shared = router, routed_scaling, shared
        n_exp = E + (1 if shared else 0)
        g = t.Generator(device="cuda")
        g.manual_seed(seed)
        self.raw = {}
        for name, (M, K) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            q = t.empty((n_exp * M, K // 2), dtype=t.uint8, device="cuda")
            s = t.empty((n_exp * M, K // gs), dtype=t.int16, device="cuda")
            per = max(1, int(2 ** 27 // (M * K)))
            for e0 in range(0, n_exp, per):
                e1 = min(n_exp, e0 + per)
                W = (t.randn(((e1 - e0) * M, K), generator=g, device="cuda") * 0.02).to(t.bfloat16)
                L.quantize_awq_sym(W, (e1 - e0) * M, K, gs, True, q[e0 * M:e1 * M], s[e0 * M:e1 * M])
                del W
            self.raw[name] = (q, s, M, K)
        rw = t.randn((E, H), generator=g, device="cuda") * 0.02
        if rw_add is not None:
            rw = rw + rw_add
        self.router_w = rw.to(t.bfloat16)
        self.bias = (t.randn((E,), generator=g, device="cuda") * 0.1).float() if router == 1 else None
        views = []
        for e in range(n_exp):
            for name in ("gate", "up", "down"):
                q, s, M, K = self.raw[name]
                views.append(L.view(q.data_ptr() + e * M * (K // 2), s.data_ptr() + e * M * (K // gs) * 2,
                                    None, M, K, gs))
        desc = L.LayerDesc(H, I, E, topk, gs, L.SCHEME_AWQ_SYM, 7, router, routed_scaling, 1 if shared else 0, 1.0)
        t.cuda.synchronize()
        self.dev = L.MoeLayer.create(desc, self.router_w, self.bias, views[:3 * E],
                                     views[3 * E:] if shared else None, device=0, on_device=True)
        self.router_bits = self.router_w.view(t.int16).cpu().numpy().view(np.uint16).copy()
        self.bias_host = self.bias.cpu().numpy().copy() if self.bias is not None else None
        self._cache = {}

    def expert(self, e: int) -> orc.Expert:
        """Expert e's QLWC bytes, copied to the host (e == E: the shared expert)."""
        if e not in self._cache:
            ws = []
            for name in ("gate", "up", "down"):
                q, s, M, K = self.raw[name]
                ws.append(orc.Int4Weight(q[e * M:(e + 1) * M].cpu().numpy(),
                                         s[e * M:(e + 1) * M].cpu().numpy().view(np.uint16),
                                         None, M, K, self.gs, orc.SCHEME_AWQ_SYM, 7))
            self._cache[e] = orc.Expert(*ws)
        return self._cache[e]

    def host_layer(self, needed) -> orc.MoeLayer:
        """The layer as the oracle sees it, with the experts in `needed` (and the
        shared one) holding their real bytes; the others stand in with the
        first needed expert's (a token routed to one of them would not match)."""
        needed = sorted(set(int(e) for e in needed))
        filler = self.expert(needed[0])
        experts = [self.expert(e) if e in set(needed) else filler for e in range(self.E)]
        return orc.MoeLayer(self.H, self.I, self.E, self.topk, self.router_bits, experts, self.router,
                            self.bias_host, self.routed_scaling,
                            self.expert(self.E) if self.has_shared else None, 1.0)

    def route_layer(self) -> orc.MoeLayer:
        """The router part only (for oracle.moe_route: no expert is read)."""
        e0 = self.expert(0)
        return orc.MoeLayer(self.H, self.I, self.E, self.topk, self.router_bits, [e0] * self.E, self.router,
                            self.bias_host, self.routed_scaling, None, 1.0)

    def close(self):
        self.dev.close()
        self.raw = {}
        self._cache = {}


def cover_sample(ids: np.ndarray, n_spread: int = 64) -> np.ndarray:
    """Tokens to check against the oracle: n_spread spread evenly over the
    batch, plus a greedy cover so that every expert the batch routes to has at
    least one of its rows among them (every expert group is checked)."""
    T = ids.shape[0]
    chosen = set(np.unique(np.linspace(0, T - 1, min(T, n_spread)).astype(int)).tolist())
    covered = set(ids[sorted(chosen)].reshape(-1).tolist())
    need = set(ids.reshape(-1).tolist()) - covered
    first = {}
    for t in range(T):
        for e in ids[t]:
            first.setdefault(int(e), t)
    while need:
        e = min(need)
        t = first[e]
        chosen.add(t)
        need -= set(ids[t].tolist())
    return np.array(sorted(chosen))
