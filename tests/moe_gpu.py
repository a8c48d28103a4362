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
