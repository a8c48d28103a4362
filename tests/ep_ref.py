"""An oracle-backed stand-in for the three device phases of the expert-
parallel forward (ep.DeviceBackend), with the same contract: expert e is owned
by rank e % world as local expert e // world; pairs are sent ordered by
(owner, local expert, token, slot); rows travel as bf16.  Test
infrastructure: the routing and the expert FFNs are the CPU oracle's."""
from __future__ import annotations

import numpy as np
import torch

import orc


class OracleBackend:
    def __init__(self, oracle: orc.Oracle, layer: orc.MoeLayer, rank: int, world: int):
        assert layer.E % world == 0
        self.o, self.layer, self.rank, self.world = oracle, layer, rank, world
        self.e_loc = layer.E // world

    def dispatch(self, X: torch.Tensor, T: int):
        L = self.layer
        Xf = X.float().numpy()
        _, ids, w, _ = self.o.moe_layer_forward(L, Xf)  # the routing of the whole layer
        key = ((ids % self.world) * self.e_loc + ids // self.world).reshape(-1)
        order = np.argsort(key, kind="stable")  # (owner, local expert), then (t, j)
        self.order, self.w = order, w
        rows = X[torch.from_numpy(order // L.topk)]
        eid = torch.from_numpy((key[order] % self.e_loc).astype(np.int32))
        cnt = torch.from_numpy(np.bincount(key // self.e_loc, minlength=self.world).astype(np.int32))
        return rows.contiguous(), eid, cnt

    def experts(self, rows: torch.Tensor, expert: torch.Tensor, n: int, n_hint=None):
        L = self.layer
        out = np.zeros((n, L.H), np.float32)
        R = rows.float().numpy()
        for r in range(n):
            if not 0 <= int(expert[r]) < self.e_loc:
                continue  # an empty slot of the fixed-capacity layout
            e = int(expert[r]) * self.world + self.rank
            out[r] = self.o.moe_ffn_routed(R[r], L.H, L.I, [L.experts[e]], np.ones(1, np.float32), None, 0.0)
        return torch.from_numpy(orc.bf16_round(out)).to(torch.bfloat16)

    def combine(self, X: torch.Tensor, T: int, ret_rows: torch.Tensor):
        L = self.layer
        inv = np.empty_like(self.order)
        inv[self.order] = np.arange(self.order.size)
        ret = ret_rows.float().numpy()
        Y = np.zeros((T, L.H), np.float32)
        Xf = X.float().numpy()
        for t in range(T):
            for j in range(L.topk):
                Y[t] += np.float32(self.w[t, j]) * ret[inv[t * L.topk + j]]
            if L.shared is not None:
                Y[t] += self.o.moe_ffn_routed(Xf[t], L.H, L.I, [], np.zeros(0, np.float32), L.shared,
                                              L.shared_scale)
        return torch.from_numpy(orc.bf16_round(Y)).to(torch.bfloat16)
