"""Expert-parallel MoE layer forward: one process per GPU, token dispatch and
combine as all-to-alls over torch.distributed (NCCL over NVLink on the GPU
box, gloo in the CPU tests).

The partition is the reference's: expert e lives on rank e % world
(DeviceMesh::owner_rank with EpShard::kMod, src/contracts/device_mesh.h:63-72),
as owner-local expert e // world; the router and the shared expert are
replicated; the transport is an all-to-all (ICollective::alltoall,
src/contracts/collective.h:13).  Every rank routes its own T tokens.  One
layer step:

    1. backend.dispatch   route, order the T*topk routed pairs by (owner,
                          owner-local expert, token, slot), gather their rows
    2. all-to-all         rows + owner-local ids in fixed-capacity regions:
                          region r of the send buffer holds the pairs for
                          owner r, up to T*topk of them, the rest marked
                          empty (id -1); equal splits, so the host never
                          reads a count and nothing waits for it
    3. backend.experts    grouped expert FFN over the received rows (empty
                          slots skipped)
    4. all-to-all         expert outputs back, region by region
    5. backend.combine    routed weights x returned rows (slot order) + shared

`DeviceBackend` runs 1, 3 and 5 through the C ABI (llmoc_moe_ep_*); any
object with the same three methods can stand in (the CPU tests use one built
on the oracle).

`P2PStep` runs the same step with the library's own NVLink transport
(llmoc_ep_p2p_*): rows are stored straight into the owners' receive buffers
(CUDA IPC peer pointers) and flagged per step, so the step has no host
synchronisation and no library collective; torch.distributed only exchanges
the IPC handles once.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist


def owner_rank(expert: int, world: int) -> int:
    """Rank that holds routed expert `expert` (the reference's kMod shard)."""
    return expert % world


def local_expert(expert: int, world: int) -> int:
    return expert // world


@dataclass
class EpTimes:
    """Device milliseconds of one step: local compute and the all-to-alls."""
    dispatch_ms: float = 0.0
    a2a_ms: float = 0.0
    experts_ms: float = 0.0
    combine_ms: float = 0.0
    sent_rows: int = 0
    recv_rows: int = 0


class _Marks:
    def __init__(self, enabled: bool):
        self.ev = [] if enabled else None
        self.on = enabled

    def mark(self):
        if self.on:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.ev.append(e)


def pack_regions(send_rows: torch.Tensor, send_expert: torch.Tensor, send_counts: torch.Tensor, cap: int):
    """The fixed-capacity send layout, on the device: the owner-ordered pairs
    of `send_rows` / `send_expert` placed at region owner * cap + (rank among
    the owner's pairs), every other slot marked empty (expert id -1).
    Returns (rows, expert ids, dest) with dest[i] the slot of pair i."""
    dev = send_rows.device
    P, H = send_rows.shape
    world = send_counts.numel()
    counts = send_counts.to(torch.int64)
    starts = torch.cumsum(counts, 0) - counts
    owner = torch.repeat_interleave(torch.arange(world, device=dev), counts, output_size=P)
    dest = owner * cap + (torch.arange(P, device=dev) - starts[owner])
    pad_rows = torch.empty((world * cap, H), dtype=send_rows.dtype, device=dev)
    pad_rows.index_copy_(0, dest, send_rows)
    pad_expert = torch.full((world * cap,), -1, dtype=send_expert.dtype, device=dev)
    pad_expert.index_copy_(0, dest, send_expert)
    return pad_rows, pad_expert, dest


def ep_forward(backend, X: torch.Tensor, T: int, group=None, times: Optional[EpTimes] = None,
               max_tokens: Optional[int] = None) -> torch.Tensor:
    """Y [T, H] (bf16) of this rank's T tokens; collective over `group`.

    The step never synchronises with the host: each routed pair's place in the
    send buffer (owner r's region r * cap, cap = max_tokens * topk, then its
    rank among the pairs for r) is computed on the device from the per-owner
    counts, and the all-to-alls move whole regions.  max_tokens bounds the T
    of every rank in this step and must be the same on all of them (default:
    T, when every rank passes the same T)."""
    H = X.shape[1]
    dev = X.device
    timed = times is not None and dev.type == "cuda"
    mk = _Marks(timed)
    mk.mark()
    send_rows, send_expert, send_counts = backend.dispatch(X, T)
    mk.mark()
    P = send_rows.shape[0]  # T * topk routed pairs, ordered by owner
    world = send_counts.numel()
    topk = P // T if T > 0 else 0
    cap = (max_tokens if max_tokens is not None else T) * topk
    if cap < P:
        raise ValueError(f"T = {T} is above max_tokens = {max_tokens}")
    pad_rows, pad_expert, dest = pack_regions(send_rows, send_expert, send_counts, cap)
    recv_rows = torch.empty_like(pad_rows)
    recv_expert = torch.empty_like(pad_expert)
    dist.all_to_all_single(recv_rows, pad_rows, group=group)
    dist.all_to_all_single(recv_expert, pad_expert, group=group)
    mk.mark()
    out_rows = backend.experts(recv_rows, recv_expert, world * cap, n_hint=P)
    mk.mark()
    ret_pad = torch.empty_like(out_rows)
    dist.all_to_all_single(ret_pad, out_rows, group=group)
    ret_rows = ret_pad.index_select(0, dest)
    mk.mark()
    Y = backend.combine(X, T, ret_rows)
    mk.mark()
    if times is not None:
        if timed:
            torch.cuda.current_stream().synchronize()
        times.sent_rows = P
        times.recv_rows = int((recv_expert >= 0).sum())  # the timing pass reads it; the step itself does not
        if timed:
            e = mk.ev
            times.dispatch_ms = e[0].elapsed_time(e[1])
            times.a2a_ms = e[1].elapsed_time(e[2]) + e[3].elapsed_time(e[4])
            times.experts_ms = e[2].elapsed_time(e[3])
            times.combine_ms = e[4].elapsed_time(e[5])
    return Y


@dataclass
class DeviceBackend:
    """The three local phases on this rank's GPU through the C ABI.

    `shard` is an llmoc_b200.EpLayerShard; buffers grow on demand (torch
    allocations outside the timed kernels)."""
    shard: object
    H: int
    topk: int
    stream: Optional[torch.cuda.Stream] = None
    _src: dict = field(default_factory=dict)
    _own: dict = field(default_factory=dict)

    def _buf(self, cache: dict, name: str, shape, dtype, dev):
        n = 1
        for d in shape:
            n *= d
        t = cache.get(name)
        if t is None or t.numel() < n or t.dtype != dtype:
            t = torch.empty(max(n, 1), dtype=dtype, device=dev)
            cache[name] = t
        return t[:n].view(*shape)

    def _stream(self):
        return self.stream if self.stream is not None else torch.cuda.current_stream()

    def dispatch(self, X, T):
        dev = X.device
        n = T * self.topk
        wsb = self.shard.source_workspace_bytes(T)
        self._src["wsb"] = wsb
        ws = self._buf(self._src, "ws", (wsb,), torch.uint8, dev)
        rows = self._buf(self._src, "rows", (n, self.H), torch.bfloat16, dev)
        eid = self._buf(self._src, "eid", (n,), torch.int32, dev)
        cnt = self._buf(self._src, "cnt", (self.shard.world,), torch.int32, dev)
        self.shard.dispatch(X, T, ws, wsb, rows, eid, cnt, self._stream())
        return rows, eid, cnt

    def experts(self, rows, expert, n, n_hint=None):
        """n received rows; with n_hint, the fixed-capacity layout (empty slots
        carry id -1, n_hint occupied slots expected)."""
        dev = rows.device
        out = self._buf(self._own, "out", (n, self.H), torch.bfloat16, dev)
        if n == 0:
            return out
        wsb = self.shard.owner_workspace_bytes(n)
        ws = self._buf(self._own, "ws", (wsb,), torch.uint8, dev)
        self.shard.experts(rows, expert, n, out, ws, wsb, self._stream(), n_hint=n_hint)
        return out

    def combine(self, X, T, ret_rows):
        Y = torch.empty((T, self.H), dtype=torch.bfloat16, device=X.device)
        self.shard.combine(X, T, ret_rows, Y, self._src["ws"], self._src["wsb"], self._stream())
        return Y


class P2PStep:
    """The expert-parallel layer step over the NVLink transport.

    `shard` is this rank's llmoc_b200.EpLayerShard, `transport` its
    llmoc_b200.EpTransport (connected: connect_p2p below, or
    EpTransport.connect_local for ranks of one process).  Each call of
    `forward` is one step (the sequence number advances); every rank calls it
    the same number of times."""

    def __init__(self, shard, transport, H: int, stream: Optional[torch.cuda.Stream] = None):
        self.shard, self.tr, self.H = shard, transport, H
        self.stream = stream
        self.seq = 0
        self.ws = None
        self.wsb = 0

    def _stream(self):
        return self.stream if self.stream is not None else torch.cuda.current_stream()

    def _ws(self, T, dev):
        need = self.tr.workspace_bytes(self.shard, T)
        if self.ws is None or self.ws.numel() < need:
            self.ws = torch.empty(need, dtype=torch.uint8, device=dev)
        self.wsb = self.ws.numel()

    def send(self, X, T):
        self.seq += 1
        self._ws(self.tr.max_tokens, X.device)
        self.tr.send(self.shard, X, T, self.seq, self.ws, self.wsb, self._stream())

    def serve(self, T):
        self.tr.serve(self.shard, T, self.seq, self.ws, self.wsb, self._stream())

    def finish(self, X, T, Y=None):
        if Y is None:
            Y = torch.empty((T, self.H), dtype=torch.bfloat16, device=X.device)
        self.tr.finish(self.shard, X, T, Y, self.seq, self.ws, self.wsb, self._stream())
        return Y

    def forward(self, X, T, times: Optional[EpTimes] = None):
        timed = times is not None
        mk = _Marks(timed)
        mk.mark()
        self.send(X, T)
        mk.mark()
        self.serve(T)
        mk.mark()
        Y = self.finish(X, T)
        mk.mark()
        if timed:
            torch.cuda.current_stream().synchronize()
            e = mk.ev
            times.dispatch_ms = e[0].elapsed_time(e[1])   # route + dispatch + push to the owners
            times.experts_ms = e[1].elapsed_time(e[2])    # wait for the sources + experts + push back
            times.combine_ms = e[2].elapsed_time(e[3])    # wait for the owners + combine
            times.a2a_ms = 0.0                            # inside the three phases (peer stores)
        return Y


def connect_p2p(transport, group=None) -> None:
    """Exchange the ranks' IPC handles (one all-gather) and open the peers:
    for an EpTransport or a Collective (anything with .ipc, .world and
    .connect(handles in rank order))."""
    import llmoc_b200 as L

    nb = int(L.lib.llmoc_ep_ipc_handle_bytes())
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    mine = torch.frombuffer(bytearray(bytes(transport.ipc)), dtype=torch.uint8).to(dev)
    allh = [torch.empty(nb, dtype=torch.uint8, device=dev) for _ in range(transport.world)]
    dist.all_gather(allh, mine, group=group)
    transport.connect(b"".join(bytes(h.cpu().numpy().tobytes()) for h in allh))
    dist.barrier(group=group)
