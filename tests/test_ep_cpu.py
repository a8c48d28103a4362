"""Expert-parallel plumbing (llm-on-cpu_b200/ep.py) across two gloo ranks on
CPU: per-peer counts, the row and expert-id all-to-alls, the return trip and
the combine order, with an oracle-backed stand-in for the device phases.
Each rank's output is checked against the single-process oracle forward of
the whole layer on that rank's tokens."""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import ep  # noqa: E402
import orc  # noqa: E402
from ep_ref import OracleBackend  # noqa: E402

CFGS = {
    "softmax": dict(H=128, I=64, E=8, topk=2, gs=32),
    "sigmoid_shared": dict(H=128, I=64, E=8, topk=3, gs=32, router=1, routed_scaling=2.5, shared=True,
                           shared_scale=0.5),
}
MAX_REL, MIN_COS = 1e-2, 0.9999


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, name, T, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        oracle = orc.Oracle()
        layer = orc.make_layer(oracle, np.random.default_rng(11), **CFGS[name])  # identical on every rank
        Tr = T + rank  # ragged token counts across ranks
        X = orc.make_tokens(np.random.default_rng(100 + rank), Tr, layer.H)
        Xt = torch.from_numpy(X).to(torch.bfloat16)
        times = ep.EpTimes()
        Y = ep.ep_forward(OracleBackend(oracle, layer, rank, world), Xt, Tr, times=times,
                          max_tokens=T + world - 1)  # the ragged counts' bound, the same on every rank
        Yref = oracle.moe_layer_forward(layer, X)[0]
        y, r = Y.float().numpy().reshape(-1).astype(np.float64), Yref.reshape(-1).astype(np.float64)
        mre = float(np.max(np.abs(y - r)) / np.max(np.abs(r)))
        cos = float(y @ r / (np.linalg.norm(y) * np.linalg.norm(r)))
        q.put((rank, mre, cos, times.sent_rows, times.recv_rows))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), None, None, None))


@pytest.mark.parametrize("name", list(CFGS))
def test_ep_forward_two_gloo_ranks(name):
    world, T = 2, 9
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, name, T, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    topk = CFGS[name]["topk"]
    sent = recv = 0
    for rank, mre, cos, s, rcv in res:
        assert cos is not None, f"rank {rank}: {mre}"
        assert mre <= MAX_REL and cos >= MIN_COS, (rank, mre, cos)
        assert s == (T + rank) * topk
        sent, recv = sent + s, recv + rcv
    assert sent == recv  # every routed pair crossed exactly once


def test_owner_map_is_the_references_kmod():
    # DeviceMesh::owner_rank with EpShard::kMod: ((e % ep) + ep) % ep
    for world in (1, 2, 4, 8):
        for e in range(64):
            assert ep.owner_rank(e, world) == e % world
            assert ep.local_expert(e, world) * world + ep.owner_rank(e, world) == e


class _FakeEnd:
    """Stands in for an EpTransport / Collective: its IPC handle is the rank
    number repeated; connect records what it was given."""

    def __init__(self, rank, world, nb):
        self.world, self.ipc, self.got = world, bytes([rank + 1]) * nb, None

    def connect(self, handles):
        self.got = handles


def _connect_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        import llmoc_b200 as L

        nb = int(L.lib.llmoc_ep_ipc_handle_bytes())
        end = _FakeEnd(rank, world, nb)
        ep.connect_p2p(end)
        q.put((rank, end.got == b"".join(bytes([r + 1]) * nb for r in range(world)), nb))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), None))


def test_connect_exchanges_handles_in_rank_order():
    """ep.connect_p2p over two gloo ranks: every rank's connect receives all
    IPC handles, rank 0's first (the layout llmoc_ep_transport_connect and
    llmoc_collective_connect read)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_connect_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    for rank, ok, nb in res:
        assert ok is True, (rank, ok)
        assert nb == 64  # sizeof(cudaIpcMemHandle_t)
