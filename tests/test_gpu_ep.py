"""Expert parallelism on the GPU: the llmoc_moe_ep_* phases through the C ABI.

Two shards of one layer on one GPU with the all-to-all done by hand (the
kernels of world = 2 without a second GPU), world = 1 against the plain
forward, the NVLink transport (llmoc_ep_p2p_*) with two ranks in one process
on one GPU (every wait already satisfied in stream order), and, where the box
has two GPUs, two ranks running ep.ep_forward over NCCL and two running the
NVLink transport.  Each rank's output is checked against the fp32 oracle of the
whole layer on that rank's tokens (bf16 output bar: normwise max relative
error 1e-2, cosine 0.9999)."""
import datetime
import os
import socket

import numpy as np
import pytest

import llmoc_b200 as L
import moe_gpu as G
import orc

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import ep  # noqa: E402

CFGS = {
    "qwen_like": dict(H=512, I=256, E=32, topk=8, gs=128),
    "glm_like_shared_sigmoid": dict(H=512, I=128, E=32, topk=8, gs=128, router=1, shared=True),
    "kimi_like_gs32": dict(H=448, I=128, E=48, topk=8, gs=32, router=1, routed_scaling=2.827, shared=True),
    "gptq_shared": dict(H=256, I=128, E=16, topk=4, gs=64, scheme=1, shared=True, shared_scale=0.75),
    "shared_gate": dict(H=256, I=128, E=16, topk=4, gs=64, scheme=1, shared=True, shared_gate=True),
}


@pytest.fixture(scope="module", autouse=True)
def cuda_ready():
    assert torch.cuda.is_available()
    assert L.lib.llmoc_cuda_probe_available() == 1, L.lib.llmoc_cuda_status()
    yield


def _check(Y, Yref, what):
    mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
    assert mre <= G.MAX_REL and cos >= G.MIN_COS, (what, mre, cos)


def _backends(layer, world):
    shards = [L.EpLayerShard.from_host_ep(layer, r, world) for r in range(world)]
    return shards, [ep.DeviceBackend(s, layer.H, layer.topk) for s in shards]


def _emulated_forward(backends, Xs):
    """ep_forward for every rank in one process: the all-to-alls as copies."""
    world = len(backends)
    sends = [b.dispatch(X, X.shape[0]) for b, X in zip(backends, Xs)]
    counts = [s[2].cpu().numpy().astype(int) for s in sends]
    bounds = [np.concatenate([[0], np.cumsum(c)]) for c in counts]
    outs = []
    for r in range(world):  # rows and ids from every source, source order
        rows = torch.cat([sends[s][0][bounds[s][r]:bounds[s][r + 1]] for s in range(world)])
        eid = torch.cat([sends[s][1][bounds[s][r]:bounds[s][r + 1]] for s in range(world)])
        outs.append((backends[r].experts(rows.contiguous(), eid.contiguous(), rows.shape[0]).clone(),
                     [counts[s][r] for s in range(world)]))
    Ys = []
    for s in range(world):  # back to the source, in its send order (by owner rank)
        parts = []
        for r in range(world):
            out, per_src = outs[r]
            o = int(sum(per_src[:s]))
            parts.append(out[o:o + per_src[s]])
        Ys.append(backends[s].combine(Xs[s], Xs[s].shape[0], torch.cat(parts).contiguous()))
    torch.cuda.synchronize()
    return Ys, counts


@pytest.mark.parametrize("name", list(CFGS))
@pytest.mark.parametrize("T", [5, 40, 200])
def test_two_shards_on_one_gpu(oracle, name, T):
    layer = orc.make_layer(oracle, np.random.default_rng(3), **CFGS[name])
    shards, bks = _backends(layer, 2)
    Xh = [orc.make_tokens(np.random.default_rng(50 + r), T + 3 * r, layer.H) for r in range(2)]
    Ys, counts = _emulated_forward(bks, [G.bf16_dev(X) for X in Xh])
    for r in range(2):
        Yref, ids, _, _ = oracle.moe_layer_forward(layer, Xh[r])
        _check(Ys[r], Yref, (name, T, r))
        # per-owner counts equal the oracle's routing
        want = np.bincount((ids % 2).reshape(-1), minlength=2)
        assert np.array_equal(counts[r], want)
    for s in shards:
        s.close()


def _emulated_forward_padded(backends, Xs, max_tokens):
    """ep_forward's fixed-capacity exchange for every rank in one process: the
    regions packed on the device (ep.pack_regions), the all-to-alls as copies
    of whole regions, the owners through llmoc_moe_ep_experts_padded."""
    world = len(backends)
    sends = [b.dispatch(X, X.shape[0]) for b, X in zip(backends, Xs)]
    topk = sends[0][0].shape[0] // Xs[0].shape[0]
    cap = max_tokens * topk
    packed = [ep.pack_regions(r, e, c, cap) for r, e, c in sends]
    outs = []
    for r in range(world):  # owner r receives region r of every source, source order
        rows = torch.cat([packed[s][0][r * cap:(r + 1) * cap] for s in range(world)]).contiguous()
        eid = torch.cat([packed[s][1][r * cap:(r + 1) * cap] for s in range(world)]).contiguous()
        outs.append(backends[r].experts(rows, eid, world * cap, n_hint=sends[r][0].shape[0]).clone())
    Ys = []
    for s in range(world):  # region s of every owner back to source s
        ret = torch.cat([outs[r][s * cap:(s + 1) * cap] for r in range(world)])
        Ys.append(backends[s].combine(Xs[s], Xs[s].shape[0], ret.index_select(0, packed[s][2]).contiguous()))
    torch.cuda.synchronize()
    return Ys


@pytest.mark.parametrize("name", list(CFGS))
@pytest.mark.parametrize("T", [5, 40])
def test_fixed_capacity_exchange_matches(oracle, name, T):
    """The host-free NCCL step's layout: every routed pair placed in its
    owner's region on the device, empty slots (id -1) skipped by the owners.
    Outputs equal the count-based exchange bit for bit (same expert groups,
    same work items) and the oracle within the layer tolerance."""
    layer = orc.make_layer(oracle, np.random.default_rng(3), **CFGS[name])
    shards, bks = _backends(layer, 2)
    Xh = [orc.make_tokens(np.random.default_rng(50 + r), T + 3 * r, layer.H) for r in range(2)]
    Xd = [G.bf16_dev(X) for X in Xh]
    Yp = _emulated_forward_padded(bks, Xd, T + 3)
    Yc, _ = _emulated_forward(bks, Xd)
    for r in range(2):
        assert torch.equal(Yp[r], Yc[r]), (name, T, r)
        _check(Yp[r], oracle.moe_layer_forward(layer, Xh[r])[0], (name, T, r))
    for s in shards:
        s.close()


@pytest.mark.parametrize("name", ["qwen_like", "glm_like_shared_sigmoid"])
def test_world_one_matches_plain_forward(oracle, name):
    layer = orc.make_layer(oracle, np.random.default_rng(4), **CFGS[name])
    shards, bks = _backends(layer, 1)
    X = orc.make_tokens(np.random.default_rng(9), 64, layer.H)
    Ys, _ = _emulated_forward(bks, [G.bf16_dev(X)])
    dl = G.DevLayer(layer, 64)
    Y, _ = dl.forward(X)
    mre, cos = G.quality(G.bf16_to_f32(Ys[0]), G.bf16_to_f32(Y))
    assert mre <= G.MAX_REL and cos >= G.MIN_COS
    _check(Ys[0], oracle.moe_layer_forward(layer, X)[0], name)
    dl.close()
    shards[0].close()


def test_shard_refuses_the_single_gpu_forward(oracle):
    layer = orc.make_layer(oracle, np.random.default_rng(5), **CFGS["qwen_like"])
    s = L.EpLayerShard.from_host_ep(layer, 0, 2)
    ws = torch.empty(s.workspace_bytes(4) + 1024, dtype=torch.uint8, device="cuda")
    X = G.bf16_dev(orc.make_tokens(np.random.default_rng(1), 4, layer.H))
    Y = torch.empty((4, layer.H), dtype=torch.bfloat16, device="cuda")
    rc = L.lib.llmoc_moe_forward(s.handle, X.data_ptr(), 4, Y.data_ptr(), ws.data_ptr(), ws.numel(), None)
    assert rc == 1 and b"expert-parallel" in L.lib.llmoc_last_error()
    with pytest.raises(L.LlmocError):  # world must divide n_experts
        L.EpLayerShard.from_host_ep(layer, 0, 3)
    s.close()


def _p2p_emulated(layer, world, Xs, steps):
    """`steps` layer steps of every rank through the NVLink transport in one
    process: sends, then serves, then finishes, all on one stream."""
    shards = [L.EpLayerShard.from_host_ep(layer, r, world) for r in range(world)]
    Tmax = max(X.shape[0] for X in Xs)
    trs = [L.EpTransport(world, r, layer.H, Tmax, layer.topk, 0, export=False) for r in range(world)]
    L.EpTransport.connect_local(trs)
    st = [ep.P2PStep(shards[r], trs[r], layer.H) for r in range(world)]
    outs = []
    for _ in range(steps):
        for r in range(world):
            st[r].send(Xs[r], Xs[r].shape[0])
        for r in range(world):
            st[r].serve(Xs[r].shape[0])
        Ys = [st[r].finish(Xs[r], Xs[r].shape[0]) for r in range(world)]
        torch.cuda.synchronize()
        outs.append(Ys)
    errs = [t.error() for t in trs]
    for t in trs:
        t.close()
    for s in shards:
        s.close()
    return outs, errs


@pytest.mark.parametrize("name", list(CFGS))
@pytest.mark.parametrize("T", [5, 40, 200])
def test_p2p_transport_two_ranks_one_gpu(oracle, name, T):
    """The NVLink transport's kernels for world = 2 (receive slots per source,
    empty-slot marking, return to the send offsets, double-buffered parities):
    three steps, each rank's output against the oracle, and every step's
    output bitwise equal to the first (the parities alternate)."""
    layer = orc.make_layer(oracle, np.random.default_rng(3), **CFGS[name])
    Xh = [orc.make_tokens(np.random.default_rng(50 + r), T + 3 * r, layer.H) for r in range(2)]
    outs, errs = _p2p_emulated(layer, 2, [G.bf16_dev(X) for X in Xh], 3)
    assert errs == [0, 0]
    for r in range(2):
        _check(outs[0][r], oracle.moe_layer_forward(layer, Xh[r])[0], (name, T, r))
        for k in (1, 2):
            assert torch.equal(outs[k][r], outs[0][r]), (name, T, r, k)


@pytest.mark.parametrize("name", ["qwen_like", "glm_like_shared_sigmoid"])
@pytest.mark.parametrize("T", [5, 40])
def test_p2p_transport_four_ranks_one_gpu(oracle, name, T):
    """world = 4 through the NVLink transport in one process (sends, then
    serves, then finishes, one stream): T = 5 takes the one-CTA routing of the
    dispatch, T = 40 the top-k kernel writing the owner keys and the
    permutation with the per-owner tail."""
    layer = orc.make_layer(oracle, np.random.default_rng(6), **CFGS[name])
    Xh = [orc.make_tokens(np.random.default_rng(80 + r), T + r, layer.H) for r in range(4)]
    outs, errs = _p2p_emulated(layer, 4, [G.bf16_dev(X) for X in Xh], 2)
    assert errs == [0, 0, 0, 0]
    for r in range(4):
        _check(outs[0][r], oracle.moe_layer_forward(layer, Xh[r])[0], (name, T, r))
        assert torch.equal(outs[1][r], outs[0][r]), (name, T, r)


def test_p2p_transport_skewed_to_one_owner(oracle):
    """Every routed slot lands on rank 0's experts (a selection bias of -16 on
    the odd ones): rank 0 serves twice the rows that its own tokens x topk
    predict, so its K-split GEMMs walk more work items than their grid has
    rows of CTAs; rank 1 serves no routed rows at all."""
    layer = orc.make_layer(oracle, np.random.default_rng(11), **CFGS["glm_like_shared_sigmoid"])
    layer.bias[1::2] -= np.float32(16.0)
    Xh = [orc.make_tokens(np.random.default_rng(70 + r), 40, layer.H) for r in range(2)]
    outs, errs = _p2p_emulated(layer, 2, [G.bf16_dev(X) for X in Xh], 2)
    assert errs == [0, 0]
    for r in range(2):
        Yref, ids, _, _ = oracle.moe_layer_forward(layer, Xh[r])
        assert np.all(ids % 2 == 0)
        _check(outs[0][r], Yref, ("skew", r))
        assert torch.equal(outs[1][r], outs[0][r])


def test_p2p_transport_world_one(oracle):
    """world = 1: the transport loops back to the rank itself."""
    layer = orc.make_layer(oracle, np.random.default_rng(8), **CFGS["glm_like_shared_sigmoid"])
    X = orc.make_tokens(np.random.default_rng(11), 24, layer.H)
    outs, errs = _p2p_emulated(layer, 1, [G.bf16_dev(X)], 2)
    assert errs == [0]
    _check(outs[1][0], oracle.moe_layer_forward(layer, X)[0], "world1")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, name, T, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist = torch.distributed
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        oracle = orc.Oracle()
        layer = orc.make_layer(oracle, np.random.default_rng(3), **CFGS[name])
        shard = L.EpLayerShard.from_host_ep(layer, rank, world, device=rank)
        bk = ep.DeviceBackend(shard, layer.H, layer.topk)
        Xh = orc.make_tokens(np.random.default_rng(70 + rank), T + rank, layer.H)
        X = G.bf16_dev(Xh).to(f"cuda:{rank}")
        Y = ep.ep_forward(bk, X, X.shape[0], max_tokens=T + world - 1)  # ragged T, one bound on every rank
        torch.cuda.synchronize()
        mre, cos = G.quality(G.bf16_to_f32(Y), oracle.moe_layer_forward(layer, Xh)[0])
        q.put((rank, mre, cos))
        dist.barrier()
        dist.destroy_process_group()
        shard.close()
    except Exception as e:
        q.put((rank, repr(e), None))


@pytest.mark.parametrize("name", ["qwen_like", "kimi_like_gs32"])
def test_two_nccl_ranks(name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_nccl_worker, args=(r, 2, port, name, 33, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, mre, cos in res:
        assert cos is not None, (rank, mre)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (rank, mre, cos)


def _p2p_worker(rank, world, port, name, T, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist = torch.distributed
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        oracle = orc.Oracle()
        layer = orc.make_layer(oracle, np.random.default_rng(3), **CFGS[name])
        shard = L.EpLayerShard.from_host_ep(layer, rank, world, device=rank)
        tr = L.EpTransport(world, rank, layer.H, T + world, layer.topk, rank)
        ep.connect_p2p(tr)
        step = ep.P2PStep(shard, tr, layer.H)
        Xh = orc.make_tokens(np.random.default_rng(70 + rank), T + rank, layer.H)
        X = G.bf16_dev(Xh).to(f"cuda:{rank}")
        Ys = [step.forward(X, X.shape[0]) for _ in range(3)]
        torch.cuda.synchronize()
        err = tr.error()
        same = all(torch.equal(Ys[0], y) for y in Ys[1:])
        mre, cos = G.quality(G.bf16_to_f32(Ys[-1]), oracle.moe_layer_forward(layer, Xh)[0])
        q.put((rank, mre, cos, err, same))
        dist.barrier()
        tr.close()
        dist.destroy_process_group()
        shard.close()
    except Exception as e:
        q.put((rank, repr(e), None, None, None))


@pytest.mark.parametrize("name", ["qwen_like", "kimi_like_gs32"])
def test_p2p_transport_two_gpus(name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_p2p_worker, args=(r, 2, port, name, 33, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, mre, cos, err, same in res:
        assert cos is not None, (rank, mre)
        assert err == 0 and same, (rank, err, same)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (rank, mre, cos)
