"""contracts::ICollective over NVLink peer memory (llmoc_collective_*):
alltoall, allreduce_sum (fp32 and bf16) and broadcast for `world` ranks held
in one process on one GPU.  Every rank's start is issued before any finish, so
each wait is already satisfied in stream order; twelve consecutive steps run
through both staging parities and the waits for the peers' acknowledgements.
The cross-process path differs only in how the peers' buffers are opened
(CUDA IPC), which the expert-parallel transport's two-GPU test covers."""
import pytest

import llmoc_b200 as L

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
Coll = L.Collective


def _world(world, max_bytes=1 << 16):
    cs = [Coll(world, r, max_bytes, 0, export=False) for r in range(world)]
    Coll.connect_local(cs)
    return cs


def _step(cs, op, srcs, dsts, nbytes, dtype=0, root=0):
    for c, s in zip(cs, srcs):
        c.start(op, s, nbytes, root)
    for c, d in zip(cs, dsts):
        c.finish(op, d, nbytes, dtype, root)
    torch.cuda.synchronize()


@pytest.mark.parametrize("world", [2, 3])
def test_collectives_ranks_in_one_process(world):
    cs = _world(world)
    assert [c.world_size() for c in cs] == [world] * world
    g = torch.Generator(device="cuda").manual_seed(7)
    for step in range(4):
        # alltoall: chunk d of rank s's send arrives as chunk s of rank d's recv
        chunk = 4096 if step % 2 == 0 else 1000  # 1000: not a multiple of 16 bytes
        send = [torch.randint(0, 256, (world * chunk,), dtype=torch.uint8, device="cuda", generator=g)
                for _ in range(world)]
        recv = [torch.zeros_like(s) for s in send]
        _step(cs, Coll.ALLTOALL, send, recv, chunk)
        for d in range(world):
            for s in range(world):
                assert torch.equal(recv[d][s * chunk:(s + 1) * chunk], send[s][d * chunk:(d + 1) * chunk])
        # allreduce_sum, in place: fp32 sums in rank order, the same bits on every rank
        dtype = Coll.F32 if step % 2 == 0 else Coll.BF16
        tdt = torch.float32 if dtype == Coll.F32 else torch.bfloat16
        xs = [torch.randn(3001, device="cuda", generator=g).to(tdt) for _ in range(world)]
        want = xs[0].float()
        for s in range(1, world):
            want = want + xs[s].float()
        want = want.to(tdt)
        bufs = [x.clone() for x in xs]
        _step(cs, Coll.ALLREDUCE_SUM, bufs, bufs, bufs[0].numel() * bufs[0].element_size(), dtype)
        for b in bufs:
            assert torch.equal(b, want)
        # broadcast from a root that moves with the step
        root = step % world
        bufs = [torch.randn(2048, device="cuda", generator=g) for _ in range(world)]
        want = bufs[root].clone()
        _step(cs, Coll.BROADCAST, bufs, bufs, 2048 * 4, 0, root)
        for b in bufs:
            assert torch.equal(b, want)
    assert [c.error() for c in cs] == [0] * world
    for c in cs:
        c.close()


def test_collective_argument_checks():
    cs = _world(2, max_bytes=4096)
    x = torch.zeros(2048, device="cuda")
    with pytest.raises(L.LlmocError):  # larger than a staging slot
        cs[0].start(Coll.ALLREDUCE_SUM, x, 8192)
    with pytest.raises(L.LlmocError):  # no start before this finish
        cs[0].finish(Coll.ALLREDUCE_SUM, x, 4096, Coll.F32)
    with pytest.raises(L.LlmocError):  # root out of range
        cs[0].start(Coll.BROADCAST, x, 4096, 2)
    with pytest.raises(L.LlmocError):  # fp32 sum of a size that is not whole floats
        cs[0].start(Coll.ALLREDUCE_SUM, x, 4094)
        cs[0].finish(Coll.ALLREDUCE_SUM, x, 4094, Coll.F32)
    for c in cs:
        c.close()
