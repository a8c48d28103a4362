"""Bounded device-side waits that run out, on the GPU, without a fault.

The NVLink collectives and the expert-parallel transport wait on flags that
other ranks raise.  A rank that never arrives must not leave a GPU waiting:
each wait spins for a budget of SM clocks, then sets bit 1 of its object's
error word and returns, and the stream goes on.  Here one rank of a two-rank
world (both in this process, on one GPU) makes its calls and the other never
does, so every flag the first waits for stays down.  The budget is cut to
about a millisecond so the test is quick; the library's default is 2^31
cycles (about a second).  Afterwards the stream has completed, the error
word reads 2, the idle rank's reads 0, and the device still runs work."""
import numpy as np
import pytest

import llmoc_b200 as L
import moe_gpu as G
import orc

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import ep  # noqa: E402

BUDGET = 2_000_000  # SM clocks per wait (~1 ms)


@pytest.fixture(scope="module", autouse=True)
def cuda_ready():
    assert torch.cuda.is_available()
    assert L.lib.llmoc_cuda_probe_available() == 1, L.lib.llmoc_cuda_status()
    yield


def _device_still_runs():
    a = torch.arange(1 << 20, device="cuda", dtype=torch.float32)
    assert float(a.sum()) == float((1 << 20) * ((1 << 20) - 1) / 2)


def test_collective_wait_gives_up_when_a_rank_never_arrives():
    cs = [L.Collective(2, r, 1 << 14, 0, export=False) for r in range(2)]
    L.Collective.connect_local(cs)
    for c in cs:
        assert L.lib.llmoc_collective_set_wait_cycles(c.handle, BUDGET) == 0
    assert L.lib.llmoc_collective_set_wait_cycles(cs[0].handle, 0) == 1  # a budget must be positive
    x = torch.ones(1024, device="cuda")
    cs[0].start(L.Collective.ALLREDUCE_SUM, x, 4096)   # rank 1 never starts
    cs[0].finish(L.Collective.ALLREDUCE_SUM, x, 4096, L.Collective.F32)
    torch.cuda.synchronize()  # the wait returned: the stream completes
    assert cs[0].error() == 2 and cs[1].error() == 0
    _device_still_runs()
    for c in cs:
        c.close()


def test_collective_finish_must_match_its_start():
    cs = [L.Collective(2, r, 1 << 14, 0, export=False) for r in range(2)]
    L.Collective.connect_local(cs)
    x = torch.zeros(1024, device="cuda")
    for c in cs:
        c.start(L.Collective.BROADCAST, x, 4096, 1)
    with pytest.raises(L.LlmocError, match="does not match"):  # other root
        cs[0].finish(L.Collective.BROADCAST, x, 4096, 0, 0)
    with pytest.raises(L.LlmocError, match="does not match"):  # other size
        cs[0].finish(L.Collective.BROADCAST, x, 2048, 0, 1)
    with pytest.raises(L.LlmocError, match="does not match"):  # other operation
        cs[0].finish(L.Collective.ALLTOALL, x, 4096, 0, 1)
    for c in cs:  # the matching finish still completes the step
        c.finish(L.Collective.BROADCAST, x, 4096, 0, 1)
    torch.cuda.synchronize()
    assert [c.error() for c in cs] == [0, 0]
    for c in cs:
        c.close()


def test_transport_waits_give_up_when_a_rank_never_sends(oracle):
    layer = orc.make_layer(oracle, np.random.default_rng(3), H=512, I=256, E=32, topk=8, gs=128)
    shards = [L.EpLayerShard.from_host_ep(layer, r, 2) for r in range(2)]
    trs = [L.EpTransport(2, r, layer.H, 16, layer.topk, 0, export=False) for r in range(2)]
    L.EpTransport.connect_local(trs)
    for t in trs:
        assert L.lib.llmoc_ep_transport_set_wait_cycles(t.handle, BUDGET) == 0
    step = ep.P2PStep(shards[0], trs[0], layer.H)
    X = G.bf16_dev(orc.make_tokens(np.random.default_rng(5), 16, layer.H))
    step.send(X, 16)       # rank 1 never sends: rank 0's serve waits for it in vain,
    step.serve(16)
    step.finish(X, 16)     # and its finish for rank 1's returned rows
    torch.cuda.synchronize()
    assert trs[0].error() == 2 and trs[1].error() == 0
    _device_still_runs()
    for t in trs:
        t.close()
    for s in shards:
        s.close()
