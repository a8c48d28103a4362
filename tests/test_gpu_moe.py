"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Bars (north star): expert ids, permutation and dequantised weights bit-exact;
router logits bit-exact (the ids depend on them); bf16 layer outputs within
normwise max relative error 1e-2 and cosine >= 0.9999 of the fp32 oracle.
"""
import ctypes as C

import numpy as np
import pytest

import llmoc_b200 as L
import moe_gpu as G
import orc

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def cuda_ready():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    assert L.lib.llmoc_cuda_probe_available() == 1, L.lib.llmoc_cuda_status()
    assert L.lib.llmoc_cuda_enable(0) == 1
    yield


SMALL = {
    "qwen_like": dict(H=512, I=256, E=32, topk=8, gs=128),
    "glm_like_shared_sigmoid": dict(H=512, I=128, E=32, topk=8, gs=128, router=1, shared=True),
    "kimi_like_gs32": dict(H=448, I=128, E=48, topk=8, gs=32, router=1, routed_scaling=2.827,
                           shared=True),
    "gptq_shared": dict(H=256, I=128, E=16, topk=4, gs=64, scheme=1, shared=True, shared_scale=0.75),
    "odd_k_chunks": dict(H=288, I=96, E=12, topk=3, gs=32),
    # Qwen3.6-style shared expert weighted per token by sigmoid(shared_expert_gate . x)
    "shared_gate_gptq": dict(H=512, I=128, E=32, topk=8, gs=128, scheme=1, shared=True, shared_gate=True),
}


def build(oracle, name, seed, max_tokens):
    rng = np.random.default_rng(seed)
    layer = orc.make_layer(oracle, rng, **SMALL[name])
    return G.DevLayer(layer, max_tokens), rng


@pytest.mark.parametrize("name", list(SMALL))
def test_dequant_bit_exact(oracle, name):
    dl, _ = build(oracle, name, 1, 1)
    h = dl.host
    for e in (0, h.E - 1) + ((h.E,) if h.shared is not None else ()):
        ex = h.experts[e] if e < h.E else h.shared
        for p, w in enumerate((ex.gate, ex.up, ex.down)):
            out = torch.empty((w.M, w.K), dtype=torch.float32, device="cuda")
            dl.dev.dequant(e, p, out)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            ref = oracle.dequant_matrix(w)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (e, p)
    dl.close()


@pytest.mark.parametrize("gs,bf16_scale", [(32, True), (128, True), (128, False)])
def test_device_quantizer_matches_reference_quantizer(oracle, gs, bf16_scale):
    rng = np.random.default_rng(gs)
    M, K = 96, 1024
    W = orc.bf16_round(rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02))
    W[3, :gs] = 0.0  # an all-zero group takes the 1e-8 floor
    ref = oracle.quant_awq_sym(W, gs, bf16_scale)
    q = torch.empty((M, K // 2), dtype=torch.uint8, device="cuda")
    s = torch.empty((M, K // gs), dtype=torch.int16, device="cuda")
    L.quantize_awq_sym(G.bf16_dev(W), M, K, gs, bf16_scale, q, s)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), ref.q)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), ref.scales)


def check_routing(oracle, dl, X, v, sample=None):
    """Logits, ids and weights of the tokens in `sample` (default: all) against
    the oracle; the permutation of all tokens against the canonical order."""
    h = dl.host
    T = X.shape[0]
    sample = range(T) if sample is None else sample
    for t in sample:
        ref_logits = oracle.gemm_bias_free(X[t], h.router_w)
        assert np.array_equal(v["logits"][t, :h.E].view(np.uint32), ref_logits.view(np.uint32)), t
        if h.router == orc.ROUTER_SOFTMAX:
            ids, w, _ = oracle.route_softmax(ref_logits, h.topk)
        else:
            ids, w = oracle.route_sigmoid_bias(ref_logits, h.bias, h.topk, h.routed_scaling)
        assert np.array_equal(v["ids"][t, :h.topk], ids), t
        np.testing.assert_allclose(v["weights"][t, :h.topk], w, rtol=2e-6, atol=0)
        if h.shared is not None:
            assert v["ids"][t, h.topk] == h.E
            if h.shared_gate_w is None:
                assert v["weights"][t, h.topk] == np.float32(h.shared_scale)
            else:  # the gate's logit is bitwise the reference's; the sigmoid within a few ulp
                gl = oracle.gemm_bias_free(X[t], h.shared_gate_w[None, :])
                assert np.array_equal(v["logits"][t, h.E:h.E + 1].view(np.uint32), gl.view(np.uint32)), t
                want = np.float32(1.0) / (np.float32(1.0) + np.exp(-gl.astype(np.float32)))
                np.testing.assert_allclose(v["weights"][t, h.topk], want[0], rtol=2e-6, atol=0)
    off, srt, inv = oracle.permute(v["ids"], dl.dev.n_exp)
    assert np.array_equal(v["offsets"], off)
    assert np.array_equal(v["sorted"], srt)
    assert np.array_equal(v["inverse"], inv)
    assert v["n_active"] == int(np.count_nonzero(np.diff(off)))


@pytest.mark.parametrize("name", list(SMALL))
@pytest.mark.parametrize("T", [1, 7, 64, 133])
def test_routing_bit_exact(oracle, name, T):
    dl, rng = build(oracle, name, 2, T)
    X = orc.make_tokens(rng, T, dl.host.H)
    v = dl.route(X)
    check_routing(oracle, dl, X, v)
    dl.close()


@pytest.mark.parametrize("T,E,H", [(3, 40, 768), (77, 40, 768), (20, 70, 768), (77, 40, 1024), (150, 40, 768),
                                   (800, 40, 768), (2400, 40, 768)])
def test_router_tiles_bit_exact(oracle, T, E, H):
    """Router logits of every token bitwise equal to the reference's AVX2 order
    on each tile shape (T <= 8: one CTA per expert row; 8 < T < 128: 8 x 16
    tiles, T = 77 and, with a partial expert tile, E = 70 at T = 20, and with
    1024-wide K chunks at H = 1024; T >= 128:
    8 x 16, 16 x 16 and 32 x 32 tiles as the grid grows, T = 150, 800, 2400),
    with partial token and expert tiles (T not a multiple of 32) and a
    non-finite activation (that token's logits become 0, as in the reference)."""
    rng = np.random.default_rng(40 + T)
    layer = orc.make_layer(oracle, rng, H=H, I=128, E=E, topk=4, gs=128)
    X = orc.make_tokens(rng, T, H)
    X[T // 2, 5] = np.inf
    dl = G.DevLayer(layer, T)
    _, ws_bytes = dl.forward(X)
    v = dl.views(T, ws_bytes)
    for t in range(T):
        ref = oracle.gemm_bias_free(X[t], layer.router_w)
        assert np.array_equal(v["logits"][t].view(np.uint32), ref.view(np.uint32)), t
    assert np.all(v["logits"][T // 2] == 0)
    dl.close()


@pytest.mark.parametrize("name", list(SMALL))
@pytest.mark.parametrize("T", [1, 5, 40, 129])
def test_layer_matches_oracle(oracle, name, T):
    dl, rng = build(oracle, name, 3, T)
    X = orc.make_tokens(rng, T, dl.host.H)
    Y, ws_bytes = dl.forward(X)
    Yref, ids, w, _ = oracle.moe_layer_forward(dl.host, X)
    v = dl.views(T, ws_bytes)
    assert v["error_flag"] == 0
    assert np.array_equal(v["ids"][:, :dl.host.topk], ids)
    mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
    assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
    for t in range(T):  # every token on its own, too
        mre_t, cos_t = G.quality(G.bf16_to_f32(Y[t]), Yref[t])
        assert mre_t <= 2 * G.MAX_REL and cos_t >= 0.999, (t, mre_t, cos_t)
    dl.close()


def test_single_token_forward_on_a_stale_workspace(oracle):
    """The fused one-token forward (one launch, grid-wide barriers whose words
    live in the workspace, tagged per launch) on a workspace full of random
    bytes, then again on what the previous launches left: every output
    matches the oracle, the same token twice gives the same bits, and the
    routing views are the canonical ones of one token."""
    dl, rng = build(oracle, "glm_like_shared_sigmoid", 11, 1)
    g = torch.Generator(device="cuda").manual_seed(5)
    dl.ws.copy_(torch.randint(0, 256, dl.ws.shape, generator=g, device="cuda", dtype=torch.int32).to(torch.uint8))
    Xs = [orc.make_tokens(rng, 1, dl.host.H) for _ in range(3)]
    outs = []
    for X in Xs + [Xs[0]]:
        Y, ws_bytes = dl.forward(X)
        Yref, ids, w, _ = oracle.moe_layer_forward(dl.host, X)
        v = dl.views(1, ws_bytes)
        assert v["error_flag"] == 0
        assert np.array_equal(v["ids"][:, :dl.host.topk], ids)
        kk = dl.dev.kk
        order = np.argsort(v["ids"][0], kind="stable")
        assert np.array_equal(v["sorted"], order)
        assert np.array_equal(v["inverse"][order], np.arange(kk))
        assert np.array_equal(v["offsets"], np.searchsorted(np.sort(v["ids"][0]), np.arange(dl.dev.n_exp + 1)))
        assert v["n_active"] == kk
        mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
        outs.append(Y.clone())
    assert torch.equal(outs[0], outs[3])
    dl.close()


@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("scheme", [orc.SCHEME_AWQ_SYM, orc.SCHEME_GPTQ_ASYM])
def test_single_token_every_group_size_and_scheme(oracle, gs, scheme):
    """Every instance of the fused one-token kernel (group 32 / 64 / 128 x AWQ /
    GPTQ; the GPTQ layers with the sigmoid+bias router and a shared expert):
    ids bit-exact, output within the tolerance of the oracle."""
    gptq = scheme == orc.SCHEME_GPTQ_ASYM
    rng = np.random.default_rng(40 + gs + scheme)
    layer = orc.make_layer(oracle, rng, H=512, I=256, E=32, topk=8, gs=gs, scheme=scheme,
                           router=orc.ROUTER_SIGMOID_BIAS if gptq else orc.ROUTER_SOFTMAX, shared=gptq)
    dl = G.DevLayer(layer, 1)
    for _ in range(2):
        X = orc.make_tokens(rng, 1, layer.H)
        Y, ws_bytes = dl.forward(X)
        Yref, ids, _, _ = oracle.moe_layer_forward(layer, X)
        v = dl.views(1, ws_bytes)
        assert v["error_flag"] == 0
        assert np.array_equal(v["ids"][:, :layer.topk], ids)
        mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (gs, scheme, mre, cos)
    dl.close()


def test_single_token_forward_replayed_from_a_cuda_graph(oracle):
    """The fused one-token forward captured into a CUDA graph and replayed (the
    launch's parameters, its epoch included, frozen): every replay correct and
    clean -- each launch's last CTA leaves the barrier's counters at zero, so a
    replay that finds its own tag in the workspace needs no reset."""
    dl, rng = build(oracle, "qwen_like", 13, 1)
    X = orc.make_tokens(rng, 1, dl.host.H)
    Xd = G.bf16_dev(X)
    Y = torch.empty((1, dl.host.H), dtype=torch.bfloat16, device="cuda")
    ws_bytes = dl.dev.workspace_bytes(1)
    dl.dev.forward(Xd, 1, Y, dl.ws, ws_bytes, torch.cuda.current_stream())  # first use outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dl.dev.forward(Xd, 1, Y, dl.ws, ws_bytes, torch.cuda.current_stream())
    Yref, _, _, _ = oracle.moe_layer_forward(dl.host, X)
    for _ in range(4):
        Y.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert dl.views(1, ws_bytes)["error_flag"] == 0
        mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
    del g
    dl.close()


def test_single_token_barrier_budget_runs_out(oracle):
    """A barrier wait of the fused one-token kernel that runs out of its
    budget (cut to one SM clock, so a CTA that arrives before the others gives
    up): bit 2 of the error word is set, the launch ends, the device still
    runs work, and with the default budget back the next forward is correct
    and clean."""
    dl, rng = build(oracle, "qwen_like", 12, 1)
    X = orc.make_tokens(rng, 1, dl.host.H)
    dl.dev.set_wait_cycles(1)
    _, ws_bytes = dl.forward(X)
    assert dl.views(1, ws_bytes)["error_flag"] & 4
    a = torch.arange(1 << 20, device="cuda", dtype=torch.float32)
    assert float(a.sum()) == float((1 << 20) * ((1 << 20) - 1) / 2)
    dl.dev.set_wait_cycles(1 << 31)
    Y, ws_bytes = dl.forward(X)
    assert dl.views(1, ws_bytes)["error_flag"] == 0
    Yref, _, _, _ = oracle.moe_layer_forward(dl.host, X)
    mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
    assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
    dl.close()


def test_zero_tokens_is_a_no_op(oracle):
    dl, _ = build(oracle, "qwen_like", 4, 4)
    assert L.lib.llmoc_moe_forward(dl.dev.handle, None, 0, None, None, 0, None) == 0
    dl.close()


def test_workspace_too_small_is_rejected(oracle):
    dl, rng = build(oracle, "qwen_like", 5, 8)
    X = G.bf16_dev(orc.make_tokens(rng, 8, dl.host.H))
    Y = torch.empty((8, dl.host.H), dtype=torch.bfloat16, device="cuda")
    st = L.lib.llmoc_moe_forward(dl.dev.handle, X.data_ptr(), 8, Y.data_ptr(), dl.ws.data_ptr(),
                                 dl.dev.workspace_bytes(8) - 1, None)
    assert st == 7
    dl.close()


@pytest.mark.parametrize("T", [200, 600])
def test_skewed_routing_hot_expert(oracle, T):
    """Every token prefers the same few experts (one expert gets all T pairs):
    exercises multi-chunk work items of one expert (T = 600: items of 256,
    256 and 88 rows on the tcgen05 path) and empty experts."""
    rng = np.random.default_rng(6)
    layer = orc.make_layer(oracle, rng, H=512, I=256, E=32, topk=4, gs=128)
    rw = orc.bits_to_f32(layer.router_w)
    rw[:4] += 0.5  # a strong shared component towards experts 0..3
    layer.router_w = orc.bf16_bits(rw)
    X = np.abs(orc.make_tokens(rng, T, 512))
    dl = G.DevLayer(layer, T)
    Y, ws_bytes = dl.forward(X)
    v = dl.views(T, ws_bytes)
    counts = np.diff(v["offsets"])
    assert counts.max() == T and (counts == 0).sum() > 0
    Yref, ids, _, _ = oracle.moe_layer_forward(layer, X)
    assert np.array_equal(v["ids"], ids)
    mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
    assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
    dl.close()


@pytest.mark.parametrize("T,in_place", [(1, False), (1, True), (5, False), (5, True), (150, False), (150, True)])
def test_forward_residual(oracle, T, in_place):
    """Y = R + MoE(X) through llmoc_moe_forward_residual: separate R, and the
    in-place residual stream (R = Y = X, the decoder's h += moe(h)); decode and
    prefill paths, and the fused one-token kernel (T = 1).  Compared with R +
    the oracle's fp32 layer output, and with
    the plain forward's output plus R."""
    rng = np.random.default_rng(30 + T)
    layer = orc.make_layer(oracle, rng, H=512, I=256, E=32, topk=8, gs=128)
    X = orc.make_tokens(rng, T, 512)
    R = X if in_place else orc.make_tokens(rng, T, 512)
    dl = G.DevLayer(layer, T)
    Xd = G.bf16_dev(X)
    Rd = Xd if in_place else G.bf16_dev(R)
    Y = Xd if in_place else torch.empty_like(Xd)
    ws_bytes = dl.dev.workspace_bytes(T)
    dl.dev.forward_residual(Xd, T, Rd, Y, dl.ws, ws_bytes, torch.cuda.current_stream())
    torch.cuda.synchronize()
    Yref, _, _, _ = oracle.moe_layer_forward(layer, X)
    # Y carries one bf16 rounding of R + MoE(X): judged against R + the oracle
    mre, cos = G.quality(G.bf16_to_f32(Y), R + Yref)
    assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
    # same arithmetic as the plain forward followed by an fp32 add of R
    Y2, _ = dl.forward(X)
    y2 = G.bf16_to_f32(Y2)
    err = np.abs(G.bf16_to_f32(Y) - (R + y2)).max()
    assert err <= 2.0 ** -6 * (np.abs(R).max() + np.abs(y2).max()), err
    dl.close()


def test_layer_from_qlwc_file(oracle, tmp_path):
    """A layer loaded by llmoc_moe_layer_create_qlwc from a file the
    reference's own tools/quantize_int4.py wrote (GPTQ experts, shared expert
    with its per-token gate): routing bit-exact and outputs within tolerance of
    the oracle on the same weights."""
    import make_golden as mg
    import test_qlwc

    path = test_qlwc.qlwc_file(tmp_path)
    layer = mg.qlwc_layer(oracle)
    kw = mg.QLWC_CASE["kw"]
    desc = L.LayerDesc(kw["H"], kw["I"], kw["E"], kw["topk"], kw["gs"], L.SCHEME_GPTQ_ASYM, 0,
                       L.ROUTER_SOFTMAX, 1.0, 1, 1.0)
    dev = L.MoeLayer.from_qlwc(path, mg.QLWC_CASE["prefix"], mg.QLWC_CASE["layer"], desc, 0)
    T = 24
    X = orc.make_tokens(np.random.default_rng(5), T, kw["H"])
    Xd = G.bf16_dev(X)
    Y = torch.empty((T, kw["H"]), dtype=torch.bfloat16, device="cuda")
    ws_bytes = dev.workspace_bytes(T)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    dev.forward(Xd, T, Y, ws, ws_bytes, torch.cuda.current_stream())
    torch.cuda.synchronize()
    v = dev.route_views(T, ws, ws_bytes)
    ids = ws[v.ids - ws.data_ptr(): v.ids - ws.data_ptr() + 4 * T * (kw["topk"] + 1)].cpu().numpy().view(np.int32)
    Yref, ids_ref, _, _ = oracle.moe_layer_forward(layer, X)
    assert np.array_equal(ids.reshape(T, -1)[:, :kw["topk"]], ids_ref)
    mre, cos = G.quality(G.bf16_to_f32(Y), Yref)
    assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
    # the desc must agree with the file
    bad = L.LayerDesc(kw["H"], kw["I"], kw["E"] + 1, kw["topk"], kw["gs"], L.SCHEME_GPTQ_ASYM, 0,
                      L.ROUTER_SOFTMAX, 1.0, 1, 1.0)
    with pytest.raises(L.LlmocError):
        L.MoeLayer.from_qlwc(path, mg.QLWC_CASE["prefix"], mg.QLWC_CASE["layer"], bad, 0)
    dev.close()


def test_zero_weights_give_zero_output(oracle):
    rng = np.random.default_rng(7)
    layer = orc.make_layer(oracle, rng, H=256, I=128, E=8, topk=2, gs=64, wstd=0.0)
    dl = G.DevLayer(layer, 3)
    Y, _ = dl.forward(orc.make_tokens(rng, 3, 256))
    assert float(Y.float().abs().max()) == 0.0
    dl.close()


# ------------------------------------------------------------- full sizes

FULL = {
    # Qwen3-30B-A3B layer
    "qwen3_30b_a3b": dict(H=2048, I=768, E=128, topk=8, gs=128),
    # GLM-4.5-Air layer (sigmoid + bias, shared expert)
    "glm45_air": dict(H=4096, I=1408, E=128, topk=8, gs=128, router=1, shared=True),
    # Kimi-K2 layer (gs 32, 384 experts, scaling 2.827, shared)
    "kimi_k2": dict(H=7168, I=2048, E=384, topk=8, gs=32, router=1, routed_scaling=2.827, shared=True),
}


def _check_full(oracle, dl, X, Xd, T):
    """Routing of every token against the oracle (logits bitwise, ids exact,
    weights within 2e-6), the permutation against the canonical order, and the
    outputs of >= 64 tokens that cover every expert group the batch uses."""
    Y = torch.empty((T, dl.H), dtype=torch.bfloat16, device="cuda")
    ws_bytes = dl.dev.workspace_bytes(T)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    dl.dev.forward(Xd, T, Y, ws, ws_bytes, torch.cuda.current_stream())
    torch.cuda.synchronize()
    v = dl.dev.route_views(T, ws, ws_bytes)
    base = ws.data_ptr()

    def grab(addr, n, dt):
        return ws[addr - base: addr - base + 4 * n].cpu().numpy().view(dt).copy()

    kk, n_exp = dl.dev.kk, dl.dev.n_exp
    assert int(grab(v.error_flag, 1, np.int32)[0]) == 0
    logits = grab(v.logits, T * dl.E, np.float32).reshape(T, dl.E)
    ids = grab(v.ids, T * kk, np.int32).reshape(T, kk)
    w = grab(v.weights, T * kk, np.float32).reshape(T, kk)
    ref_logits, ref_ids, ref_w = oracle.moe_route(dl.route_layer(), X)
    assert np.array_equal(logits.view(np.uint32), ref_logits.view(np.uint32))
    assert np.array_equal(ids[:, :dl.topk], ref_ids)
    np.testing.assert_allclose(w[:, :dl.topk], ref_w, rtol=2e-6, atol=0)
    if dl.has_shared:
        assert np.all(ids[:, dl.topk] == dl.E)
    off, srt, inv = oracle.permute(ids, n_exp)
    assert np.array_equal(grab(v.offsets, n_exp + 1, np.int32), off)
    assert np.array_equal(grab(v.sorted, T * kk, np.int32), srt)
    assert np.array_equal(grab(v.inverse, T * kk, np.int32), inv)
    sample = G.cover_sample(ids[:, :dl.topk])
    assert len(sample) >= min(T, 64)
    assert set(ids[sample, :dl.topk].reshape(-1)) == set(ids[:, :dl.topk].reshape(-1))
    layer = dl.host_layer(ids[sample, :dl.topk].reshape(-1))
    Yref, ids_s, _, _ = oracle.moe_layer_forward(layer, X[sample])
    assert np.array_equal(ids_s, ref_ids[sample])
    got = G.bf16_to_f32(Y[torch.as_tensor(sample, device="cuda")])
    mre, cos = G.quality(got, Yref)
    assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
    for i in range(len(sample)):  # every sampled token on its own, too
        mre_t, cos_t = G.quality(got[i], Yref[i])
        assert mre_t <= 2 * G.MAX_REL and cos_t >= 0.999, (int(sample[i]), mre_t, cos_t)
    return ids


@pytest.mark.parametrize("name,T", [("qwen3_30b_a3b", 1), ("qwen3_30b_a3b", 8), ("qwen3_30b_a3b", 64),
                                    ("qwen3_30b_a3b", 512), ("glm45_air", 1), ("glm45_air", 64), ("glm45_air", 512), ("glm45_air", 1024),
                                    ("glm45_air", 4096), ("kimi_k2", 1), ("kimi_k2", 64),
                                    ("kimi_k2", 1024), ("kimi_k2", 8192)])
def test_full_size_layer(oracle, name, T):
    """The BASELINE shapes and token counts the bench times, every expert
    distinct (no expert shares another's bytes, so an indexing slip in the
    expert table, the repacked arena or the work list cannot pass): routing
    bit-exact for every token, outputs on a sample covering every expert group
    (each token's output depends on that token alone)."""
    dl = G.DeviceBuiltLayer(**FULL[name], seed=100 + T)
    g = torch.Generator(device="cuda").manual_seed(7 + T)
    Xd = torch.randn((T, dl.H), generator=g, device="cuda").to(torch.bfloat16)
    X = G.bf16_to_f32(Xd)
    _check_full(oracle, dl, X, Xd, T)
    dl.close()


def test_zipf_skewed_residual_stack(oracle):
    """Four distinct Qwen3-30B-A3B-shape layers with router rows pushed towards
    a Zipf(1.1) popularity (BASELINE config 3's skew: a few hot experts with
    long groups, many cold or empty ones), run as a decoder stack through
    llmoc_moe_forward_residual in place (h += moe(h)), T = 16.  Each layer's
    output is checked against its input plus the oracle's layer output on that
    same input (read back from the device), and the routing against the
    oracle's, so an error in any layer of the stack shows up where it is.
    The routed part is checked on its own (the plain forward of the same input
    against the oracle), then the residual forward against input + that output
    (one bf16 rounding of an fp32 sum apart)."""
    E, H, T, n_layers = 128, 2048, 16, 4
    g = torch.Generator(device="cuda").manual_seed(11)
    v = torch.randn(H, generator=g, device="cuda")
    v = v / v.norm()
    ranks = torch.arange(1, E + 1, device="cuda", dtype=torch.float32)
    boost = 0.2 * ranks ** -1.1  # a logit boost of ~3.2 for the hottest expert along 16 v
    layers = [G.DeviceBuiltLayer(**FULL["qwen3_30b_a3b"], seed=500 + l,
                                 rw_add=boost[torch.randperm(E, generator=g, device="cuda")][:, None] * v[None, :])
              for l in range(n_layers)]
    h = (torch.randn((T, H), generator=g, device="cuda") + 16.0 * v).to(torch.bfloat16)
    ws_bytes = layers[0].dev.workspace_bytes(T)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    top_share = []
    stream = torch.cuda.current_stream()
    for dl in layers:
        x_in = G.bf16_to_f32(h)
        Y = torch.empty_like(h)
        dl.dev.forward(h, T, Y, ws, ws_bytes, stream)
        torch.cuda.synchronize()
        rv = dl.dev.route_views(T, ws, ws_bytes)
        ids = ws[rv.ids - ws.data_ptr(): rv.ids - ws.data_ptr() + 4 * T * 8].cpu().numpy().view(np.int32)
        ids = ids.reshape(T, 8).copy()
        _, ref_ids, _ = oracle.moe_route(dl.route_layer(), x_in)
        assert np.array_equal(ids, ref_ids)
        top_share.append(np.bincount(ids.reshape(-1), minlength=E).max() / T)
        Yref, _, _, _ = oracle.moe_layer_forward(dl.host_layer(ids.reshape(-1)), x_in)
        y = G.bf16_to_f32(Y)
        mre, cos = G.quality(y, Yref)
        assert mre <= G.MAX_REL and cos >= G.MIN_COS, (mre, cos)
        dl.dev.forward_residual(h, T, h, h, ws, ws_bytes, stream)  # h += moe(h), in place
        torch.cuda.synchronize()
        err = np.abs(G.bf16_to_f32(h) - (x_in + y)).max()
        assert err <= 2.0 ** -6 * (np.abs(x_in).max() + np.abs(y).max()), err
    assert max(top_share) >= 0.5, top_share  # skewed: some expert takes at least half of the tokens
    for dl in layers:
        dl.close()


# ------------------------------------------- the reference's host-fp32 API

@pytest.fixture
def fresh_cache():
    """The host-pointer API caches weights keyed by the host qweight address
    (src/hal/cuda_backend.cpp:607); numpy reuses freed addresses between tests,
    so each test starts from an empty cache (disable() frees it)."""
    L.lib.llmoc_cuda_disable()
    assert L.lib.llmoc_cuda_enable(0) == 1
    yield
    L.lib.llmoc_cuda_disable()
    assert L.lib.llmoc_cuda_enable(0) == 1


def unit_case(name):
    import make_golden as mg

    g = np.load(f"{mg.HERE}/unit_cases.npz")
    d = {k.split("/")[1]: g[k] for k in g.files if k.startswith(name + "/")}
    sc = int(d["scheme"])
    W = orc.Int4Weight(d["q"], d["s"], d.get("z"), int(d["M"]), int(d["K"]), int(d["gs"]), sc,
                       7 if sc == 2 else 0)
    return d, W


@pytest.mark.parametrize("case", ["awq_scalar", "awq_gemv", "gptq_gemv"])
def test_try_gemm_int4_reference_cases(case, fresh_cache):
    """GpuGemmMatchesCpuIfCuda / AwqGemvJitMatchesCpu / GptqGemvJitMatchesCpu
    (tests/unit/test_int4_gemm.cpp:151-198, test_gpu_quant_gemm.cpp:130-245):
    GPU vs the reference CPU result, rel 1e-3."""
    d, W = unit_case(case)
    y = np.full(W.M, -1e9, np.float32)
    v = L.view_of(W)
    assert L.lib.llmoc_try_gemm_int4(L.ptr(d["x"]), C.byref(v), L.ptr(y)) == 1, L.last_error()
    assert np.all(np.abs(y - d["y"]) < 1e-3 * (1 + np.abs(d["y"])))
    dq = np.empty((W.M, W.K), np.float32)
    assert L.lib.llmoc_try_dequant_int4_matrix(C.byref(v), L.ptr(dq)) == 1
    assert np.array_equal(dq.view(np.uint32), d["dq"].view(np.uint32))


@pytest.mark.parametrize("case", ["awq", "gptq", "awq_tie", "awq_nan", "awq_large", "gptq_neg"])
def test_try_gemm_int4_argmax(oracle, case, fresh_cache):
    """llmoc_try_gemm_int4_argmax against the reference's hal::gemm_int4_argmax
    (golden cases): equal largest rows -> the first; every row non-finite ->
    (0, -1e30); otherwise the same row wherever the oracle's top two rows are
    further apart than the GEMV tolerance, and the value within rel 1e-3 (the
    reference GPU tests' bar)."""
    import make_golden as mg

    g = np.load(f"{mg.HERE}/argmax_cases.npz")
    x, W = mg.argmax_weight(case)
    want_i, want_v = int(g[f"{case}/index"]), np.float32(g[f"{case}/value"])
    idx, val = C.c_int32(-1), C.c_float(0.0)
    v = L.view_of(W)
    assert L.lib.llmoc_try_gemm_int4_argmax(L.ptr(x), C.byref(v), C.byref(idx), C.byref(val)) == 1, L.last_error()
    if case == "awq_nan":
        assert (idx.value, val.value) == (0, np.float32(-1e30))
        return
    y = oracle.gemm_int4(x, W)
    top = np.sort(y)[-2:]
    if case == "awq_tie" or top[1] - top[0] > 1e-3 * (1 + abs(top[1])):
        assert idx.value == want_i
    assert abs(val.value - want_v) < 1e-3 * (1 + abs(want_v))


@pytest.mark.parametrize("case", ["awq_batch", "gptq_batch"])
def test_try_gemm_int4_batch_reference_cases(case, fresh_cache):
    d, W = unit_case(case)
    X = np.ascontiguousarray(d["X"])
    Y = np.empty((X.shape[0], W.M), np.float32)
    v = L.view_of(W)
    assert L.lib.llmoc_try_gemm_int4_batch(L.ptr(X), X.shape[0], C.byref(v), L.ptr(Y)) == 1
    assert np.all(np.abs(Y - d["Y"]) < 1e-3 * (1 + np.abs(d["Y"])))


@pytest.mark.parametrize("M,K,gs,n,scheme", [(4096, 4096, 128, 1, 2), (11008, 4096, 128, 8, 2),
                                             (768, 2048, 128, 64, 1), (2048, 7168, 32, 3, 2)])
def test_try_gemm_int4_config1_shapes(oracle, M, K, gs, n, scheme, fresh_cache):
    rng = np.random.default_rng(M + n)
    Wf = orc.bf16_round(rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02))
    W = oracle.quant_awq_sym(Wf, gs, True) if scheme == 2 else oracle.quant_gptq_asym(Wf, gs)
    X = rng.standard_normal((n, K), dtype=np.float32)
    Y = np.empty((n, M), np.float32)
    v = L.view_of(W)
    assert L.lib.llmoc_try_gemm_int4_batch(L.ptr(X), n, C.byref(v), L.ptr(Y)) == 1, L.last_error()
    ref = oracle.gemm_int4_batch(X, W)
    assert np.all(np.abs(Y - ref) < 1e-3 * (1 + np.abs(ref)))


@pytest.mark.parametrize("n", [2, 3, 4])
def test_try_gemm_int4_multi_distinct_weights(oracle, n, fresh_cache):
    """try_gemm_int4_multi (cuda_backend.cpp:3048-3112: up to 4 GEMVs sharing
    x) with n different weights of different M: each ys[i] against the oracle
    GEMV of its own W_i, and bitwise equal to the single-weight call on it, so
    a swap or mix-up of the weights cannot pass."""
    rng = np.random.default_rng(40 + n)
    K = 2048
    Ms = [768, 1536, 256, 2048][:n]
    Wts = [oracle.quant_awq_sym(orc.bf16_round(rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02)),
                                128, True) for M in Ms]
    x = rng.standard_normal(K, dtype=np.float32)
    vs = [L.view_of(w) for w in Wts]
    ys = [np.full(M, np.nan, np.float32) for M in Ms]
    Ws = (C.POINTER(L.Int4View) * n)(*[C.pointer(v) for v in vs])
    yp = (C.c_void_p * n)(*[L.ptr(a) for a in ys])
    assert L.lib.llmoc_try_gemm_int4_multi(L.ptr(x), Ws, yp, n) == 1, L.last_error()
    for i in range(n):
        ref = oracle.gemm_int4(x, Wts[i])
        assert np.all(np.abs(ys[i] - ref) < 1e-3 * (1 + np.abs(ref))), i
        one = np.empty(Ms[i], np.float32)
        assert L.lib.llmoc_try_gemm_int4(L.ptr(x), C.byref(vs[i]), L.ptr(one)) == 1
        assert np.array_equal(ys[i], one), i


@pytest.mark.parametrize("shared", [False, True])
def test_try_moe_ffn_int4(oracle, shared, fresh_cache):
    """hal::cuda::try_moe_ffn_int4 contract: one token, given experts and weights."""
    rng = np.random.default_rng(11)
    layer = orc.make_layer(oracle, rng, H=1024, I=384, E=12, topk=6, gs=128, shared=shared)
    x = orc.make_tokens(rng, 1, 1024)[0]
    w = np.array([0.3, 0.2, 1e-13, 0.25, 0.15, 0.1], np.float32)
    sel = [5, 1, 7, 0, 11, 3]
    views = []
    exps = (L.MoeExpertInt4 * 6)()
    for i, e in enumerate(sel):
        ex = layer.experts[e]
        trio = [L.view_of(ex.gate), L.view_of(ex.up), L.view_of(ex.down)]
        views.append(trio)
        exps[i] = L.MoeExpertInt4(C.pointer(trio[0]), C.pointer(trio[1]), C.pointer(trio[2]), float(w[i]))
    sh = [L.view_of(layer.shared.gate), L.view_of(layer.shared.up), L.view_of(layer.shared.down)] \
        if shared else [None, None, None]
    shp = [C.pointer(s) if s is not None else None for s in sh]
    y = np.empty(1024, np.float32)
    ok = L.lib.llmoc_try_moe_ffn_int4(L.ptr(x), 1024, 384, exps, 6, shp[0], shp[1], shp[2], 0.5, L.ptr(y))
    assert ok == 1, L.last_error()
    ref = oracle.moe_ffn_routed(x, 1024, 384, [layer.experts[e] for e in sel], w,
                                layer.shared if shared else None, 0.5)
    mre, cos = G.quality(y, ref)
    assert mre <= 1e-3 and cos >= 0.99999, (mre, cos)


def test_resident_cache_budget_and_pinning(oracle, fresh_cache):
    """LRU eviction under the VRAM budget skips pinned weights
    (cuda_backend.cpp:618-639); a shape change at a cached address is refused."""
    rng = np.random.default_rng(12)
    ws = [oracle.quant_awq_sym(orc.bf16_round(rng.standard_normal((256, 1024), dtype=np.float32) * 0.02), 128)
          for _ in range(4)]
    vs = [L.view_of(w) for w in ws]
    assert L.lib.llmoc_pin_int4_weight(C.byref(vs[0])) == 1
    one = L.lib.llmoc_cuda_vram_used()
    L.lib.llmoc_cuda_set_vram_budget(int(one * 2.5))
    for v in vs[1:]:
        assert L.lib.llmoc_prefetch_int4_weight(C.byref(v)) == 1
    assert L.lib.llmoc_cuda_vram_used() <= int(one * 2.5)
    x = rng.standard_normal(1024, dtype=np.float32)
    for w, v in zip(ws, vs):  # evicted weights re-upload transparently
        y = np.empty(256, np.float32)
        assert L.lib.llmoc_try_gemm_int4(L.ptr(x), C.byref(v), L.ptr(y)) == 1
        ref = oracle.gemm_int4(x, w)
        assert np.all(np.abs(y - ref) < 1e-3 * (1 + np.abs(ref)))
    L.lib.llmoc_cuda_set_vram_budget(0)
    bad = L.view(ws[0].q, ws[0].scales, None, 128, 1024, 128)
    y = np.empty(128, np.float32)
    assert L.lib.llmoc_try_gemm_int4(L.ptr(x), C.byref(bad), L.ptr(y)) == 0
    assert "mismatch" in L.last_error()
