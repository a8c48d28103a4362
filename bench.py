#!/usr/bin/env python3
"""Benchmark of the B200 INT4 MoE expert-FFN path (one JSON line on rank 0).

Workload: one Qwen3-30B-A3B-shape MoE layer — hidden
2048, 128 routed experts, top-8, expert intermediate 768, SwiGLU, softmax
router (bf16 weights N(0, 0.02)), expert weights N(0, 0.02) quantized INT4
AWQ-symmetric, group 128, bf16-valued scales; hidden states N(0,1) bf16.
A step is one layer forward over T tokens (default T=64, the largest
decode-size batch); the line also carries a sweep over T in {1, 8, 64, 512}.
All data is synthetic, generated on the device from fixed seeds.

L2 (126 MB): the timed loop rotates over R distinct copies of the layer
(different random weights), sized so the weights the steps touch exceed
3x L2, so weights stream from HBM every step.

Arms:
  (default)          this library through its C ABI (libllmoc_b200.so)
  --impl reference   the reference's own CPU implementation of the path
                     (oracle/_ref: its src/hal AVX2/OpenMP operators, per-token
                     moe_ffn_token loop) on the host cores, bounded samples.
Multi-GPU (torchrun, --gpus N): expert parallelism — GPU r holds the experts
e with e % N == r of every layer copy (router and shared expert replicated),
routes its own T tokens, and the routed token rows go to their experts' GPUs
and back by NCCL all-to-alls (ep.py).  Weak scaling: T tokens per GPU; value
= N * T / step time, the time the max over ranks; the all-to-all time is
reported beside the local compute.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "llm-on-cpu_b200"))

CONFIGS = {
    "qwen3_30b_a3b": dict(H=2048, I=768, E=128, topk=8, gs=128, router=0, scaling=1.0, shared=False),
    "glm45_air": dict(H=4096, I=1408, E=128, topk=8, gs=128, router=1, scaling=1.0, shared=True),
    "kimi_k2": dict(H=7168, I=2048, E=384, topk=8, gs=32, router=1, scaling=2.827, shared=True),
}
# 48 Qwen3-30B-A3B-shape MoE layers (router + FFN, residual
# add between layers), decode T in {1, 4, 16}, expert popularity Zipf(s=1.1)
STACKS = {"qwen3_30b_a3b_stack48": dict(base="qwen3_30b_a3b", layers=48, zipf=1.1, mu=16.0)}
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="llmoc", choices=["llmoc", "reference"])
    ap.add_argument("--config", default="qwen3_30b_a3b", choices=list(CONFIGS) + list(STACKS))
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--sweep", default="1,8,64,512", help="extra T values ('' = none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"],
                    help="multi-GPU: the library's NVLink peer-store transport, or NCCL all-to-alls")
    ap.add_argument("--no-targets", action="store_true",
                    help="skip the north-star target workloads (Kimi-K2 x4, GLM-4.5-Air prefill) of the N=1 line")
    ap.add_argument("--copies", type=int, default=0,
                    help="distinct layer copies to rotate (0 = enough to defeat L2); small values "
                         "make ncu captures cheap")
    return ap.parse_args()


# ----------------------------------------------------------------- helpers

def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(
        os.environ.get("LOCAL_RANK", 0))


def expected_touched(E, k, T):
    return E * (1.0 - (1.0 - k / E) ** T)


def layer_bytes(cfg):
    """(gate+up bytes, down bytes) one expert streams: packed q + fp16 scales."""
    H, I, gs = cfg["H"], cfg["I"], cfg["gs"]
    gu = 2 * (I * H // 2 + I * (H // gs) * 2)
    dn = H * I // 2 + H * (I // gs) * 2
    return gu, dn


class Clocks:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = out.strip().splitlines()[2:]  # the first samples can predate the load
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 TFLOP/s: (burst, sustained, kind)."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 1590.0, 1400.0, "fallback"


def ncu_traffic(config: str, T: int):
    """dram bytes per launch of the dominant kernel from a committed ncu summary."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    d = json.load(open(p)).get(f"{config}:T{T}")
    return d["dram_bytes_per_launch"] if d else None


# ------------------------------------------------------- device workload

def build_layers(torch, L, cfg, R, seed, keep_host=False, device=0, ep=None, rw_add=None):
    """R distinct layers generated and quantized in HBM (llmoc_quantize_awq_sym),
    then repacked by llmoc_moe_layer_create_device (or, with ep = (rank,
    world), this rank's expert-parallel shard of each).  keep_host returns the
    first layer's QLWC tensors on the host for the CPU baseline.  rw_add(r)
    returns an [E, H] fp32 tensor added to copy r's router weights before
    they are rounded to bf16 (the Zipf-skewed stack)."""
    H, I, E, gs = cfg["H"], cfg["I"], cfg["E"], cfg["gs"]
    n_exp = E + (1 if cfg["shared"] else 0)
    g = torch.Generator(device="cuda")
    layers, host = [], None
    stream = torch.cuda.current_stream()
    for r in range(R):
        g.manual_seed(seed + 1000 * r)
        raw = {}
        for name, (M, K) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            q = torch.empty((n_exp * M, K // 2), dtype=torch.uint8, device="cuda")
            s = torch.empty((n_exp * M, K // gs), dtype=torch.int16, device="cuda")
            per = max(1, int(2 ** 28 // (M * K)))  # experts per generation chunk (<= 1 GiB fp32)
            for e0 in range(0, n_exp, per):
                e1 = min(n_exp, e0 + per)
                W = (torch.randn(((e1 - e0) * M, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
                L.quantize_awq_sym(W, (e1 - e0) * M, K, gs, True, q[e0 * M:e1 * M], s[e0 * M:e1 * M], stream)
                del W
            raw[name] = (q, s, M, K)
        rw = torch.randn((E, H), generator=g, device="cuda") * 0.02
        if rw_add is not None:
            rw = rw + rw_add(r)
        rw = rw.to(torch.bfloat16)
        bias = (torch.randn((E,), generator=g, device="cuda") * 0.1).float() if cfg["router"] == 1 else None
        views = []
        for e in range(n_exp):
            for name in ("gate", "up", "down"):
                q, s, M, K = raw[name]
                views.append(L.view(q.data_ptr() + e * M * (K // 2), s.data_ptr() + e * M * (K // gs) * 2,
                                    None, M, K, gs))
        desc = L.LayerDesc(H, I, E, cfg["topk"], gs, L.SCHEME_AWQ_SYM, 7, cfg["router"], cfg["scaling"],
                           1 if cfg["shared"] else 0, 1.0)
        torch.cuda.synchronize()
        if ep is not None:
            layer = L.EpLayerShard.create_ep(desc, rw, bias, views[:3 * E], views[3 * E:] if cfg["shared"] else None,
                                             ep[0], ep[1], device=device, on_device=True)
        else:
            layer = L.MoeLayer.create(desc, rw, bias, views[:3 * E], views[3 * E:] if cfg["shared"] else None,
                                      device=device, on_device=True)
        layers.append(layer)
        if keep_host and r == 0:
            host = {k: (v[0].cpu().numpy(), v[1].cpu().numpy().view(np.uint16), v[2], v[3]) for k, v in raw.items()}
            host["router_w"] = rw.view(torch.int16).cpu().numpy().view(np.uint16)
            host["bias"] = bias.cpu().numpy() if bias is not None else None
        del raw
    torch.cuda.synchronize()
    return layers, host


def host_layer(cfg, host):
    """The kept layer as oracle objects (for the reference CPU path)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import orc

    H, I, E, gs = cfg["H"], cfg["I"], cfg["E"], cfg["gs"]
    n_exp = E + (1 if cfg["shared"] else 0)
    ex = []
    for e in range(n_exp):
        ws = []
        for name in ("gate", "up", "down"):
            q, s, M, K = host[name]
            ws.append(orc.Int4Weight(q[e * M:(e + 1) * M], s[e * M:(e + 1) * M], None, M, K, gs,
                                     orc.SCHEME_AWQ_SYM, 7))
        ex.append(orc.Expert(*ws))
    return orc.MoeLayer(H, I, E, cfg["topk"], host["router_w"], ex[:E], cfg["router"], host["bias"],
                        cfg["scaling"], ex[E] if cfg["shared"] else None, 1.0)


def reference_cpu(cfg, layer_obj, T_total, budget_s=4.0, min_tokens=4):
    """Time the reference's CPU path (oracle/_ref) on a bounded token sample."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import orc

    R = orc.Reference()
    rng = np.random.default_rng(7)
    Xs = orc.make_tokens(rng, max(min_tokens, 64), cfg["H"])
    done, t0 = 0, time.perf_counter()
    R.moe_layer_forward(layer_obj, Xs[:1])  # warm
    t0 = time.perf_counter()
    while True:
        n = min(len(Xs), max(1, min_tokens))
        R.moe_layer_forward(layer_obj, Xs[:n])
        done += n
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "tokens/s", "cores": R.max_threads(), "kind": "reference",
            "sample": f"{done} tokens of the {cfg['H']}-hidden layer through the reference's per-token "
                      f"moe_ffn_token CPU path (src/hal AVX2/OpenMP, {R.max_threads()} OpenMP threads), "
                      f"{dt:.1f} s"}


# ------------------------------------------------------------------- arms

def run_llmoc(args):
    import torch
    import llmoc_b200 as L

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    cfg = CONFIGS[args.config]
    H, E, k = cfg["H"], cfg["E"], cfg["topk"]
    Ts = sorted({args.tokens} | ({int(x) for x in args.sweep.split(",") if x} if args.sweep else set()))
    gu_b, dn_b = layer_bytes(cfg)
    exp_b = gu_b + dn_b
    touched_min = min(expected_touched(E, k, T) for T in Ts) + (1 if cfg["shared"] else 0)
    R = int(max(2, min(24, np.ceil(3 * L2_BYTES / (touched_min * exp_b)))))
    if args.copies > 0:
        R = args.copies
    layers, host = build_layers(torch, L, cfg, R, seed=1234 + rank, keep_host=(rank == 0 and not args.no_cpu_baseline))
    Tmax = max(Ts)
    ws_bytes = layers[0].workspace_bytes(Tmax)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    Xpool = [(torch.randn((Tmax, H), generator=g, device="cuda")).to(torch.bfloat16) for _ in range(R)]
    Y = torch.empty((Tmax, H), dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step(i, T):
        layers[i % R].forward(Xpool[i % R], T, Y, ws, ws_bytes, sp)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(T, K, fn):
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(K):
            fn(i, T)
        b.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(a.elapsed_time(b))

    results = {}
    clocks = Clocks(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                    if os.environ.get("CUDA_VISIBLE_DEVICES") else local)
    for T in Ts:
        for i in range(args.warmup):
            step(i, T)
        torch.cuda.synchronize()
        if T == args.tokens:
            # back-to-back untimed steps so the clock samples (200 ms apart)
            # see the GPU under this load; the timed region follows directly
            clocks.start()
            t_end = time.perf_counter() + 1.5
            i = 0
            while time.perf_counter() < t_end:
                for _ in range(50):
                    step(i, T)
                    i += 1
                torch.cuda.synchronize()
            n0 = L.launch_count()
        ms = timed(T, args.steps, step)
        if T == args.tokens:
            launches = L.launch_count() - n0
            clk = clocks.stop()
        # stage timing pass (separate; events around each stage)
        for lay in layers:
            lay.set_stage_timing(True)
        for i in range(args.steps):
            step(i, T)
        torch.cuda.synchronize()
        stage = {s: 0.0 for s in L.MoeLayer.STAGES}
        calls = 0
        touched = []
        for lay in layers:
            st, n = lay.stage_times()
            for s_, v in st.items():
                stage[s_] += v
            calls += n
            lay.set_stage_timing(False)
        for j in range(R):  # experts touched per layer copy with its own input
            step(j, T)
            v = layers[j % R].route_views(T, ws, ws_bytes)
            torch.cuda.synchronize()
            off = ws[v.offsets - ws.data_ptr(): v.offsets - ws.data_ptr() + 4 * (layers[0].n_exp + 1)]
            cnt = np.diff(off.cpu().numpy().view(np.int32))
            touched.append(int(np.count_nonzero(cnt)))
        results[T] = dict(ms=ms, stage={s_: v / max(calls, 1) for s_, v in stage.items()},
                          touched=float(np.mean(touched)))

    # e2e through the public API with host buffers (pinned), copies inside the timed region
    T = args.tokens
    Xh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    Xh.copy_(Xpool[0][:T].cpu())
    Yh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    Xd = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")

    def e2e_step(i, T):
        Xd.copy_(Xh, non_blocking=True)
        layers[i % R].forward(Xd, T, Y, ws, ws_bytes, sp)
        Yh.copy_(Y[:T], non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i, T)
    ms_e2e = timed(T, args.steps, e2e_step)

    targets = None
    if world == 1 and not args.no_targets and args.config == "qwen3_30b_a3b":
        for lay in layers:
            lay.close()
        layers = []
        del ws, Xpool
        torch.cuda.empty_cache()
        targets = run_targets(torch, L, args.steps, args.warmup)

    out = None
    if rank == 0:
        world_tokens = world * T * args.steps
        r = results[T]
        peak, peak_kind = measured_peak()
        # dominant kernel: grouped gate/up (+SiLU*mul) — its algorithmic bytes per launch
        gu_ms = r["stage"]["gate_up"]
        touched = r["touched"]
        alg_bytes = touched * gu_b + T * H * 2 + T * (k + (1 if cfg["shared"] else 0)) * cfg["I"] * 2
        step_bytes = touched * exp_b + E * H * 2 + 2 * T * H * 2
        kname = "k_int4_mma<GATE_UP> (grouped gate/up + SiLU*mul)"
        if T == 1:  # the whole layer is one launch (k_moe_decode1), timed as the gate/up stage
            alg_bytes, kname = step_bytes, "k_moe_decode1 (the whole layer for one token, one launch)"
        achieved = alg_bytes / (gu_ms * 1e-3) / 1e9 if gu_ms > 0 else None
        sweep = {}
        for t_, rr in results.items():
            per_step = rr["ms"] / args.steps
            b = rr["touched"] * exp_b + E * H * 2 + 2 * t_ * H * 2
            sweep[str(t_)] = {"tokens_per_s": world * t_ * args.steps / (rr["ms"] * 1e-3),
                              "ms_per_step": per_step, "touched_experts": rr["touched"],
                              "layer_GBps": b / (per_step * 1e-3) / 1e9,
                              "layer_hbm_frac": b / (per_step * 1e-3) / 1e9 / peak,
                              "stage_ms": {s_: round(v, 5) for s_, v in rr["stage"].items()}}
        cpu = None
        if host is not None:
            try:
                cpu = reference_cpu(cfg, host_layer(cfg, host), T)
            except Exception as ex:  # the baseline is reported, not required
                cpu = {"value": None, "unit": "tokens/s", "cores": None, "kind": "reference",
                       "sample": f"unavailable: {ex}"}
        metric, config = line_identity(args, world)
        out = {
            "metric": metric,
            "value": world_tokens / (r["ms"] * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": r["ms"] / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int4 weights x bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded device RNG; BASELINE shapes and distributions)",
            "config": config,
            "e2e": {"value": world * T * args.steps / (ms_e2e * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2},
            "roofline": {"bound": "hbm", "kernel": kname,
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak if achieved else None,
                         "peak_kind": peak_kind, "traffic": ncu_traffic(args.config, T),
                         "alg_bytes_per_launch": alg_bytes, "launch_ms": gu_ms},
            "layer_roofline": {"achieved_GBps": step_bytes / (r["ms"] / args.steps * 1e-3) / 1e9,
                               "frac": step_bytes / (r["ms"] / args.steps * 1e-3) / 1e9 / peak,
                               "bytes_per_step": step_bytes},
            "sweep": sweep,
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": int(launches),
        }
        if targets is not None:
            out["targets"] = targets
        print(json.dumps(out), flush=True)
    for lay in layers:
        lay.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return out


# The north-star targets measured beside the headline (one GPU): BASELINE
# config 5 (four Kimi-K2 layers: decode T = 1, 64 against the HBM roofline,
# prefill T = 8192 against the tensor roofline) and config 4's prefill
# (GLM-4.5-Air, T = 4096).  A step runs the target's layers in sequence with
# the residual add fused (llmoc_moe_forward_residual, in place), starting each
# step from the same input rows (a T x H copy inside the step); every layer is
# distinct and larger than L2.
TARGETS = {
    "kimi_k2_x4": dict(cfg="kimi_k2", layers=4, Ts=(1, 64, 8192), config="BASELINE config 5 (1 GPU)"),
    "glm45_air": dict(cfg="glm45_air", layers=2, Ts=(4096,), config="BASELINE config 4 (prefill)"),
}


def run_targets(torch, L, steps, warmup):
    """Per target and T: step time, touched experts, per-stage times (CUDA
    events around each stage, a separate pass), and the two GEMMs' roofline
    fractions from their algorithmic bytes (decode) or FLOPs (prefill)."""
    hbm, _ = measured_peak()
    tf_burst, tf_sust, tf_kind = measured_tensor_peak()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    out = {}
    for name, tg in TARGETS.items():
        cfg = CONFIGS[tg["cfg"]]
        H, I, E, k = cfg["H"], cfg["I"], cfg["E"], cfg["topk"]
        kk = k + (1 if cfg["shared"] else 0)
        gu_b, dn_b = layer_bytes(cfg)
        layers, _ = build_layers(torch, L, cfg, tg["layers"], seed=2468)
        Tmax = max(tg["Ts"])
        ws_bytes = layers[0].workspace_bytes(Tmax)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(13)
        X0 = torch.randn((Tmax, H), generator=g, device="cuda").to(torch.bfloat16)
        X = torch.empty_like(X0)
        res = {}
        for T in tg["Ts"]:
            K = max(2, min(steps, 10 if T < 1024 else 4))

            def step():  # the layers in sequence on the residual stream, from the same input every step
                X[:T].copy_(X0[:T])
                for lay in layers:
                    lay.forward_residual(X, T, X, X, ws, ws_bytes, sp)

            for _ in range(max(3, warmup)):
                step()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(K):
                step()
            b.record(stream)
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / K
            # per-stage times (serialised by the events) and touched experts per layer
            for lay in layers:
                lay.set_stage_timing(True)
            touched = []
            for _ in range(K):
                X[:T].copy_(X0[:T])
                for lay in layers:
                    lay.forward_residual(X, T, X, X, ws, ws_bytes, sp)
                    vw = lay.route_views(T, ws, ws_bytes)
                    off = ws[vw.offsets - ws.data_ptr(): vw.offsets - ws.data_ptr() + 4 * (E + 1)]
                    touched.append(int(np.count_nonzero(np.diff(off.cpu().numpy().view(np.int32)))))
            torch.cuda.synchronize()
            stage = {s_: 0.0 for s_ in L.MoeLayer.STAGES}
            calls = 0
            for lay in layers:
                st_, n_ = lay.stage_times()
                for s_, v in st_.items():
                    stage[s_] += v
                calls += n_
                lay.set_stage_timing(False)
            stage = {s_: v / max(calls, 1) for s_, v in stage.items()}  # per layer forward
            tch = float(np.mean(touched)) + (1 if cfg["shared"] else 0)  # experts streamed per layer
            r = {"ms_per_step": ms, "tokens_per_s": T / (ms * 1e-3), "layers_per_step": len(layers),
                 "touched_experts_per_layer": tch, "stage_ms_per_layer": {s_: round(v, 5) for s_, v in stage.items()}}
            if T <= 128:  # decode: bytes (weights of the touched experts + activations) per GEMM launch
                gu_bytes = tch * gu_b + T * H * 2 + T * kk * I * 2
                dn_bytes = tch * dn_b + T * kk * (I * 2 + H * 4)
                layer_bytes_ = tch * (gu_b + dn_b) + E * H * 2 + 2 * T * H * 2
                if T == 1:  # one launch for the whole layer (k_moe_decode1), timed as the gate/up stage
                    r["fused_kernel"] = {"kernel": "k_moe_decode1", "alg_bytes": layer_bytes_,
                                         "ms": stage["gate_up"],
                                         "GBps": layer_bytes_ / (stage["gate_up"] * 1e-3) / 1e9,
                                         "hbm_frac": layer_bytes_ / (stage["gate_up"] * 1e-3) / 1e9 / hbm}
                else:
                    r["gate_up"] = {"alg_bytes": gu_bytes, "ms": stage["gate_up"],
                                    "GBps": gu_bytes / (stage["gate_up"] * 1e-3) / 1e9,
                                    "hbm_frac": gu_bytes / (stage["gate_up"] * 1e-3) / 1e9 / hbm}
                    r["down"] = {"alg_bytes": dn_bytes, "ms": stage["down"],
                                 "GBps": dn_bytes / (stage["down"] * 1e-3) / 1e9,
                                 "hbm_frac": dn_bytes / (stage["down"] * 1e-3) / 1e9 / hbm}
                r["layer"] = {"alg_bytes": layer_bytes_, "ms": ms / len(layers),
                              "hbm_frac": layer_bytes_ / (ms / len(layers) * 1e-3) / 1e9 / hbm}
                r["peak"] = {"hbm_GBps": hbm}
            else:  # prefill: FLOPs per GEMM launch (routed + shared rows)
                gu_fl = 2.0 * T * kk * 2 * I * H
                dn_fl = 2.0 * T * kk * I * H
                r["gate_up"] = {"flops": gu_fl, "ms": stage["gate_up"],
                                "TFLOPs": gu_fl / (stage["gate_up"] * 1e-3) / 1e12,
                                "tensor_frac_burst": gu_fl / (stage["gate_up"] * 1e-3) / 1e12 / tf_burst,
                                "tensor_frac_sustained": gu_fl / (stage["gate_up"] * 1e-3) / 1e12 / tf_sust}
                r["down"] = {"flops": dn_fl, "ms": stage["down"],
                             "TFLOPs": dn_fl / (stage["down"] * 1e-3) / 1e12,
                             "tensor_frac_burst": dn_fl / (stage["down"] * 1e-3) / 1e12 / tf_burst}
                r["layer"] = {"flops": 3.0 * gu_fl / 2 + 2.0 * T * E * H, "ms": ms / len(layers),
                              "TFLOPs": (3.0 * gu_fl / 2 + 2.0 * T * E * H) / (ms / len(layers) * 1e-3) / 1e12}
                r["peak"] = {"bf16_tflops_burst": tf_burst, "bf16_tflops_sustained": tf_sust, "kind": tf_kind}
            res[f"T{T}"] = r
        out[name] = {"config": tg["config"], "workload": f"{tg['cfg']} x {tg['layers']} distinct layers",
                     "results": res}
        for lay in layers:
            lay.close()
        del ws, X, X0
        torch.cuda.empty_cache()
    return out


def zipf_targets(E, k, s):
    """Per-expert selection frequencies f_r = min(1, c r^-s), sum k (a token
    picks an expert at most once, so the most popular ones saturate at 1)."""
    r = np.arange(1, E + 1, dtype=np.float64)
    lo, hi = 0.0, 1e6
    for _ in range(200):
        c = 0.5 * (lo + hi)
        if np.minimum(1.0, c * r ** -s).sum() > k:
            hi = c
        else:
            lo = c
    return np.minimum(1.0, lo * r ** -s)


def sweep_tokens(args):
    """Token counts a one-layer run measures (headline T = args.tokens)."""
    return sorted({args.tokens} | ({int(x) for x in args.sweep.split(",") if x} if args.sweep else set()))


def stack_tokens(args):
    """Token counts the 48-layer stack measures (headline T = the largest)."""
    return sorted({args.tokens if args.tokens <= 16 else 16} | ({1, 4, 16} if args.sweep else set()))


def copies_for(cfg, Ts, world=1):
    """Distinct layer copies the timed loop rotates so that the experts the
    step touches (per rank: the world's tokens over its shard) are >= 3x L2."""
    E, k = cfg["E"], cfg["topk"]
    gu_b, dn_b = layer_bytes(cfg)
    touched_min = min(expected_touched(E, k, world * T) / world for T in Ts) + (1 if cfg["shared"] else 0)
    return int(max(2, min(24, np.ceil(3 * L2_BYTES / (touched_min * (gu_b + dn_b))))))


def line_identity(args, world):
    """(metric, config) of this run's bench line -- the library arm's and,
    for the same configuration and N, the reference arm's."""
    if args.config in STACKS:
        st = STACKS[args.config]
        cfg = CONFIGS[st["base"]]
        T = max(stack_tokens(args))
        tgt = zipf_targets(cfg["E"], cfg["topk"], st["zipf"])
        tgt = tgt / tgt.sum()
        return ("INT4 MoE 48-layer stack tokens/s (decode, T=%d)" % T,
                {"workload": "qwen3_30b_a3b x 48 layers (BASELINE config 3)", "tokens": T, "layers": st["layers"],
                 "zipf_s": st["zipf"], "l2": "48 distinct layers (15 GB of experts)",
                 "zipf_target_share": {"top1": round(float(tgt[0]), 4), "top8": round(float(tgt[:8].sum()), 4),
                                       "top32": round(float(tgt[:32].sum()), 4)}})
    cfg = CONFIGS[args.config]
    H, E, k, T = cfg["H"], cfg["E"], cfg["topk"], args.tokens
    R = args.copies if args.copies > 0 else copies_for(cfg, sweep_tokens(args), world)
    l2 = f"rotating {R} distinct layer copies (touched weights >= 3x the 126 MB L2)"
    if world > 1:
        return ("INT4 MoE FFN tokens/s (decode, T=%d per GPU)" % T,
                {"workload": f"{args.config} MoE layer, expert-parallel", "tokens_per_gpu": T, "hidden": H,
                 "experts": E, "experts_per_gpu": E // world, "topk": k, "inter": cfg["I"],
                 "group_size": cfg["gs"], "parallelism": f"ep{world}", "l2": l2})
    return ("INT4 MoE FFN tokens/s (decode, T=%d)" % T,
            {"workload": f"{args.config} MoE layer (BASELINE config 2)" if args.config == "qwen3_30b_a3b"
             else f"{args.config} MoE layer", "tokens": T, "hidden": H, "experts": E,
             "topk": k, "inter": cfg["I"], "group_size": cfg["gs"], "parallelism": "single GPU", "l2": l2})


def calibrate_boosts(E, k, sigma, target, seed, iters=80, n=16384):
    """Logit offsets b (mean 0) so that top-k of N(0, sigma^2) noise + b picks
    expert r with frequency target[r]."""
    rng = np.random.default_rng(seed)
    noise = rng.standard_normal((n, E)) * sigma
    b = np.zeros(E)
    f = None
    for _ in range(iters):
        top = np.argpartition(-(noise + b), k, axis=1)[:, :k]
        f = np.bincount(top.ravel(), minlength=E) / n
        b += 0.5 * (np.log(target + 1e-4) - np.log(f + 1e-4))
        b -= b.mean()
    return b, f


def run_stack(args):
    """a step is one decode pass of T tokens through 48 MoE
    layers (router + expert FFN, in-place residual add fused into the combine:
    llmoc_moe_forward_residual), T in {1, 4, 16}.  Expert popularity follows
    Zipf(1.1): every router row gets c_e * v and every hidden state mu * v for
    a fixed unit vector v, with c_e calibrated on the host against truncated
    Zipf targets (each layer its own random expert order); the measured
    selection histogram is reported beside the target's."""
    import torch
    import llmoc_b200 as L

    st = STACKS[args.config]
    cfg = CONFIGS[st["base"]]
    H, E, k, NL = cfg["H"], cfg["E"], cfg["topk"], st["layers"]
    torch.cuda.set_device(0)
    Ts = sorted({args.tokens if args.tokens <= 16 else 16} | ({1, 4, 16} if args.sweep else set()))
    target = zipf_targets(E, k, st["zipf"])
    # selection depends on offset / noise only: calibrate once for unit logit noise
    b_unit, f_model = calibrate_boosts(E, k, 1.0, target, seed=5)
    g = torch.Generator(device="cuda").manual_seed(77)
    v = torch.randn((H,), generator=g, device="cuda")
    v = v / v.norm()
    perms = [np.random.default_rng(100 + l).permutation(E) for l in range(NL)]
    mu = st["mu"]
    X0 = (torch.randn((max(Ts), H), generator=g, device="cuda") + mu * v[None, :]).to(torch.bfloat16)
    # Layers are built in order while a 256-token probe batch runs through them:
    # layer l's offsets are scaled by the logit noise of ITS input (the residual
    # adds grow the hidden states layer by layer) and applied as c_e = b / mu_l,
    # mu_l the probe's mean component along v.
    Tp = 256
    Xp = (torch.randn((Tp, H), generator=g, device="cuda") + mu * v[None, :]).to(torch.bfloat16)
    wsp, wsp_b = None, 0
    layers = []
    for l in range(NL):  # one distinct layer each (15 GB of experts: no reuse through L2 across layers)
        xf = Xp.float()
        along = xf @ v
        noise = xf - along[:, None] * v[None, :]
        sigma_l = 0.02 * float(noise.norm(dim=1).mean())  # logit std for N(0, 0.02^2) router rows
        mu_l = float(along.mean())
        c = torch.tensor(b_unit[np.argsort(perms[l])] * sigma_l / mu_l, dtype=torch.float32, device="cuda")
        lay, _ = build_layers(torch, L, cfg, 1, seed=4321 + 7 * l, rw_add=lambda r, c=c: c[:, None] * v[None, :])
        layers += lay
        if wsp is None:
            wsp_b = lay[0].workspace_bytes(Tp)
            wsp = torch.empty(wsp_b, dtype=torch.uint8, device="cuda")
        lay[0].forward_residual(Xp, Tp, Xp, Xp, wsp, wsp_b, torch.cuda.current_stream().cuda_stream)
    del Xp, wsp
    Tmax = max(Ts)
    ws_bytes = layers[0].workspace_bytes(Tmax)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    X = torch.empty_like(X0)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    gu_b, dn_b = layer_bytes(cfg)
    exp_b = gu_b + dn_b

    def step(T):
        # every step starts from the calibrated input rows (a device copy of T
        # rows), as the e2e loop's host copy does: run back to back, the 48
        # residual adds would otherwise feed each step's output into the next
        # and the timed steps would route drifted hidden states, not the
        # Zipf-calibrated workload
        X[:T].copy_(X0[:T])
        layers_forward(T)

    def layers_forward(T):
        for lay in layers:
            lay.forward_residual(X, T, X, X, ws, ws_bytes, sp)

    results = {}
    clocks = Clocks(0)
    clk, launches = None, 0
    for T in Ts:
        X.copy_(X0)
        for _ in range(max(3, args.warmup)):
            step(T)
        # selection histogram and touched experts of one step, layer by layer
        X.copy_(X0)
        hist = np.zeros(E)
        touched = 0
        for l, lay in enumerate(layers):
            lay.forward_residual(X, T, X, X, ws, ws_bytes, sp)
            vw = lay.route_views(T, ws, ws_bytes)
            off = ws[vw.offsets - ws.data_ptr(): vw.offsets - ws.data_ptr() + 4 * (E + 1)].cpu().numpy().view(np.int32)
            cnt = np.diff(off)
            touched += int(np.count_nonzero(cnt))
            hist += cnt[perms[l]]  # by popularity rank
        torch.cuda.synchronize()
        if T == max(Ts):
            clocks.start()
            t_end = time.perf_counter() + 1.5
            while time.perf_counter() < t_end:
                step(T)
                torch.cuda.synchronize()
            n0 = L.launch_count()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            step(T)
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        if T == max(Ts):
            launches = L.launch_count() - n0
            clk = clocks.stop()
        results[T] = dict(ms=ms, touched=touched, hist=hist)

    T = max(Ts)
    Xh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    Xh.copy_(X0[:T].cpu())
    Yh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)

    def e2e_step():
        X[:T].copy_(Xh, non_blocking=True)  # the step's input rows from the host
        layers_forward(T)
        Yh.copy_(X[:T], non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize()
    ms_e2e = a.elapsed_time(b)

    peak, peak_kind = measured_peak()
    sweep = {}
    for t_, rr in results.items():
        per = rr["ms"] / args.steps
        byts = rr["touched"] * exp_b + NL * (E * H * 2 + 2 * t_ * H * 2)
        h = rr["hist"] / rr["hist"].sum()
        sweep[str(t_)] = {"tokens_per_s": t_ * args.steps / (rr["ms"] * 1e-3), "ms_per_step": per,
                          "touched_experts_per_layer": rr["touched"] / NL, "GBps": byts / (per * 1e-3) / 1e9,
                          "hbm_frac": byts / (per * 1e-3) / 1e9 / peak,
                          "pair_share_by_rank": {"top1": round(float(h[0]), 4), "top8": round(float(h[:8].sum()), 4),
                                                 "top32": round(float(h[:32].sum()), 4)}}
    r = results[T]
    per = r["ms"] / args.steps
    byts = r["touched"] * exp_b + NL * (E * H * 2 + 2 * T * H * 2)
    metric, config = line_identity(args, 1)
    out = {
        "metric": metric,
        "value": T * args.steps / (r["ms"] * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": per, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4 weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded device RNG; BASELINE config 3 shapes, Zipf-skewed router)",
        "config": config,
        "e2e": {"value": T * args.steps / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        "roofline": {"bound": "hbm", "kernel": "whole 48-layer step", "achieved": byts / (per * 1e-3) / 1e9,
                     "peak": peak, "unit": "GB/s", "frac": byts / (per * 1e-3) / 1e9 / peak, "peak_kind": peak_kind,
                     "traffic": None, "alg_bytes_per_launch": byts, "launch_ms": per},
        "sweep": sweep, "cpu_baseline": None, "clocks": clk, "gpu_launches": int(launches),
    }
    print(json.dumps(out), flush=True)
    for lay in layers:
        lay.close()
    return out


def reference_layer(O, cfg, X, rng, weight_budget=2.5e9):
    """A layer for the reference arm with every expert distinct: the router
    (and selection bias) first, then the tokens of X are taken in order while
    the experts they route to stay within `weight_budget` weights, and only
    those experts (and the shared one) are drawn and quantized -- the CPU path
    reads no other.  Returns (layer, token indices of that pool)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import orc

    H, I, E, k, gs = cfg["H"], cfg["I"], cfg["E"], cfg["topk"], cfg["gs"]
    rw = orc.bf16_bits(rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02))
    bias = (rng.standard_normal(E, dtype=np.float32) * np.float32(0.1)) if cfg["router"] == 1 else None
    tiny = orc.Int4Weight(np.zeros((16, 16), np.uint8), np.zeros((16, 1), np.uint16), None, 16, 32, 32)
    stub = orc.Expert(tiny, tiny, tiny)
    probe = orc.MoeLayer(H, I, E, k, rw, [stub] * E, cfg["router"], bias, cfg["scaling"], None, 1.0)
    _, ids, _ = O.moe_route(probe, X)
    max_e = max(k + 1, int(weight_budget // (3 * I * H)))
    need, pool = set(), []
    for t in range(X.shape[0]):
        s = need | set(ids[t].tolist())
        if len(s) > max_e and pool:
            break
        need, pool = s, pool + [t]

    def q(M, K, g):
        W = orc.bf16_round(g.standard_normal((M, K), dtype=np.float32) * np.float32(0.02))
        return O.quant_awq_sym(W, gs, bf16_scale=True)

    made = {}
    for e in sorted(need):
        g = np.random.default_rng(10_000 + e)
        made[e] = orc.Expert(q(I, H, g), q(I, H, g), q(H, I, g))
    filler = made[min(need)]
    experts = [made.get(e, filler) for e in range(E)]
    sh = None
    if cfg["shared"]:
        g = np.random.default_rng(9_999)
        sh = orc.Expert(q(I, H, g), q(I, H, g), q(H, I, g))
    return orc.MoeLayer(H, I, E, k, rw, experts, cfg["router"], bias, cfg["scaling"], sh, 1.0), pool


def run_reference(args):
    """The reference's own CPU implementation of the path on the host cores."""
    rank, world, _ = dist_env()
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import orc

    if not orc.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libllmoc_ref.so was not built"}))
        return None
    # the library arm's metric and config for this configuration and N; a
    # stack step is its layers' per-token CPU path one after another
    metric, config = line_identity(args, world)
    n_layers = STACKS[args.config]["layers"] if args.config in STACKS else 1
    cfg = CONFIGS[STACKS[args.config]["base"]] if args.config in STACKS else CONFIGS[args.config]
    rng = np.random.default_rng(1234)
    O = orc.Oracle()
    R = orc.Reference()
    T = config.get("tokens", config.get("tokens_per_gpu"))
    X = orc.make_tokens(rng, T, cfg["H"])
    layer, pool = reference_layer(O, cfg, X, rng)
    Xp = X[pool]
    per_step = max(1, min(len(pool), 8))  # bounded sample of each step's tokens
    for i in range(args.warmup):
        R.moe_layer_forward(layer, Xp[:per_step])
    t0 = time.perf_counter()
    for i in range(args.steps):
        R.moe_layer_forward(layer, Xp[(i * per_step) % len(pool):][:per_step])
    dt = time.perf_counter() - t0
    v = per_step * args.steps / dt / n_layers
    line = {"impl": "reference", "metric": metric, "value": v,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3 * n_layers, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 weights x fp32 activations (AVX2 fp32)",
            "data": "synthetic", "config": config,
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": R.max_threads(), "kind": "reference",
                             "sample": f"{per_step} tokens per step, cycling over {len(pool)} of the {T} "
                                       f"tokens (every expert they route to distinct) through the reference's "
                                       f"per-token moe_ffn_token CPU path"
                                       + (f", one layer, rate / {n_layers} layers" if n_layers > 1 else "")},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return line


def run_ep(args):
    """--gpus N > 1: the expert-parallel layer step across N ranks (NCCL)."""
    import datetime

    import torch
    import torch.distributed as dist

    import ep as EP
    import llmoc_b200 as L

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = CONFIGS[args.config]
    H, E, k, I = cfg["H"], cfg["E"], cfg["topk"], cfg["I"]
    Ts = sorted({args.tokens} | ({int(x) for x in args.sweep.split(",") if x} if args.sweep else set()))
    gu_b, dn_b = layer_bytes(cfg)
    exp_b = gu_b + dn_b

    def touched_local(T):  # expected routed experts of this shard that the world's tokens touch
        return expected_touched(E, k, world * T) / world

    touched_min = min(touched_local(T) for T in Ts) + (1 if cfg["shared"] else 0)
    R = int(max(2, min(24, np.ceil(3 * L2_BYTES / (touched_min * exp_b)))))
    if args.copies > 0:
        R = args.copies
    shards, _ = build_layers(torch, L, cfg, R, seed=1234, device=local, ep=(rank, world))
    backends = [EP.DeviceBackend(s, H, k) for s in shards]
    Tmax = max(Ts)
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    Xpool = [(torch.randn((Tmax, H), generator=g, device="cuda")).to(torch.bfloat16) for _ in range(R)]
    stream = torch.cuda.current_stream()
    p2p = args.ep_transport == "p2p"
    if p2p:  # one transport for every layer copy (same shape); one step sequence
        tr = L.EpTransport(world, rank, H, Tmax, k, local)
        EP.connect_p2p(tr)
        pstep = EP.P2PStep(shards[0], tr, H)

    def fwd(i, X, T, times=None):
        if p2p:
            pstep.shard = shards[i % R]
            return pstep.forward(X, T, times=times)
        return EP.ep_forward(backends[i % R], X, T, times=times)

    def step(i, T):
        fwd(i, Xpool[i % R][:T], T)

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(T, K, fn):
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(K):
            fn(i, T)
        b.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        return max_over_ranks(a.elapsed_time(b))

    results = {}
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = Clocks(int(vis.split(",")[local]) if vis else local)
    clk, launches = None, 0
    for T in Ts:
        for i in range(max(3, args.warmup)):
            step(i, T)
        torch.cuda.synchronize()
        if T == args.tokens:
            # ~1.5 s of back-to-back steps for the clock samples.  Every rank
            # runs the same number of steps (a count agreed from one timed
            # batch, max over ranks): a rank that ran ahead would wait on
            # sequence flags its peers never raise until its budget ran out.
            clocks.start()
            t0 = time.perf_counter()
            for i in range(10):
                step(i, T)
            torch.cuda.synchronize()
            batches = int(np.ceil(1.5 / max(max_over_ranks(time.perf_counter() - t0), 1e-4)))
            for i in range(10, 10 * batches):
                step(i, T)
            torch.cuda.synchronize()
            n0 = L.launch_count()
        ms = timed(T, args.steps, step)
        if T == args.tokens:
            launches = L.launch_count() - n0
            clk = clocks.stop()
        # phase times (a separate pass: events around each phase)
        acc = {"dispatch_ms": 0.0, "a2a_ms": 0.0, "experts_ms": 0.0, "combine_ms": 0.0}
        rows = [0, 0]
        for i in range(args.steps):
            tm = EP.EpTimes()
            fwd(i, Xpool[i % R][:T], T, times=tm)
            for key in acc:
                acc[key] += getattr(tm, key) / args.steps
            rows[0] += tm.sent_rows if not p2p else T * k
            rows[1] += tm.recv_rows if not p2p else T * k  # expected: the rows stay on the device
        phases = {key: max_over_ranks(v) for key, v in acc.items()}
        recv_max = max_over_ranks(rows[1] / args.steps)
        results[T] = dict(ms=ms, phases=phases, recv_rows_max=recv_max)

    # e2e: host tokens in, host outputs out, every step on every rank
    T = args.tokens
    Xh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    Xh.copy_(Xpool[0][:T].cpu())
    Yh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    Xd = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")

    def e2e_step(i, T):
        Xd.copy_(Xh, non_blocking=True)
        Y = fwd(i, Xd, T)
        Yh.copy_(Y, non_blocking=True)

    for i in range(max(3, args.warmup)):
        e2e_step(i, T)
    ms_e2e = timed(T, args.steps, e2e_step)

    out = None
    if rank == 0:
        r = results[T]
        peak, peak_kind = measured_peak()
        ph = r["phases"]
        per_step = r["ms"] / args.steps
        tl = touched_local(T) + (1 if cfg["shared"] else 0)
        # the local expert phase streams the shard's touched experts and reads/writes the received rows
        alg = tl * exp_b + r["recv_rows_max"] * H * 2 * 2
        achieved = alg / (ph["experts_ms"] * 1e-3) / 1e9 if ph["experts_ms"] > 0 else None
        sweep = {}
        for t_, rr in results.items():
            ps = rr["ms"] / args.steps
            sweep[str(t_)] = {"tokens_per_s": world * t_ * args.steps / (rr["ms"] * 1e-3), "ms_per_step": ps,
                              "phases_ms": {a: round(b, 5) for a, b in rr["phases"].items()}}
        a2a_bytes = T * k * H * 2 * 2 + T * k * 4  # rows out and back (bf16) + expert ids, per GPU
        metric, config = line_identity(args, world)
        out = {
            "metric": metric,
            "value": world * T * args.steps / (r["ms"] * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": per_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int4 weights x bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded device RNG; BASELINE shapes and distributions)",
            "config": config,
            "ep": {"phases_ms": ph, "a2a_bytes_per_gpu_per_step": a2a_bytes,
                   "a2a_GBps_per_gpu": a2a_bytes / (ph["a2a_ms"] * 1e-3) / 1e9 if ph["a2a_ms"] > 0 else None,
                   "transport": ("library NVLink transport: rows stored into the owners' receive buffers "
                                 "(CUDA IPC peer pointers) with per-step flags, no host sync; the transfer "
                                 "time is inside the send / serve / finish phases (dispatch_ms, experts_ms, "
                                 "combine_ms), including each phase's wait for its peers")
                   if p2p else "NCCL all_to_all_single over NVLink (torch.distributed)"},
            "e2e": {"value": world * T * args.steps / (ms_e2e * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2},
            "roofline": {"bound": "hbm", "kernel": "local expert phase (grouped gate/up + down on the shard)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak if achieved else None, "peak_kind": peak_kind, "traffic": None,
                         "alg_bytes_per_launch": alg, "launch_ms": ph["experts_ms"]},
            "sweep": sweep,
            "cpu_baseline": None,
            "clocks": clk,
            "gpu_launches": int(launches),
        }
        print(json.dumps(out), flush=True)
    dist.barrier()
    if p2p:
        tr.close()
    for s in shards:
        s.close()
    dist.destroy_process_group()
    return out


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.config in STACKS:
        run_stack(args)
    elif dist_env()[1] > 1:
        run_ep(args)
    else:
        run_llmoc(args)


if __name__ == "__main__":
    main()
