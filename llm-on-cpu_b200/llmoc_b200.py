"""ctypes binding of libllmoc_b200.so (C ABI: include/llmoc_b200.h).

Loads the in-tree sm_100a library and exposes its entry points to Python
callers (tests, bench.py, a ctypes-based host).  Device buffers are passed
as integer addresses or as objects with ``data_ptr()`` (torch tensors).
Importing this module never falls back to anything: a missing library
raises at import time.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from typing import Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libllmoc_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "llmoc_b200.h")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is not built; run `make -C {HERE}` (or __graft_entry__.build())")
lib = C.CDLL(LIB_PATH)

OK = 0
STATUS = {0: "OK", 1: "INVALID", 2: "NO_DEVICE", 3: "CUDA", 4: "NO_MEMORY", 5: "NOT_ENABLED",
          6: "UNSUPPORTED", 7: "WORKSPACE", 8: "TIMEOUT"}
SCHEME_GPTQ_ASYM = 1
SCHEME_AWQ_SYM = 2
ROUTER_SOFTMAX = 0
ROUTER_SIGMOID_BIAS = 1


class Int4View(C.Structure):
    _fields_ = [("qweight", C.c_void_p), ("scales", C.c_void_p), ("zeros", C.c_void_p),
                ("scales_f32", C.c_void_p), ("M", C.c_int32), ("K", C.c_int32),
                ("group_size", C.c_int32), ("scheme", C.c_uint32), ("awq_zp", C.c_int32)]


class MoeExpertInt4(C.Structure):
    _fields_ = [("gate", C.POINTER(Int4View)), ("up", C.POINTER(Int4View)),
                ("down", C.POINTER(Int4View)), ("weight", C.c_float)]


class LayerDesc(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("n_experts", C.c_int32),
                ("topk", C.c_int32), ("group_size", C.c_int32), ("scheme", C.c_int32),
                ("awq_zp", C.c_int32), ("router", C.c_int32), ("routed_scaling", C.c_float),
                ("has_shared", C.c_int32), ("shared_scale", C.c_float)]


class QlwcLayerInfo(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("n_experts", C.c_int32),
                ("group_size", C.c_int32), ("scheme", C.c_int32), ("has_router", C.c_int32),
                ("has_shared", C.c_int32), ("has_shared_gate", C.c_int32), ("has_bias", C.c_int32)]


class RouteViews(C.Structure):
    _fields_ = [("logits", C.c_void_p), ("ids", C.c_void_p), ("weights", C.c_void_p),
                ("offsets", C.c_void_p), ("sorted", C.c_void_p), ("inverse", C.c_void_p),
                ("n_active", C.c_void_p), ("error_flag", C.c_void_p)]


_vp, _i, _sz, _f = C.c_void_p, C.c_int, C.c_size_t, C.c_float
_SIGS = {
    "llmoc_cuda_probe_available": (_i, []),
    "llmoc_cuda_enabled": (_i, []),
    "llmoc_cuda_status": (C.c_char_p, []),
    "llmoc_cuda_device_count": (_i, []),
    "llmoc_cuda_enable": (_i, [_sz]),
    "llmoc_cuda_disable": (None, []),
    "llmoc_cuda_vram_used": (_sz, []),
    "llmoc_cuda_vram_budget": (_sz, []),
    "llmoc_cuda_set_vram_budget": (None, [_sz]),
    "llmoc_cuda_device_mem_info": (_i, [C.POINTER(_sz), C.POINTER(_sz)]),
    "llmoc_cuda_host_register": (_i, [_vp, _sz]),
    "llmoc_cuda_host_unregister": (_i, [_vp]),
    "llmoc_last_error": (C.c_char_p, []),
    "llmoc_try_gemm_int4": (_i, [_vp, C.POINTER(Int4View), _vp]),
    "llmoc_try_gemm_int4_argmax": (_i, [_vp, C.POINTER(Int4View), C.POINTER(C.c_int32), C.POINTER(C.c_float)]),
    "llmoc_collective_create": (_i, [_i, _i, C.c_size_t, _i, C.POINTER(_vp), _vp]),
    "llmoc_collective_connect": (_i, [_vp, _vp]),
    "llmoc_collective_connect_local": (_i, [_vp, C.POINTER(_vp)]),
    "llmoc_collective_destroy": (None, [_vp]),
    "llmoc_collective_world_size": (_i, [_vp]),
    "llmoc_collective_error": (_i, [_vp]),
    "llmoc_collective_set_wait_cycles": (_i, [_vp, C.c_longlong]),
    "llmoc_collective_start": (_i, [_vp, _i, _vp, C.c_size_t, _i, _vp]),
    "llmoc_collective_finish": (_i, [_vp, _i, _vp, C.c_size_t, _i, _i, _vp]),
    "llmoc_collective_alltoall": (_i, [_vp, _vp, _vp, C.c_size_t, _vp]),
    "llmoc_collective_allreduce_sum": (_i, [_vp, _vp, C.c_size_t, _i, _vp]),
    "llmoc_collective_broadcast": (_i, [_vp, _vp, C.c_size_t, _i, _vp]),
    "llmoc_try_gemm_int4_batch": (_i, [_vp, _i, C.POINTER(Int4View), _vp]),
    "llmoc_try_gemm_int4_multi": (_i, [_vp, C.POINTER(C.POINTER(Int4View)), C.POINTER(_vp), _i]),
    "llmoc_try_gemm_int4_batch_multi": (_i, [_vp, _i, C.POINTER(C.POINTER(Int4View)),
                                             C.POINTER(_vp), _i]),
    "llmoc_prefetch_int4_weight": (_i, [C.POINTER(Int4View)]),
    "llmoc_pin_int4_weight": (_i, [C.POINTER(Int4View)]),
    "llmoc_try_dequant_int4_matrix": (_i, [C.POINTER(Int4View), _vp]),
    "llmoc_try_moe_ffn_int4": (_i, [_vp, _i, _i, C.POINTER(MoeExpertInt4), _i, C.POINTER(Int4View),
                                    C.POINTER(Int4View), C.POINTER(Int4View), _f, _vp]),
    "llmoc_moe_layer_create": (_i, [C.POINTER(LayerDesc), _vp, _vp, C.POINTER(Int4View),
                                    C.POINTER(Int4View), _i, C.POINTER(_vp)]),
    "llmoc_moe_layer_create_device": (_i, [C.POINTER(LayerDesc), _vp, _vp, C.POINTER(Int4View),
                                           C.POINTER(Int4View), _i, C.POINTER(_vp)]),
    "llmoc_moe_layer_destroy": (None, [_vp]),
    "llmoc_moe_layer_weight_bytes": (_sz, [_vp]),
    "llmoc_expert_storage_bytes": (_sz, [_i, _i, _i, _i]),
    "llmoc_moe_workspace_bytes": (_sz, [_vp, _i]),
    "llmoc_moe_forward": (_i, [_vp, _vp, _i, _vp, _vp, _sz, _vp]),
    "llmoc_moe_layer_set_shared_gate": (_i, [_vp, _vp, _i]),
    "llmoc_qlwc_describe": (_i, [C.c_char_p, C.c_char_p, _i, C.POINTER(QlwcLayerInfo)]),
    "llmoc_qlwc_moe_layers": (_i, [C.c_char_p, C.c_char_p, C.POINTER(C.c_int32), _i]),
    "llmoc_moe_layer_create_qlwc": (_i, [C.c_char_p, C.c_char_p, _i, C.POINTER(LayerDesc), _i, C.POINTER(_vp)]),
    "llmoc_moe_forward_residual": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _sz, _vp]),
    "llmoc_moe_route_views": (_i, [_vp, _i, _vp, _sz, C.POINTER(RouteViews)]),
    "llmoc_moe_route": (_i, [_vp, _vp, _i, _vp, _sz, _vp]),
    "llmoc_moe_dequant": (_i, [_vp, _i, _i, _vp, _vp]),
    "llmoc_quantize_awq_sym": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    "llmoc_kernel_launch_count": (C.c_uint64, []),
    "llmoc_moe_layer_set_wait_cycles": (_i, [_vp, C.c_longlong]),
    "llmoc_moe_set_stage_timing": (_i, [_vp, _i]),
    "llmoc_moe_forward_noalloc": (_i, [_vp, _vp, _i, _vp, _vp]),
    "llmoc_moe_noalloc_capacity": (_sz, []),
    "llmoc_moe_noalloc_status": (_i, [_vp, _i, _vp]),
    "llmoc_moe_stage_times": (_i, [_vp, C.POINTER(C.c_float), C.POINTER(_i)]),
    "llmoc_moe_layer_create_ep": (_i, [C.POINTER(LayerDesc), _vp, _vp, C.POINTER(Int4View),
                                       C.POINTER(Int4View), _i, _i, _i, _i, C.POINTER(_vp)]),
    "llmoc_moe_ep_source_workspace_bytes": (_sz, [_vp, _i]),
    "llmoc_moe_ep_owner_workspace_bytes": (_sz, [_vp, _i]),
    "llmoc_moe_ep_dispatch": (_i, [_vp, _vp, _i, _vp, _sz, _vp, _vp, _vp, _vp]),
    "llmoc_moe_ep_experts": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _sz, _vp]),
    "llmoc_moe_ep_experts_padded": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _sz, _vp]),
    "llmoc_moe_ep_combine": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _sz, _vp]),
    "llmoc_ep_ipc_handle_bytes": (_sz, []),
    "llmoc_ep_transport_create": (_i, [_i, _i, _i, _i, _i, _i, C.POINTER(_vp), _vp]),
    "llmoc_ep_transport_connect": (_i, [_vp, _vp]),
    "llmoc_ep_transport_connect_local": (_i, [_vp, C.POINTER(_vp)]),
    "llmoc_ep_transport_destroy": (None, [_vp]),
    "llmoc_ep_transport_error": (_i, [_vp]),
    "llmoc_ep_transport_set_wait_cycles": (_i, [_vp, C.c_longlong]),
    "llmoc_ep_p2p_workspace_bytes": (_sz, [_vp, _vp, _i]),
    "llmoc_ep_p2p_send": (_i, [_vp, _vp, _vp, _i, C.c_uint32, _vp, _sz, _vp]),
    "llmoc_ep_p2p_serve": (_i, [_vp, _vp, _i, C.c_uint32, _vp, _sz, _vp]),
    "llmoc_ep_p2p_finish": (_i, [_vp, _vp, _vp, _i, _vp, C.c_uint32, _vp, _sz, _vp]),
}
for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def header_symbols(path: str = HEADER) -> list:
    """Every function the C header declares."""
    txt = open(path).read()
    return sorted(set(re.findall(r"LLMOC_API\s+[\w\s\*]+?\b(llmoc_\w+)\s*\(", txt)))


def ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if hasattr(x, "ctypes"):
        return int(x.ctypes.data)
    raise TypeError(f"cannot take the address of {type(x)}")


def last_error() -> str:
    return (lib.llmoc_last_error() or b"").decode()


class LlmocError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status != OK:
        raise LlmocError(f"{what}: {STATUS.get(status, status)}: {last_error()}")


def stream_ptr(stream) -> Optional[int]:
    """cudaStream_t of a torch stream (or an int / None)."""
    if stream is None or isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def view(q, scales, zeros, M: int, K: int, group_size: int, scheme: int = SCHEME_AWQ_SYM,
         awq_zp: int = 7) -> Int4View:
    """An Int4View over host (numpy) or device (torch / int) buffers."""
    return Int4View(ptr(q), ptr(scales), ptr(zeros) if zeros is not None else None, None, M, K,
                    group_size, scheme, awq_zp)


def view_of(w) -> Int4View:
    """Int4View of an oracle.orc.Int4Weight-like object (host numpy arrays)."""
    return view(w.q, w.scales, w.zeros, w.M, w.K, w.group_size, w.scheme, w.awq_zp)


class MoeLayer:
    """A device-resident MoE layer (llmoc_moe_layer_*)."""

    def __init__(self, handle: int, desc: LayerDesc):
        self.handle = handle
        self.desc = desc

    @classmethod
    def create(cls, desc: LayerDesc, router_w, bias, experts: Sequence[Int4View],
               shared: Optional[Sequence[Int4View]], device: int = 0, on_device: bool = False):
        n = len(experts)
        arr = (Int4View * n)(*experts)
        sh = (Int4View * 3)(*shared) if shared is not None else None
        h = C.c_void_p()
        fn = lib.llmoc_moe_layer_create_device if on_device else lib.llmoc_moe_layer_create
        check(fn(C.byref(desc), ptr(router_w), ptr(bias), arr, sh, device, C.byref(h)),
              "llmoc_moe_layer_create")
        return cls(h.value, desc)

    @classmethod
    def from_host(cls, layer, device: int = 0) -> "MoeLayer":
        """From an oracle.orc.MoeLayer (host numpy weights)."""
        e0 = layer.experts[0].gate
        desc = LayerDesc(layer.H, layer.I, layer.E, layer.topk, e0.group_size, e0.scheme,
                         e0.awq_zp if e0.awq_zp > 0 else 7, layer.router, layer.routed_scaling,
                         1 if layer.shared is not None else 0, layer.shared_scale)
        views = []
        for ex in layer.experts:
            views += [view_of(ex.gate), view_of(ex.up), view_of(ex.down)]
        sh = None
        if layer.shared is not None:
            sh = [view_of(layer.shared.gate), view_of(layer.shared.up), view_of(layer.shared.down)]
        dev = cls.create(desc, layer.router_w, layer.bias, views, sh, device)
        if getattr(layer, "shared_gate_w", None) is not None:
            dev.set_shared_gate(layer.shared_gate_w)
        return dev

    @classmethod
    def from_qlwc(cls, path: str, prefix: str, layer: int, desc: "LayerDesc", device: int = 0) -> "MoeLayer":
        """Layer `layer` of a QLWC file (llmoc_moe_layer_create_qlwc)."""
        h = C.c_void_p()
        check(lib.llmoc_moe_layer_create_qlwc(path.encode(), prefix.encode(), layer, C.byref(desc), device,
                                              C.byref(h)), "llmoc_moe_layer_create_qlwc")
        return cls(h.value, desc)

    def set_shared_gate(self, gate_row, on_device: bool = False) -> None:
        """Per-token shared-expert weight sigmoid(gate_row . x) (bf16 [hidden])."""
        check(lib.llmoc_moe_layer_set_shared_gate(self.handle, ptr(gate_row), 1 if on_device else 0),
              "llmoc_moe_layer_set_shared_gate")

    def close(self) -> None:
        if self.handle:
            lib.llmoc_moe_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def kk(self) -> int:
        return self.desc.topk + self.desc.has_shared

    @property
    def n_exp(self) -> int:
        return self.desc.n_experts + self.desc.has_shared

    def weight_bytes(self) -> int:
        return int(lib.llmoc_moe_layer_weight_bytes(self.handle))

    def workspace_bytes(self, T: int) -> int:
        return int(lib.llmoc_moe_workspace_bytes(self.handle, T))

    def forward(self, X, T: int, Y, ws, ws_bytes: int, stream=None) -> None:
        check(lib.llmoc_moe_forward(self.handle, ptr(X), T, ptr(Y), ptr(ws), ws_bytes,
                                    stream_ptr(stream)), "llmoc_moe_forward")

    def forward_residual(self, X, T: int, R, Y, ws, ws_bytes: int, stream=None) -> None:
        """Y = R + MoE(X) (R may be Y, and both may be X)."""
        check(lib.llmoc_moe_forward_residual(self.handle, ptr(X), T, ptr(R), ptr(Y), ptr(ws), ws_bytes,
                                             stream_ptr(stream)), "llmoc_moe_forward_residual")

    def route(self, X, T: int, ws, ws_bytes: int, stream=None) -> None:
        check(lib.llmoc_moe_route(self.handle, ptr(X), T, ptr(ws), ws_bytes, stream_ptr(stream)),
              "llmoc_moe_route")

    def route_views(self, T: int, ws, ws_bytes: int) -> RouteViews:
        v = RouteViews()
        check(lib.llmoc_moe_route_views(self.handle, T, ptr(ws), ws_bytes, C.byref(v)),
              "llmoc_moe_route_views")
        return v

    STAGES = ("router", "topk", "permute", "gate_up", "down", "combine")

    def set_wait_cycles(self, cycles: int) -> None:
        """Budget (SM clocks) of each barrier wait of the fused one-token forward."""
        check(lib.llmoc_moe_layer_set_wait_cycles(self.handle, int(cycles)), "llmoc_moe_layer_set_wait_cycles")

    def set_stage_timing(self, enable: bool) -> None:
        check(lib.llmoc_moe_set_stage_timing(self.handle, int(enable)), "llmoc_moe_set_stage_timing")

    def stage_times(self):
        """(dict stage -> summed ms, number of timed calls); clears the record."""
        ms = (C.c_float * 6)()
        n = C.c_int()
        check(lib.llmoc_moe_stage_times(self.handle, ms, C.byref(n)), "llmoc_moe_stage_times")
        return dict(zip(self.STAGES, [float(v) for v in ms])), n.value

    def dequant(self, expert: int, proj: int, out, stream=None) -> None:
        check(lib.llmoc_moe_dequant(self.handle, expert, proj, ptr(out), stream_ptr(stream)),
              "llmoc_moe_dequant")


def quantize_awq_sym(W, M: int, K: int, gs: int, bf16_scale: bool, q, scales, stream=None) -> None:
    check(lib.llmoc_quantize_awq_sym(ptr(W), M, K, gs, int(bf16_scale), ptr(q), ptr(scales),
                                     stream_ptr(stream)), "llmoc_quantize_awq_sym")


def launch_count() -> int:
    return int(lib.llmoc_kernel_launch_count())


class EpLayerShard(MoeLayer):
    """One rank's shard of an expert-parallel layer (llmoc_moe_layer_create_ep):
    routed experts e with e % world == rank, plus the router and shared expert."""

    def __init__(self, handle: int, desc: LayerDesc, rank: int, world: int):
        super().__init__(handle, desc)
        self.rank, self.world = rank, world

    @classmethod
    def create_ep(cls, desc: LayerDesc, router_w, bias, experts: Sequence[Int4View],
                  shared: Optional[Sequence[Int4View]], rank: int, world: int, device: int = 0,
                  on_device: bool = False):
        n = len(experts)
        arr = (Int4View * n)(*experts)
        sh = (Int4View * 3)(*shared) if shared is not None else None
        h = C.c_void_p()
        check(lib.llmoc_moe_layer_create_ep(C.byref(desc), ptr(router_w), ptr(bias), arr, sh, device, rank, world,
                                            1 if on_device else 0, C.byref(h)), "llmoc_moe_layer_create_ep")
        return cls(h.value, desc, rank, world)

    @classmethod
    def from_host_ep(cls, layer, rank: int, world: int, device: int = 0) -> "EpLayerShard":
        e0 = layer.experts[0].gate
        desc = LayerDesc(layer.H, layer.I, layer.E, layer.topk, e0.group_size, e0.scheme,
                         e0.awq_zp if e0.awq_zp > 0 else 7, layer.router, layer.routed_scaling,
                         1 if layer.shared is not None else 0, layer.shared_scale)
        views = []
        for ex in layer.experts:
            views += [view_of(ex.gate), view_of(ex.up), view_of(ex.down)]
        sh = None
        if layer.shared is not None:
            sh = [view_of(layer.shared.gate), view_of(layer.shared.up), view_of(layer.shared.down)]
        dev = cls.create_ep(desc, layer.router_w, layer.bias, views, sh, rank, world, device)
        if getattr(layer, "shared_gate_w", None) is not None:
            dev.set_shared_gate(layer.shared_gate_w)
        return dev

    @property
    def e_loc(self) -> int:
        return self.desc.n_experts // self.world

    def source_workspace_bytes(self, T: int) -> int:
        return int(lib.llmoc_moe_ep_source_workspace_bytes(self.handle, T))

    def owner_workspace_bytes(self, rows: int) -> int:
        return int(lib.llmoc_moe_ep_owner_workspace_bytes(self.handle, rows))

    def dispatch(self, X, T, ws, ws_bytes, send_rows, send_expert, send_counts, stream=None) -> None:
        check(lib.llmoc_moe_ep_dispatch(self.handle, ptr(X), T, ptr(ws), ws_bytes, ptr(send_rows), ptr(send_expert),
                                        ptr(send_counts), stream_ptr(stream)), "llmoc_moe_ep_dispatch")

    def experts(self, rows, expert, n, out_rows, ws, ws_bytes, stream=None, n_hint=None) -> None:
        """n rows of owner-local expert ids; with n_hint, the fixed-capacity
        layout (ids outside the shard's experts are empty slots, n_hint the
        occupied slots expected: llmoc_moe_ep_experts_padded)."""
        if n_hint is None:
            check(lib.llmoc_moe_ep_experts(self.handle, ptr(rows), ptr(expert), n, ptr(out_rows), ptr(ws),
                                           ws_bytes, stream_ptr(stream)), "llmoc_moe_ep_experts")
        else:
            check(lib.llmoc_moe_ep_experts_padded(self.handle, ptr(rows), ptr(expert), n, n_hint, ptr(out_rows),
                                                  ptr(ws), ws_bytes, stream_ptr(stream)),
                  "llmoc_moe_ep_experts_padded")

    def combine(self, X, T, ret_rows, Y, ws, ws_bytes, stream=None) -> None:
        check(lib.llmoc_moe_ep_combine(self.handle, ptr(X), T, ptr(ret_rows), ptr(Y), ptr(ws), ws_bytes,
                                       stream_ptr(stream)), "llmoc_moe_ep_combine")


class EpTransport:
    """This rank's end of the NVLink expert-parallel transport
    (llmoc_ep_transport_*): buffers for `world` ranks of a layer with `hidden`
    and `topk`, up to max_tokens tokens per rank and step."""

    def __init__(self, world: int, rank: int, hidden: int, max_tokens: int, topk: int, device: int = 0,
                 export: bool = True):
        self.world, self.rank, self.max_tokens = world, rank, max_tokens
        h = C.c_void_p()
        self.ipc = (C.c_char * int(lib.llmoc_ep_ipc_handle_bytes()))() if export else None
        check(lib.llmoc_ep_transport_create(world, rank, hidden, max_tokens, topk, device, C.byref(h),
                                            C.cast(self.ipc, C.c_void_p) if export else None),
              "llmoc_ep_transport_create")
        self.handle = h.value
        self.seq = 0

    def connect(self, handles: bytes) -> None:
        """handles: every rank's IPC handle, in rank order."""
        buf = C.create_string_buffer(handles, len(handles))
        check(lib.llmoc_ep_transport_connect(self.handle, C.cast(buf, C.c_void_p)), "llmoc_ep_transport_connect")

    @staticmethod
    def connect_local(transports) -> None:
        """Every rank of the world in this process (tests)."""
        arr = (C.c_void_p * len(transports))(*[t.handle for t in transports])
        for t in transports:
            check(lib.llmoc_ep_transport_connect_local(t.handle, arr), "llmoc_ep_transport_connect_local")

    def error(self) -> int:
        return int(lib.llmoc_ep_transport_error(self.handle))

    def workspace_bytes(self, shard, T: int) -> int:
        return int(lib.llmoc_ep_p2p_workspace_bytes(shard.handle, self.handle, T))

    def send(self, shard, X, T: int, seq: int, ws, ws_bytes: int, stream=None) -> None:
        check(lib.llmoc_ep_p2p_send(shard.handle, self.handle, ptr(X), T, seq, ptr(ws), ws_bytes,
                                    stream_ptr(stream)), "llmoc_ep_p2p_send")

    def serve(self, shard, T: int, seq: int, ws, ws_bytes: int, stream=None) -> None:
        check(lib.llmoc_ep_p2p_serve(shard.handle, self.handle, T, seq, ptr(ws), ws_bytes, stream_ptr(stream)),
              "llmoc_ep_p2p_serve")

    def finish(self, shard, X, T: int, Y, seq: int, ws, ws_bytes: int, stream=None) -> None:
        check(lib.llmoc_ep_p2p_finish(shard.handle, self.handle, ptr(X), T, ptr(Y), seq, ptr(ws), ws_bytes,
                                      stream_ptr(stream)), "llmoc_ep_p2p_finish")

    def close(self) -> None:
        if self.handle:
            lib.llmoc_ep_transport_destroy(self.handle)
            self.handle = None


class Collective:
    """This rank's end of the NVLink collectives (llmoc_collective_*), the
    contracts::ICollective operations between the GPUs of a box."""

    ALLTOALL, ALLREDUCE_SUM, BROADCAST = 0, 1, 2
    F32, BF16 = 0, 1

    def __init__(self, world: int, rank: int, max_bytes: int, device: int = 0, export: bool = True):
        self.world, self.rank = world, rank
        h = C.c_void_p()
        self.ipc = (C.c_char * int(lib.llmoc_ep_ipc_handle_bytes()))() if export else None
        check(lib.llmoc_collective_create(world, rank, max_bytes, device, C.byref(h),
                                          C.cast(self.ipc, C.c_void_p) if export else None),
              "llmoc_collective_create")
        self.handle = h.value

    def connect(self, handles: bytes) -> None:
        """handles: every rank's IPC handle, in rank order."""
        buf = C.create_string_buffer(handles, len(handles))
        check(lib.llmoc_collective_connect(self.handle, C.cast(buf, C.c_void_p)), "llmoc_collective_connect")

    @staticmethod
    def connect_local(colls) -> None:
        """Every rank of the world in this process (tests)."""
        arr = (C.c_void_p * len(colls))(*[c.handle for c in colls])
        for c in colls:
            check(lib.llmoc_collective_connect_local(c.handle, arr), "llmoc_collective_connect_local")

    def world_size(self) -> int:
        return int(lib.llmoc_collective_world_size(self.handle))

    def error(self) -> int:
        return int(lib.llmoc_collective_error(self.handle))

    def start(self, op: int, src, nbytes: int, root: int = 0, stream=None) -> None:
        check(lib.llmoc_collective_start(self.handle, op, ptr(src), nbytes, root, stream_ptr(stream)),
              "llmoc_collective_start")

    def finish(self, op: int, dst, nbytes: int, dtype: int = 0, root: int = 0, stream=None) -> None:
        check(lib.llmoc_collective_finish(self.handle, op, ptr(dst), nbytes, dtype, root, stream_ptr(stream)),
              "llmoc_collective_finish")

    def alltoall(self, send, recv, chunk_bytes: int, stream=None) -> None:
        check(lib.llmoc_collective_alltoall(self.handle, ptr(send), ptr(recv), chunk_bytes, stream_ptr(stream)),
              "llmoc_collective_alltoall")

    def allreduce_sum(self, inout, nbytes: int, dtype: int, stream=None) -> None:
        check(lib.llmoc_collective_allreduce_sum(self.handle, ptr(inout), nbytes, dtype, stream_ptr(stream)),
              "llmoc_collective_allreduce_sum")

    def broadcast(self, buf, nbytes: int, root: int, stream=None) -> None:
        check(lib.llmoc_collective_broadcast(self.handle, ptr(buf), nbytes, root, stream_ptr(stream)),
              "llmoc_collective_broadcast")

    def close(self) -> None:
        if self.handle:
            lib.llmoc_collective_destroy(self.handle)
            self.handle = None


def qlwc_moe_layers(path: str, prefix: str) -> list:
    """Layer numbers of the QLWC file's MoE layers, ascending."""
    n = int(lib.llmoc_qlwc_moe_layers(path.encode(), prefix.encode(), None, 0))
    if n < 0:
        raise LlmocError("llmoc_qlwc_moe_layers: " + last_error())
    arr = (C.c_int32 * max(1, n))()
    lib.llmoc_qlwc_moe_layers(path.encode(), prefix.encode(), arr, n)
    return list(arr[:n])


def qlwc_describe(path: str, prefix: str, layer: int) -> QlwcLayerInfo:
    info = QlwcLayerInfo()
    check(lib.llmoc_qlwc_describe(path.encode(), prefix.encode(), layer, C.byref(info)), "llmoc_qlwc_describe")
    return info
