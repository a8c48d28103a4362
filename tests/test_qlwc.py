"""The QLWC loader's file side, on the CPU: a one-layer file written by the
reference's own tools/quantize_int4.py (write_qlwc, fixture in
tests/golden/qlwc_cases.npz) described through the C ABI, and malformed files
refused with LLMOC_ERR_INVALID.  The device side (upload, forward) is in
tests/test_gpu_moe.py."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as mg  # noqa: E402
import llmoc_b200 as L  # noqa: E402


def qlwc_file(tmp_path) -> str:
    blob = np.load(os.path.join(HERE, "golden", "qlwc_cases.npz"))["qlwc_gptq_shared_gate/file"]
    p = tmp_path / "layer.qlwc"
    p.write_bytes(blob.tobytes())
    return str(p)


def test_describe_reference_written_file(tmp_path):
    path = qlwc_file(tmp_path)
    kw = mg.QLWC_CASE["kw"]
    info = L.qlwc_describe(path, mg.QLWC_CASE["prefix"], mg.QLWC_CASE["layer"])
    assert (info.hidden, info.inter, info.n_experts, info.group_size) == (kw["H"], kw["I"], kw["E"], kw["gs"])
    assert info.scheme == L.SCHEME_GPTQ_ASYM
    assert (info.has_router, info.has_shared, info.has_shared_gate, info.has_bias) == (1, 1, 1, 0)


def test_missing_layer_and_bad_files(tmp_path):
    path = qlwc_file(tmp_path)
    with pytest.raises(L.LlmocError):  # no such layer
        L.qlwc_describe(path, mg.QLWC_CASE["prefix"], mg.QLWC_CASE["layer"] + 1)
    raw = bytearray(open(path, "rb").read())
    bad = tmp_path / "bad_magic.qlwc"
    bad.write_bytes(b"XXXX" + bytes(raw[4:]))
    with pytest.raises(L.LlmocError):
        L.qlwc_describe(str(bad), "model.", 3)
    raw[40] ^= 0xFF  # a catalog byte: the FNV-1a checksum no longer matches
    bad2 = tmp_path / "bad_crc.qlwc"
    bad2.write_bytes(bytes(raw))
    with pytest.raises(L.LlmocError):
        L.qlwc_describe(str(bad2), "model.", 3)
    short = tmp_path / "short.qlwc"
    short.write_bytes(bytes(raw[:20]))
    with pytest.raises(L.LlmocError):
        L.qlwc_describe(str(short), "model.", 3)


def _fnv1a64(b: bytes) -> int:
    h = 14695981039346656037
    for c in b:
        h = ((h ^ c) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def test_int4_payload_sizes_checked(tmp_path):
    """A catalog whose first INT4 tensor claims only M scales (instead of M x
    K/gs) is refused, even with a valid checksum."""
    import struct

    raw = bytearray(open(qlwc_file(tmp_path), "rb").read())
    clen = struct.unpack_from("<Q", raw, 8)[0]
    cat = bytearray(raw[24:24 + clen])
    p = 12
    n = struct.unpack_from("<Q", cat, p)[0]
    p += 8
    for _ in range(n):
        ln = struct.unpack_from("<I", cat, p)[0]
        p += 4 + ln
        kind = struct.unpack_from("<I", cat, p)[0]
        rank = struct.unpack_from("<Q", cat, p + 4)[0]
        dims = struct.unpack_from(f"<{rank}Q", cat, p + 12)
        p += 12 + 8 * rank
        if kind == 1:
            s_n_at = p + 4 + 8 * 3  # gs, q_off, q_n, s_off, then s_n
            struct.pack_into("<Q", cat, s_n_at, dims[0] * 2)
            break
        p += 4 + 16
    raw[24:24 + clen] = cat
    struct.pack_into("<Q", raw, 16, _fnv1a64(bytes(cat)))
    bad = tmp_path / "bad_sizes.qlwc"
    bad.write_bytes(bytes(raw))
    with pytest.raises(L.LlmocError):
        L.qlwc_describe(str(bad), "model.", 3)


# --------------------------------------------------------------------------
# A minimal QLWC v1 writer (the container of src/weights/qlwc_format.cpp:
# preface "QLW1", u32 version, u64 catalog bytes, u64 FNV-1a 64 of the
# catalog; catalog = u32 scheme, u32 group size, u32 alignment, u64 count,
# then per tensor name, kind, rank, dims and its payload records).  Payload
# bytes are zeros: describe reads the catalog only.

def _qlwc_bytes(scheme, gs, tensors):
    import struct

    cat = bytearray(struct.pack("<IIIQ", scheme, gs, 64, len(tensors)))
    off = 4096
    for t in tensors:
        name = t["name"].encode()
        cat += struct.pack("<I", len(name)) + name + struct.pack("<IQ", t["kind"], len(t["shape"]))
        cat += struct.pack(f"<{len(t['shape'])}Q", *t["shape"])
        if t["kind"] == 0:
            cat += struct.pack("<IQQ", t["dtype"], off, t["nbytes"])
            off += t["nbytes"]
        else:
            cat += struct.pack("<I", gs)
            for n in (t["q"], t["s"], t["z"]):
                cat += struct.pack("<QQ", off, n)
                off += n
    pre = b"QLW1" + struct.pack("<IQQ", 1, len(cat), _fnv1a64(bytes(cat)))
    body = pre + bytes(cat)
    return body + bytes(max(0, off - len(body)))


def _int4(name, M, K, gs, gptq=True, zeros=None):
    ng = K // gs
    z = (M * ng * 2 if gptq else 0) if zeros is None else zeros
    return dict(name=name, kind=1, shape=[M, K], q=M * K // 2, s=M * ng * 2, z=z)


def _layer(base, E, H, I, gs, gptq, shared=None, router=True, bias_dtype=None, zeros=None):
    ts = []
    for e in range(E):
        for pn, (M, K) in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            ts.append(_int4(f"{base}experts.{e}.{pn}.weight", M, K, gs, gptq, zeros))
    if shared:
        for pn, (M, K) in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            ts.append(_int4(f"{base}{shared}{pn}.weight", M, K, gs, gptq))
    if router:
        ts.append(dict(name=base + "gate.weight", kind=0, shape=[E, H], dtype=1, nbytes=E * H * 2))
    if bias_dtype:
        ts.append(dict(name=base + "gate.e_score_correction_bias", kind=0, shape=[E], dtype=bias_dtype,
                       nbytes=E * 2))
    return ts


def test_describe_glm_naming_awq_with_bias(tmp_path):
    """GLM/DeepSeek-style names (shared_experts.), AWQ (no zeros), a 16-bit
    selection bias, five experts."""
    p = tmp_path / "glm.qlwc"
    p.write_bytes(_qlwc_bytes(2, 64, _layer("model.layers.7.mlp.", 5, 256, 128, 64, False,
                                              shared="shared_experts.", bias_dtype=2)))
    info = L.qlwc_describe(str(p), "model.", 7)
    assert (info.hidden, info.inter, info.n_experts, info.group_size, info.scheme) == (256, 128, 5, 64, 2)
    assert (info.has_router, info.has_shared, info.has_shared_gate, info.has_bias) == (1, 1, 0, 1)


def test_describe_without_router_and_bad_zeros(tmp_path):
    p = tmp_path / "norouter.qlwc"
    p.write_bytes(_qlwc_bytes(1, 64, _layer("model.layers.0.mlp.", 4, 128, 64, 64, True, router=False)))
    info = L.qlwc_describe(str(p), "model.", 0)
    assert (info.n_experts, info.has_router, info.has_shared, info.has_bias) == (4, 0, 0, 0)
    p2 = tmp_path / "nozeros.qlwc"  # GPTQ experts without their fp16 zeros
    p2.write_bytes(_qlwc_bytes(1, 64, _layer("model.layers.0.mlp.", 4, 128, 64, 64, True, zeros=0)))
    with pytest.raises(L.LlmocError):
        L.qlwc_describe(str(p2), "model.", 0)
    p3 = tmp_path / "awqzeros.qlwc"  # AWQ experts with a zeros payload
    p3.write_bytes(_qlwc_bytes(2, 64, _layer("model.layers.0.mlp.", 4, 128, 64, 64, False, zeros=128 * 2 * 2)))
    with pytest.raises(L.LlmocError):
        L.qlwc_describe(str(p3), "model.", 0)


def test_moe_layer_listing(tmp_path):
    """llmoc_qlwc_moe_layers: the reference-written file holds layer 3; a file
    with MoE layers 0, 7 and 12 and a dense MLP layer 5 lists the three MoE
    layers in order; a file that is not QLWC is an error."""
    assert L.qlwc_moe_layers(qlwc_file(tmp_path), "model.") == [3]
    ts = []
    for n in (12, 0, 7):
        ts += _layer(f"model.layers.{n}.mlp.", 2, 128, 64, 64, False)
    ts.append(_int4("model.layers.5.mlp.gate_proj.weight", 64, 128, 64, False))  # a dense MLP
    p = tmp_path / "three.qlwc"
    p.write_bytes(_qlwc_bytes(2, 64, ts))
    assert L.qlwc_moe_layers(str(p), "model.") == [0, 7, 12]
    assert L.qlwc_moe_layers(str(p), "other.") == []
    bad = tmp_path / "bad.qlwc"
    bad.write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(L.LlmocError):
        L.qlwc_moe_layers(str(bad), "model.")
