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
