"""The .myai format and the host-side C ABI (no GPU needed).

Offsets and sizes are checked against an arithmetic restatement of
src/model/weight_index.rs:85-263 written here, against the byte counts the
blueprint derives for the three model shapes, and against the oracle's own
parser; malformed files must be rejected with the reference's messages
(header.rs:101-109, engine.rs:98-100).
"""
import os
import re
import struct

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def expert_bytes(d, H, g):
    return 2 * H * ((d + 1) // 2) + 2 * H * ((d + g - 1) // g) * 4 + d * ((H + 1) // 2) + \
        d * ((H + g - 1) // g) * 4


def test_expert_and_file_sizes(chalot):
    # per-expert bytes: Qwen 8,171,520; 1B 21,626,880; tiny 491,520
    assert expert_bytes(896, 4864, 32) == 8_171_520
    assert expert_bytes(2048, 5632, 32) == 21_626_880
    assert expert_bytes(256, 1024, 32) == 491_520
    assert chalot.myai.inspect_expected("tiny") == 18_965_888


def test_writer_matches_index(chalot, tmp_path):
    for over in ({}, {"n_experts": 1, "top_k": 1}, {"int4_group_size": 64}):
        p = chalot.write_shape(str(tmp_path / "m.myai"), "tiny", n_layers=2, vocab_size=512, **over)
        info = chalot.inspect(p)
        assert os.path.getsize(p) == info["total_bytes"]
        assert info["total_bytes"] == chalot.myai.inspect_expected("tiny", n_layers=2, vocab_size=512, **over)


def test_header_fields(chalot, tmp_path):
    p = chalot.write_shape(str(tmp_path / "q.myai"), "tiny", n_layers=1, vocab_size=256,
                           rope_theta_x100=100000000, max_seq_len=2048)
    raw = open(p, "rb").read(256)
    u = struct.unpack_from("<8I", raw, 0)
    v2 = struct.unpack_from("<6I", raw, 128)
    assert u[0] == 0x4D594149 and u[1] == 2 and u[2:7] == (256, 1024, 1, 4, 256)
    assert u[7] == 0b111  # quantized | int4 | moe
    assert v2 == (8, 2, 32, 0, 2048, 100000000)
    info = chalot.inspect(p)
    assert info["rope_theta"] == 1e6 and info["head_dim"] == 64


def test_config_defaults(chalot, tmp_path):
    # config.rs:40-69: top_k 0 -> min(E,2); group 0 -> 64; max_seq 0 -> 512;
    # rope 0 -> 10000; n_experts < 2 -> 1
    p = str(tmp_path / "d.myai")
    chalot.write_shape(p, "tiny", n_layers=1, vocab_size=256, int4_group_size=64, max_seq_len=512)
    raw = bytearray(open(p, "rb").read())
    struct.pack_into("<I", raw, 132, 0)  # top_k
    struct.pack_into("<I", raw, 136, 0)  # group (64 is the default)
    struct.pack_into("<I", raw, 144, 0)  # max_seq
    open(p, "wb").write(raw)
    info = chalot.inspect(p)
    assert info["top_k"] == 2 and info["int4_group_size"] == 64 and info["max_seq_len"] == 512
    assert info["rope_theta"] == 10000.0


@pytest.mark.parametrize("mutate,msg", [
    (lambda r: struct.pack_into("<I", r, 0, 0x12345678), "Bad magic: 0x12345678"),
    (lambda r: struct.pack_into("<I", r, 4, 3), "Unsupported version: 3"),
    (lambda r: struct.pack_into("<I", r, 4, 0), "Unsupported version: 0"),
])
def test_bad_headers_rejected(chalot, tmp_path, mutate, msg):
    p = str(tmp_path / "bad.myai")
    chalot.write_shape(p, "tiny", n_layers=1, vocab_size=256)
    raw = bytearray(open(p, "rb").read())
    mutate(raw)
    open(p, "wb").write(raw)
    with pytest.raises(chalot.ChalotError) as ei:
        chalot.inspect(p)
    assert ei.value.code == -3 and msg in str(ei.value)


def test_short_file_rejected(chalot, tmp_path):
    p = str(tmp_path / "short.myai")
    open(p, "wb").write(b"MYAI" * 8)
    with pytest.raises(chalot.ChalotError, match="File too small for header"):
        chalot.inspect(p)


def test_missing_file(chalot):
    with pytest.raises(chalot.ChalotError) as ei:
        chalot.inspect("/nonexistent/model.myai")
    assert ei.value.code == -2


def test_oracle_parses_same_sizes(chalot, oracle_lib, tmp_path):
    p = chalot.write_shape(str(tmp_path / "o.myai"), "tiny", n_layers=2, vocab_size=512)
    e = oracle_lib.OracleEngine(p, threads=1)
    assert e.config["total_bytes"] == chalot.inspect(p)["total_bytes"]


def test_writer_deterministic_across_threads(chalot, tmp_path):
    a = chalot.write_shape(str(tmp_path / "a.myai"), "tiny", n_layers=1, vocab_size=512, n_threads=1)
    b = chalot.write_shape(str(tmp_path / "b.myai"), "tiny", n_layers=1, vocab_size=512, n_threads=7)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_writer_quantization_semantics(chalot, tmp_path):
    """int8 tensors carry one per-tensor scale in every row slot; int4 expert
    scales are per row and group, and every packed byte decodes to -8..7."""
    p = chalot.write_shape(str(tmp_path / "s.myai"), "tiny", n_layers=1, vocab_size=512)
    raw = np.fromfile(p, np.uint8)
    d, H, V, g = 256, 1024, 512, 32
    off = 256
    emb = raw[off:off + V * d].view(np.int8)
    off += V * d
    es = raw[off:off + V * 4].view(np.float32)
    off += V * 4
    assert np.all(es == es[0]) and np.abs(emb).max() == 127
    off += d * 4  # rms_attn
    qkv = raw[off:off + 3 * d * d].view(np.int8)
    assert np.abs(qkv).max() == 127
    off += 3 * d * d
    qs = raw[off:off + 3 * d * 4].view(np.float32)
    assert np.all(qs == qs[0])
    off += 3 * d * 4 + d * d + d * 4 + d * 4 + 8 * d * 4 + 8 * 4  # O, O scales, rms_ffn, router
    gu = raw[off:off + 2 * H * d // 2]
    lo, hi = (gu & 0xF).astype(int) - 8, (gu >> 4).astype(int) - 8
    assert lo.min() >= -8 and hi.max() <= 7 and (lo == 7).any() or (lo == -7).any()
    off += 2 * H * d // 2
    gs = raw[off:off + 2 * H * (d // g) * 4].view(np.float32)
    assert gs.min() > 0 and len(np.unique(gs)) > 1000


def test_header_declares_every_exported_symbol(chalot):
    """Every function include/chalot_b200.h declares is exported by the
    library and bound in the Python ctypes table (no compute is called)."""
    import ctypes
    from chalot_c1_b200 import _capi
    hdr = open(os.path.join(ROOT, "include", "chalot_b200.h")).read()
    names = set(re.findall(r"\b(chalot_[a-z0-9_]+)\s*\(", hdr))
    assert names, "no declarations found"
    L = ctypes.CDLL(_capi.LIB_PATH)
    for n in sorted(names):
        assert hasattr(L, n), f"{n} not exported"
        assert n in _capi.SIGNATURES, f"{n} not bound in _capi.SIGNATURES"
    assert _capi.lib().chalot_abi_version() == 100
