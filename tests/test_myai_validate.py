"""chalot_myai_validate (host only): a file the writer made passes; a
truncated copy, extra trailing bytes, unknown flag bits and the header layout
of train_distill.py:898-915 (v2 fields packed after the v1 fields, max_seq_len
in the flags word) are reported."""
import shutil
import struct

import pytest


@pytest.fixture(scope="module")
def small(chalot, tmp_path_factory):
    d = tmp_path_factory.mktemp("val")
    return chalot.write_shape(str(d / "t.myai"), "tiny", n_layers=1, vocab_size=256)


def _copy(src, tmp_path, name):
    dst = str(tmp_path / name)
    shutil.copy(src, dst)
    return dst


def test_valid_file(chalot, small):
    from chalot_c1_b200 import myai
    ok, rep = myai.validate(small)
    assert ok and rep == []


def test_truncated_and_trailing(chalot, small, tmp_path):
    from chalot_c1_b200 import myai
    want = chalot.inspect(small)["total_bytes"]
    t = _copy(small, tmp_path, "trunc.myai")
    with open(t, "r+b") as f:
        f.truncate(want - 100)
    ok, rep = myai.validate(t)
    assert not ok and any(f"needs {want} (100 missing)" in r for r in rep)
    x = _copy(small, tmp_path, "extra.myai")
    with open(x, "ab") as f:
        f.write(b"\0" * 7)
    ok, rep = myai.validate(x)
    assert ok and rep == [f"note: 7 bytes after the last tensor (the weights end at {want})"]


def test_unknown_flag_bits(chalot, small, tmp_path):
    from chalot_c1_b200 import myai
    p = _copy(small, tmp_path, "flags.myai")
    with open(p, "r+b") as f:
        f.seek(28)
        f.write(struct.pack("<I", 0x17))
    ok, rep = myai.validate(p)
    assert not ok and any("flags 0x17" in r for r in rep)


def test_packed_v2_layout_rejected(chalot, small, tmp_path):
    """The header as train_distill.py:898-915 writes it: after vocab_size come
    max_seq, n_experts, top_k, group, flags, depth router and rope bits, packed."""
    from chalot_c1_b200 import myai
    cfg = chalot.inspect(small)
    p = _copy(small, tmp_path, "packed.myai")
    rope_bits = struct.unpack("I", struct.pack("f", cfg["rope_theta"]))[0]
    hdr = struct.pack("<14I", 0x4D594149, 2, cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["n_heads"],
                      cfg["vocab_size"], cfg["max_seq_len"], cfg["n_experts"], cfg["top_k"],
                      cfg["int4_group_size"], 1, 0, rope_bits)
    hdr += b"\0" * (256 - len(hdr))
    with open(p, "r+b") as f:
        f.write(hdr)
    ok, rep = myai.validate(p)
    assert not ok
    assert any("reserved header bytes 32-127" in r for r in rep)
    assert any(f"flags 0x{cfg['max_seq_len']:X}" in r for r in rep)


def test_bad_magic(chalot, small, tmp_path):
    from chalot_c1_b200 import myai
    p = _copy(small, tmp_path, "magic.myai")
    with open(p, "r+b") as f:
        f.write(b"XXXX")
    ok, rep = myai.validate(p)
    assert not ok and any("Bad magic" in r for r in rep)


def test_one_expert_reads_as_dense(chalot, tmp_path):
    """src/model/header.rs:17 treats n_experts < 2 as dense: a dense file whose
    header says n_experts = 1 is valid (with a note), as the reference loads it."""
    from chalot_c1_b200 import myai
    p = chalot.write_shape(str(tmp_path / "dense.myai"), "tiny", n_layers=1, vocab_size=256, n_experts=0)
    with open(p, "r+b") as f:
        f.seek(128)
        f.write(struct.pack("<I", 1))
    ok, rep = myai.validate(p)
    assert ok, rep
    assert any("n_experts 1" in r for r in rep)
