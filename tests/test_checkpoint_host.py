"""The engine's checkpoint loader (alphazero-go_b200/csrc/checkpoint.cpp,
azb_checkpoint_config / azb_checkpoint_read) against the reference's own
saveNetwork / loadNetwork (src/checkpoint.cpp), following the reference's
tests/test_checkpoint.cpp: round trip, missing file, bad magic and version,
a header that does not match its tensors, trailing data, truncation (inside
the tensors, inside the header, empty), the ownership flag and versions.

The fixtures in tests/golden/ were written by the reference's saveNetwork
(tests/golden/make_checkpoints.py); checkpoints.json holds the sha256 of the
arenas its loadNetwork rebuilds. Corrupted copies are made here, byte edits
as the reference's tests make them; each message is checked against the
reference loader's text (its format, src/checkpoint.cpp:36-143) and, where
the reference is built (oracle/_ref), against what it actually throws.
"""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
PLAIN = os.path.join(GOLDEN, "ckpt_9x9_b2_f16.azn")
OWNER = os.path.join(GOLDEN, "ckpt_9x9_h8_b1_f8_own.azn")
HEADER = 4 + 4 + 5 * 4   # magic, version, five shape fields


@pytest.fixture(scope="module")
def E():
    import azb200

    return azb200


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "checkpoints.json")) as f:
        return json.load(f)


def _ref_message(path):
    """The reference loader's message for `path`, or None without the reference build."""
    import oracle as O

    if not O.ref_available():
        return None
    got = O.ref_load_checkpoint(path)
    return got if isinstance(got, str) else ""


def _expect_error(E, path, message):
    with pytest.raises(RuntimeError) as e:
        E.load_checkpoint(path)
    assert str(e.value) == message
    ref = _ref_message(path)
    if ref is not None:
        assert ref == message, (ref, message)


def _write(tmp_path, name, data: bytes) -> str:
    p = str(tmp_path / name)
    with open(p, "wb") as f:
        f.write(data)
    return p


def _read(path) -> bytes:
    with open(path, "rb") as f:
        return f.read()


@pytest.mark.parametrize("name", ["ckpt_9x9_b2_f16.azn", "ckpt_9x9_h8_b1_f8_own.azn"])
def test_round_trip(E, golden, oracle, name):
    """The reference-written file loads to the arenas the reference's loader
    rebuilds (sha256), which are those of Network(cfg, seed) + the test
    randomiser in the oracle's own restatement."""
    g = golden[name]
    desc, params, buffers = E.load_checkpoint(os.path.join(GOLDEN, name))
    shape = [desc.board, desc.history, desc.blocks, desc.filters, desc.value_hidden, desc.ownership]
    assert shape == g["shape"]
    assert hashlib.sha256(params.tobytes()).hexdigest() == g["params_sha256"]
    assert hashlib.sha256(buffers.tobytes()).hexdigest() == g["buffers_sha256"]
    cfg = oracle.NetConfig(*shape[:5], bool(shape[5]))
    p2, b2 = oracle.make_network(cfg, g["seed"], oracle.KIND_TEST)
    assert np.array_equal(params.view(np.uint32), p2.view(np.uint32))
    assert np.array_equal(buffers.view(np.uint32), b2.view(np.uint32))
    d = E.checkpoint_config(os.path.join(GOLDEN, name))
    assert [d.board, d.history, d.blocks, d.filters, d.value_hidden, d.ownership] == shape


def test_missing_file(E, tmp_path):
    path = str(tmp_path / "does_not_exist.azn")
    _expect_error(E, path, "cannot open checkpoint " + path)
    with pytest.raises(RuntimeError, match="^cannot open checkpoint " + path + "$"):
        E.checkpoint_config(path)


def test_bad_magic_and_version(E, tmp_path):
    path = _write(tmp_path, "bad_magic.azn", b"NOT A CHECKPOINT AT ALL, JUST TEXT")
    _expect_error(E, path, path + ": not an AZGO checkpoint")
    data = bytearray(_read(PLAIN))
    data[4] = 7   # the version field, little-endian u32 at offset 4
    versioned = _write(tmp_path, "version7.azn", bytes(data))
    _expect_error(E, versioned, versioned + ": unsupported version 7")
    with pytest.raises(RuntimeError) as e:
        E.checkpoint_config(versioned)
    assert str(e.value) == versioned + ": unsupported version 7"


def test_header_does_not_match_tensors(E, tmp_path):
    """A header claiming one filter more than the tensors hold: the first
    tensor's size gives it away; trailing bytes are refused; a different
    architecture loads as that architecture."""
    data = bytearray(_read(PLAIN))
    data[8 + 3 * 4] += 1   # filters: the 4th i32 of the shape
    path = _write(tmp_path, "one_more_filter.azn", bytes(data))
    d = E.checkpoint_config(path)
    assert d.filters == 17
    _expect_error(E, path, path + ": tensor 'stem.conv.w' has 576 values but expected 612")
    trailing = _write(tmp_path, "trailing.azn", _read(PLAIN) + b"x")
    _expect_error(E, trailing, trailing + ": unexpected data after the last tensor")
    desc, _, _ = E.load_checkpoint(OWNER)
    assert (desc.history, desc.blocks, desc.filters, desc.ownership) == (8, 1, 8, 1)


def test_tensor_count_and_names(E, tmp_path):
    data = bytearray(_read(PLAIN))
    count = struct.unpack_from("<I", data, HEADER)[0]
    struct.pack_into("<I", data, HEADER, count + 1)
    path = _write(tmp_path, "count.azn", bytes(data))
    _expect_error(E, path, f"{path}: has {count + 1} tensors but the network needs {count}")
    data = bytearray(_read(PLAIN))
    at = HEADER + 4 + 4   # the first tensor's name, after the count and its length
    assert data[at:at + 11] == b"stem.conv.w"
    data[at] = ord("x")
    path = _write(tmp_path, "name.azn", bytes(data))
    _expect_error(E, path, path + ": tensor 0 is 'xtem.conv.w' but expected 'stem.conv.w'")
    data = bytearray(_read(PLAIN))
    struct.pack_into("<i", data, 8, 4)   # board 4: outside the shapes a checkpoint may hold
    path = _write(tmp_path, "board4.azn", bytes(data))
    _expect_error(E, path, path + ": invalid network shape in header")


def test_truncated_checkpoint_names_file(E, tmp_path):
    data = _read(PLAIN)
    path = _write(tmp_path, "half.azn", data[: len(data) // 2])
    _expect_error(E, path, path + ": truncated")
    path = _write(tmp_path, "header.azn", data[:10])
    _expect_error(E, path, path + ": truncated")
    with pytest.raises(RuntimeError) as e:
        E.checkpoint_config(path)
    assert str(e.value) == path + ": truncated"
    path = _write(tmp_path, "empty.azn", b"")
    _expect_error(E, path, path + ": truncated")


def test_ownership_flag_and_versions(E, golden, tmp_path):
    """Version 1 has no flag; version 2 a flag of 1 (or 0: a plain network);
    any other flag is a corrupt header."""
    p, o = _read(PLAIN), _read(OWNER)
    assert struct.unpack_from("<I", p, 4)[0] == 1
    assert struct.unpack_from("<II", o, 4)[0] == 2 and struct.unpack_from("<i", o, HEADER)[0] == 1
    v2plain = bytearray(p)
    v2plain[4] = 2
    v2plain[HEADER:HEADER] = b"\0\0\0\0"
    path = _write(tmp_path, "v2plain.azn", bytes(v2plain))
    desc, params, buffers = E.load_checkpoint(path)
    assert desc.ownership == 0
    assert hashlib.sha256(params.tobytes()).hexdigest() == golden["ckpt_9x9_b2_f16.azn"]["params_sha256"]
    bad = bytearray(o)
    bad[HEADER] = 2
    path = _write(tmp_path, "bad_flag.azn", bytes(bad))
    _expect_error(E, path, path + ": invalid ownership flag in header")


def test_leftover_tmp_is_ignored(E, tmp_path):
    """A stale "<path>.tmp" from an interrupted save does not affect loading."""
    path = _write(tmp_path, "leftover.azn", _read(PLAIN))
    _write(tmp_path, "leftover.azn.tmp", b"half-written garbage from a crash")
    desc, _, _ = E.load_checkpoint(path)
    assert desc.filters == 16
