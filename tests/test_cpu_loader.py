"""CPU: the runtime's .knx loader (kernix_b200/csrc/knx_load.c, via the host-only kx_knx_inspect / kx_knx_plan entry
points) accepts and rejects exactly what the reference loader does, and derives the same graph.

  * the hand-made bad files of the reference's test/model_test.c:51-98 are rejected, the repaired one is accepted;
  * truncation / trailing bytes / bad magic of a good file are rejected;
  * a fuzz in the style of test/knx_fuzz_test.py:43-59 (truncate, boundary u32, random header bytes, trailing garbage)
    over the golden graphs: accept/reject agrees with the numpy oracle's reader and, where the compiled reference is
    built, with the reference itself (and so do n_steps, shapes and the storage plan of accepted files);
  * fixtures: n_steps, input/output shapes, layout and the storage plan equal the reference's."""
import os
import struct

import numpy as np
import pytest

from conftest import ROOT
from oracle import knx_oracle as ko
from oracle import ref_lib

GOLD = os.path.join(ROOT, "tests", "golden")
ALL = ["small", "wide", "inplace_first", "small_int8", "q8_s", "cnn_s", "tfm_s", "g_cnn", "g_attn", "g_rnn"]
MAGIC = 0x31584E4B  # "KNX1"


@pytest.fixture(scope="module")
def kx(libkx):
    from kernix_b200 import kx_abi
    return kx_abi


def accepts(kx, path):
    try:
        kx.inspect(path)
        return True
    except ValueError:
        return False


def write(tmp_path, name, data):
    p = str(tmp_path / name)
    with open(p, "wb") as f:
        f.write(data)
    return p


def u32s(*v):
    return struct.pack(f"<{len(v)}I", *v)


def test_reference_rejection_cases(kx, tmp_path):
    """test/model_test.c:51-98"""
    small = open(os.path.join(GOLD, "small.knx"), "rb").read()
    bad = {
        "half": small[: len(small) // 2],
        "trailing": small + b"\0\0\0\0",
        "magic": small[:3] + b"2" + small[4:],
        "zero_ops": u32s(MAGIC, 0),
        "many_ops": u32s(MAGIC, 1025),
        "huge": u32s(MAGIC, 1, 0, 0xFFFFFFFF, 0xFFFFFFFF, 1),
        "big_no_data": u32s(MAGIC, 1, 0, 30000, 30000, 0),
        "zero_dim": u32s(MAGIC, 1, 0, 0, 4, 0),
        "bad_kind": u32s(MAGIC, 1, 9),
        "bad_act": u32s(MAGIC, 1, 1, 9),
        "act_only": u32s(MAGIC, 1, 1, 0),
    }
    chain = [MAGIC, 2, 0, 4, 8, 0] + [0] * 32 + [0, 9, 2, 0] + [0] * 18  # Linear(4,8) then Linear(9,2)
    bad["chain"] = u32s(*chain)
    ln = [MAGIC, 2, 0, 4, 8, 0] + [0] * 32 + [2, 7, 0, 0x3727C5AC]  # Linear(4,8) then LayerNorm(7)
    bad["ln"] = u32s(*ln)
    for name, data in bad.items():
        p = write(tmp_path, name + ".knx", data)
        assert not accepts(kx, p), name
        with pytest.raises(ko.KnxError):
            ko.load(p)
    chain[39] = 8  # the same file as Linear(8, 2) must load
    p = write(tmp_path, "good.knx", u32s(*chain[:-2]))
    info = kx.inspect(p)
    assert (info["in_dim"], info["out_dim"], info["n_steps"]) == (4, 2, 2)


@pytest.mark.parametrize("name", ALL)
def test_fixture_structure_matches_reference(kx, name):
    p = os.path.join(GOLD, f"{name}.knx")
    info = kx.inspect(p)
    m = ko.load(p)
    assert info["n_steps"] == m["n_fused_steps"]
    assert [k for k, _ in info["steps"]] == [k for k, _ in m["fused_steps"]]
    assert [a for _, a in info["steps"]] == [a for _, a in m["fused_steps"]]
    assert info["in_shape"] == m["in_shape"] and info["out_shape"] == m["out_shape"] and info["layout"] == m["layout"]
    if ref_lib.available():
        r = ref_lib.RefModel(p)
        ri = r.info()
        assert (ri["n_steps"], ri["in_dim"], ri["out_dim"], ri["seq_len"], ri["layout"]) == \
            (info["n_steps"], info["in_dim"], info["out_dim"], info["seq_len"], info["layout"])
        assert r.steps() == info["steps"]
        assert r.plan() == kx.plan(p), "storage plan differs from the reference's"


def _mutations(data, n, rng):
    words = len(data) // 4
    for i in range(n):
        b = bytearray(data)
        kind = i % 4
        if kind == 0:
            yield bytes(b[: rng.integers(0, len(b))])
        elif kind == 1:
            w = rng.integers(0, min(words, 400))
            b[4 * w:4 * w + 4] = struct.pack("<I", int(rng.choice([0, 1, 2, 3, 7, 255, 65535, 65536, 2**31 - 1, 2**31, 2**32 - 1])))
            yield bytes(b)
        elif kind == 2:
            for _ in range(rng.integers(1, 4)):
                b[rng.integers(0, min(len(b), 1600))] = rng.integers(0, 256)
            yield bytes(b)
        else:
            yield bytes(b) + bytes(rng.integers(0, 256, rng.integers(1, 9)).astype(np.uint8))


def legacy_lstm_file():
    """A KNX1 file with the legacy LSTM record (in, units, act, ret_seq, sequence length; float weights W, U, bias)
    followed by a Linear and a softmax: the version-1/2 header rules of ACT and LSTM."""
    rng = np.random.default_rng(3)
    cin, u, T = 3, 4, 5
    rec = struct.pack("<6I", 4, cin, u, 4, 0, T)  # LSTM, tanh, last state only
    rec += rng.standard_normal(cin * 4 * u).astype("<f4").tobytes() + rng.standard_normal(u * 4 * u).astype("<f4").tobytes()
    rec += rng.standard_normal(4 * u).astype("<f4").tobytes()
    lin = struct.pack("<4I", 0, u, 2, 1) + rng.standard_normal(u * 2 + 2).astype("<f4").tobytes()
    return b"KNX1" + struct.pack("<I", 4) + rec + lin + struct.pack("<2I", 1, 0) + struct.pack("<I", 3)


@pytest.mark.parametrize("name", ["g_cnn", "g_attn", "g_rnn", "inplace_first", "cnn_s", "tfm_s", "small_int8",
                                  "legacy_lstm"])
def test_fuzzed_files_agree_with_reference(kx, name, tmp_path):
    """Every op kind's header and data rules (the golden graphs hold all 21 kinds; small_int8 and legacy_lstm the
    KNX2 / KNX1 variants)."""
    rng = np.random.default_rng(len(name))
    if name == "legacy_lstm":
        data = legacy_lstm_file()
        assert accepts(kx, write(tmp_path, "legacy_lstm.knx", data))
    else:
        data = open(os.path.join(GOLD, f"{name}.knx"), "rb").read()
    n_acc = 0
    for i, mdata in enumerate(_mutations(data, 240, rng)):
        p = write(tmp_path, f"m{i}.knx", mdata)
        mine = accepts(kx, p)
        try:
            ko.load(p)
            oracle_ok = True
        except (ko.KnxError, ValueError, OverflowError, IndexError):
            oracle_ok = False
        if ref_lib.available():
            try:
                r = ref_lib.RefModel(p)
                ref_ok = True
            except ValueError:
                ref_ok = False
            assert mine == ref_ok, f"mutation {i}: runtime {'accepts' if mine else 'rejects'}, reference does not"
            if ref_ok:
                assert r.plan() == kx.plan(p) and r.steps() == kx.inspect(p)["steps"]
                r.close()
        if oracle_ok != mine:  # the oracle's reader skips a few of the loader's range checks on RNN fields
            assert name in ("g_rnn", "legacy_lstm"), f"mutation {i}: oracle {'accepts' if oracle_ok else 'rejects'}, runtime does not"
        n_acc += mine
        os.remove(p)
    assert 0 < n_acc < 240
