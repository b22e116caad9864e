"""CPU: pin the numpy oracle (oracle/knx_oracle.py) to the reference.

  * golden fixtures (tests/golden/, made by make_golden.py with the reference's own exporters and compiled forward):
    oracle == reference output, and oracle ~ PyTorch within the reference zoo test's bounds (test/zoo_torch_test.py:53-54,
    :207-208);
  * the reference's int8 known answers (test/model_test.c:363-446): LCG-generated cases, NaN and zero rows, the int32
    overflow edge -- oracle == a scalar int64 restatement of the test's ref_qmatmul, and == the compiled reference's
    kernix_qmatmul bit for bit when oracle/_ref is built;
  * the five benchmark configurations, and LSTM / GRU / SimpleRNN steps in every direction, merge and output mode
    with float and int8 recurrent weights, when the compiled reference is present."""
import os

import numpy as np
import pytest

from conftest import ROOT, rel_err
from oracle import knx_oracle as ko
from oracle import ref_lib

GOLD = os.path.join(ROOT, "tests", "golden")
FIXTURES = ["small", "wide", "inplace_first", "small_int8", "q8_s", "cnn_s", "tfm_s", "g_cnn", "g_attn", "g_rnn"]
INT8 = {"small_int8", "q8_s"}


def load_fixture(name):
    d = np.load(os.path.join(GOLD, f"{name}.npz"))
    n = len([k for k in d.files if k.startswith("x")])
    return [(d[f"x{i}"], d[f"y_ref{i}"], d.get(f"y_torch{i}")) for i in range(n)]


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_matches_reference_outputs(name):
    model = ko.load(os.path.join(GOLD, f"{name}.knx"))
    for x, y_ref, y_torch in load_fixture(name):
        got = ko.forward(model, x).reshape(y_ref.shape)
        if name in INT8:
            # int8 layers are bit-exact; GELU between them uses numpy's exp vs glibc's expf, so a requantisation may
            # flip by one step -- bounded by the reference's own int8 tolerance on the output scale
            assert rel_err(got, y_ref) <= 1e-4
        else:
            assert rel_err(got, y_ref) <= 1e-5
        if y_torch is not None:
            assert rel_err(got, y_torch.reshape(got.shape)) <= (5e-2 if name in INT8 else 2e-4)


def _lcg(seed=12345):
    state = [seed]

    def qrand():
        state[0] = (state[0] * 1664525 + 1013904223) & 0xFFFFFFFF
        return state[0] >> 8
    return qrand


def ref_qmatmul_int64(x, q, scale, bias):
    """test/model_test.c:363-382: same quantisation, int64 accumulation, scalar loops (vectorised here)."""
    m = np.max(np.abs(x), axis=1)
    sx = np.where(m > 0, m / np.float32(127), np.float32(1)).astype(np.float32)
    inv = (np.float32(1) / sx).astype(np.float32)
    v = np.clip(np.rint((x * inv[:, None]).astype(np.float32)), -127, 127).astype(np.int64)
    acc = v @ q.astype(np.int64)
    r = ((acc.astype(np.float32) * sx[:, None]).astype(np.float32) * scale[None, :]).astype(np.float32)
    return (r + (bias if bias is not None else np.float32(0))).astype(np.float32)


@pytest.mark.parametrize("k,n,rows", [(55, 31, 1), (64, 256, 1), (128, 512, 3), (114, 512, 32), (16, 16, 1), (1, 1, 1)])
def test_int8_known_answers(k, n, rows):
    qrand = _lcg()
    q = np.array([(qrand() % 255) - 127 for _ in range(k * n)], np.int8).reshape(k, n)
    scale = np.empty(n, np.float32)
    bias = np.empty(n, np.float32)
    for i in range(n):
        scale[i] = np.float32(0.001) + np.float32(qrand() % 1000) * np.float32(1e-5)
        bias[i] = np.float32(qrand() % 200) * np.float32(0.01) - np.float32(1.0)
    x = np.array([np.float32(qrand() % 2001) * np.float32(0.003) - np.float32(3.0) for _ in range(rows * k)], np.float32)
    x = x.reshape(rows, k)
    got = ko.qlinear(x, q, scale, bias)
    assert np.array_equal(got, ref_qmatmul_int64(x, q, scale, bias))
    if ref_lib.available():
        assert np.array_equal(got.view(np.uint32), ref_lib.qmatmul(x, q, scale, bias).view(np.uint32))
    if rows >= 3:  # row 1 has a NaN -> whole row NaN; row 2 is zero -> exactly the bias (model_test.c:413-425)
        x[1, 0] = np.nan
        x[2, :] = 0.0
        got = ko.qlinear(x, q, scale, bias)
        assert np.all(np.isnan(got[1])) and np.array_equal(got[2], bias)
        assert not np.any(np.isnan(got[0]))


def test_int8_int32_edge():
    """test/model_test.c:430-440: K = 131072, q = -128, x = 1 -> exactly -128*127*K/127, no int32 overflow."""
    k = ko.INT8_MAX_K
    q = np.full((k, 1), -128, np.int8)
    got = ko.qlinear(np.ones((1, k), np.float32), q, np.ones(1, np.float32), None)
    assert got[0, 0] == np.float32(-128.0 * 127.0 * k) * np.float32(1.0 / 127.0)


@pytest.mark.reference
@pytest.mark.skipif(not ref_lib.available(), reason="compiled reference (oracle/_ref) not built here")
@pytest.mark.parametrize("cfg,batch", [("c1", 16), ("c2", 3), ("c3", 2), ("c4", 1), ("c5", 3)])
def test_oracle_matches_reference_on_configs(cfg, batch, tmp_path):
    from kernix_b200 import configs
    p = configs.model_path(cfg, str(tmp_path))
    m = ref_lib.RefModel(p)
    if cfg == "c2":
        m.set_workspace_limit(1)
    x = configs.inputs(cfg, batch)
    assert rel_err(ko.forward(ko.load(p), x), m.forward(x)) <= (1e-4 if cfg == "c2" else 1e-5)
    m.close()


def rnn_model(path, kind, T, cin, u, dirs, merge, ret_seq, act, int8, rng):
    from kernix_b200 import knx_writer
    g = {"lstm": 4, "gru": 3, "rnn": 1}[kind]
    gu = g * u
    G = knx_writer.Graph((T, cin), int8=int8)
    ws = [(rng.normal(0, 0.4, (cin, gu)).astype(np.float32), rng.normal(0, 0.4, (u, gu)).astype(np.float32),
           rng.normal(0, 0.3, 2 * gu if kind == "gru" else gu).astype(np.float32)) for _ in range(dirs)]
    G.rnn(0, kind, u, ws, act=act, ret_seq=ret_seq, merge=merge)
    G.write(path)


@pytest.mark.reference
@pytest.mark.skipif(not ref_lib.available(), reason="compiled reference (oracle/_ref) not built here")
@pytest.mark.parametrize("kind", ["lstm", "gru", "rnn"])
@pytest.mark.parametrize("dirs,merge", [(1, "concat"), (2, "concat"), (2, "sum"), (2, "mul"), (2, "ave")])
def test_oracle_rnn_matches_reference(kind, dirs, merge, tmp_path):
    """kernix_rnn_dir / kernix_rnn_run (include/kernix_model.h:560-648): every output mode, float recurrent weights,
    and int8 ones both below (the reference's int8 kernel, B <= 2) and above its row threshold."""
    rng = np.random.default_rng(len(kind) * 10 + dirs)
    for ret_seq in (0, 1):
        for int8, B in ((False, 5), (True, 2), (True, 4)):
            p = str(tmp_path / f"{kind}_{ret_seq}_{int8}.knx")
            rnn_model(p, kind, 7, 5, 6, dirs, merge, ret_seq, "relu" if kind == "rnn" else "tanh", int8, rng)
            x = rng.standard_normal((B * 7, 5)).astype(np.float32)
            r = ref_lib.RefModel(p)
            want = r.forward(x)
            r.close()
            assert rel_err(ko.forward(ko.load(p), x), want) <= 1e-6, (ret_seq, int8, B)
