"""GPU: LSTM / GRU / SimpleRNN steps (kernix_rnn_dir / kernix_rnn_run, include/kernix_model.h:560-648) against the
numpy oracle, which is pinned to the compiled reference (tests/test_cpu_oracle_pin.py): every kind, one and two
directions with each merge, per-step and final-state outputs, float and int8 recurrent weights, a size that spans
several blocks, chunking, and an RNN inside a larger graph."""
import os

import numpy as np
import pytest

from conftest import rel_err
from oracle import knx_oracle as ko

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
F32 = np.float32


@pytest.fixture(scope="module")
def Model(libkx):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import Model
    return Model


def make(path, kind, T, cin, u, dirs, merge, ret_seq, act, int8, seed):
    from kernix_b200 import knx_writer
    rng = np.random.default_rng(seed)
    g = {"lstm": 4, "gru": 3, "rnn": 1}[kind]
    gu = g * u
    G = knx_writer.Graph((T, cin), int8=int8)
    ws = [(rng.normal(0, 0.6 / np.sqrt(cin), (cin, gu)).astype(F32), rng.normal(0, 0.6 / np.sqrt(u), (u, gu)).astype(F32),
           rng.normal(0, 0.3, 2 * gu if kind == "gru" else gu).astype(F32)) for _ in range(dirs)]
    G.rnn(0, kind, u, ws, act=act, ret_seq=ret_seq, merge=merge)
    G.write(path)
    return path


@pytest.mark.parametrize("kind", ["lstm", "gru", "rnn"])
@pytest.mark.parametrize("dirs,merge", [(1, "concat"), (2, "concat"), (2, "sum"), (2, "mul"), (2, "ave")])
@pytest.mark.parametrize("ret_seq", [0, 1])
def test_rnn_matches_oracle(Model, model_dir, kind, dirs, merge, ret_seq):
    p = make(os.path.join(model_dir, f"rnn_{kind}_{dirs}{merge}{ret_seq}.knx"), kind, 9, 5, 6, dirs, merge, ret_seq,
             "relu" if kind == "rnn" else "tanh", False, 7)
    x = np.random.default_rng(1).standard_normal((4 * 9, 5)).astype(F32)
    got = Model(p)(x)
    assert rel_err(got, ko.forward(ko.load(p), x).reshape(got.shape)) <= 1e-5


@pytest.mark.parametrize("kind", ["lstm", "gru"])
def test_rnn_int8_recurrent_weights(Model, model_dir, kind):
    """I8_COL recurrent weights run with their float copy (the reference's at more than 2 sequences per chunk)."""
    p = make(os.path.join(model_dir, f"rnn8_{kind}.knx"), kind, 6, 4, 8, 2, "concat", 1, "tanh", True, 3)
    x = np.random.default_rng(2).standard_normal((5 * 6, 4)).astype(F32)
    got = Model(p)(x)
    assert rel_err(got, ko.forward(ko.load(p), x).reshape(got.shape)) <= 1e-5


@pytest.mark.parametrize("kind", ["lstm", "gru"])
def test_rnn_wide_and_chunked(Model, model_dir, kind):
    """256 units (two blocks of units), 70 sequences (blocks of 8 rows), 24 steps; any workspace limit and piece cut
    gives bitwise the same output."""
    p = make(os.path.join(model_dir, f"rnnw_{kind}.knx"), kind, 24, 48, 256, 2, "ave", 0, "tanh", False, 5)
    x = np.random.default_rng(4).standard_normal((70 * 24, 48)).astype(F32)
    whole = Model(p, workspace_mb=0)(x)
    assert rel_err(whole, ko.forward(ko.load(p), x)) <= 1e-5
    assert np.array_equal(Model(p, workspace_mb=2)(x), whole)


def test_rnn_in_a_graph(Model, model_dir):
    """The reference fuzz test's RNN graph (GRU and LSTM in parallel, concat, a bidirectional SimpleRNN, select)."""
    p = os.path.join(os.path.dirname(__file__), "golden", "g_rnn.knx")
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "g_rnn.npz"))
    got = Model(p)(d["x0"])
    assert rel_err(got, d["y_ref0"].reshape(got.shape)) <= 1e-5
    x = np.random.default_rng(9).standard_normal((13 * 7, 5)).astype(F32)
    assert rel_err(Model(p)(x), ko.forward(ko.load(p), x)) <= 1e-5
