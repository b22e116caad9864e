"""GPU: each golden fixture (models exported by the reference's own tools, outputs from the reference's own compiled
forward -- tests/golden/make_golden.py) through the public API, against those reference outputs."""
import os

import numpy as np
import pytest

from conftest import ROOT, rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
GOLD = os.path.join(ROOT, "tests", "golden")
# wide's last layer has K = 9000: it drains its partial sums every 256 (the GEMM's long-reduction mode), which keeps
# it at the dense-MLP bound 1e-5; the reference's own bound for this model is 1e-4 (test/model_test.c:127-142)
TOL = dict(small=1e-5, wide=1e-5, inplace_first=1e-5, small_int8=1e-4, q8_s=1e-4, cnn_s=1e-4, tfm_s=1e-4, g_cnn=1e-5,
           g_attn=1e-5, g_rnn=1e-5)


@pytest.fixture(scope="module")
def Model(libkx):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import Model
    return Model


@pytest.mark.parametrize("name", sorted(TOL))
def test_fixture_matches_reference_forward(Model, name):
    m = Model(os.path.join(GOLD, f"{name}.knx"))
    d = np.load(os.path.join(GOLD, f"{name}.npz"))
    i = 0
    while f"x{i}" in d.files:
        x, want = d[f"x{i}"], d[f"y_ref{i}"]
        got = m(x.reshape(-1, m.in_dim)).reshape(want.shape)
        assert rel_err(got, want) <= TOL[name], f"input {i}"
        i += 1
