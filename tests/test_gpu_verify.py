"""The verify workflow on this library (survey's next step: the reference's tools/verify.py): a PyTorch original and
its .knx agree within the tolerance (exit 0), and a .knx whose weights differ is caught (exit 1)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_verify_pytorch_original(tmp_path, capsys):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import knx_writer, verify
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(20, 64), torch.nn.ReLU(), torch.nn.Linear(64, 10), torch.nn.Tanh())
    pt = str(tmp_path / "model.pt")
    torch.save(model, pt)
    layers = [(model[0].weight.detach().numpy().T, model[0].bias.detach().numpy()),
              (model[2].weight.detach().numpy().T, model[2].bias.detach().numpy())]

    def write(path, bump=0.0):
        s = knx_writer.Sequential()
        s.linear(layers[0][0] + bump, layers[0][1]).act("relu").linear(layers[1][0], layers[1][1]).act("tanh")
        s.write(path)

    good, bad = str(tmp_path / "good.knx"), str(tmp_path / "bad.knx")
    write(good)
    write(bad, bump=0.01)
    assert verify.main([pt, good, "--batch", "32"]) == 0
    out = capsys.readouterr().out
    assert "verdict: pass" in out and "largest relative error" in out
    assert verify.main([pt, bad, "--batch", "32"]) == 1
    assert "verdict: FAIL" in capsys.readouterr().out
