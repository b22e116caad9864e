"""Check that a .knx gives the answers of the model it was converted from, and how fast, on this library.

    python -m kernix_b200.verify model.pt model.knx [--input x.npy] [--batch 64] [--tol 1e-4]
    python -m kernix_b200.verify model.h5 model.knx          (Keras / TFLite originals need tensorflow)

The same workflow as the reference's tools/verify.py (its arguments, report and exit code): the original runs in its
own framework, the .knx through kernix_b200.Model on the GPU, both on the same input (the --input .npy, first axis the
batch, or seeded standard-normal samples); it prints the largest error relative to the original's output scale
(max |a - b| / max |a|), the argmax agreement and the batch-1 and whole-batch times, and exits with 1 when the error
exceeds --tol. torch.load unpickles: only pass files you made.
"""
import argparse
import statistics
import sys
import time

import numpy as np

from .kernix import Model


def load_original(path):
    """(framework name, numpy -> numpy function) of the original model (reference tools/verify.py:25-52)"""
    ext = path.rsplit(".", 1)[-1].lower() if "." in path else ""
    if ext in ("pt", "pth"):
        import torch
        model = torch.load(path, weights_only=False).eval()

        def run(x):
            with torch.no_grad():
                return model(torch.from_numpy(x)).numpy()
        return "PyTorch", run
    if ext in ("h5", "keras", "tflite"):
        import tensorflow as tf  # noqa: F401  (absent here: reported as a missing package)
        raise ValueError("Keras / TFLite originals: run this tool where tensorflow is installed")
    raise ValueError(f"extension .{ext}: .h5/.keras, .tflite or .pt/.pth")


def compare(want, got):
    """(largest error relative to the output scale, argmax agreement or None); absolute error if the original's
    output is all zeros (reference tools/verify.py:55-63)"""
    want, got = np.asarray(want, np.float64), np.asarray(got, np.float64).reshape(np.shape(want))
    scale = np.abs(want).max()
    err = np.abs(want - got).max() / (scale if scale > 0 else 1.0)
    agree = (want.argmax(-1) == got.argmax(-1)).mean() if want.ndim >= 2 and want.shape[-1] >= 2 else None
    return float(err), agree


def median_ms(fn, x, runs=20):
    """median of `runs` back-to-back calls after 3 warm-up calls"""
    for _ in range(3):
        fn(x)
    t = []
    for _ in range(runs):
        s = time.perf_counter()
        fn(x)
        t.append((time.perf_counter() - s) * 1000)
    return statistics.median(t)


def main(argv=None):
    ap = argparse.ArgumentParser(description="compare a KERNIX .knx with its original model on the GPU")
    ap.add_argument("original", help=".pt/.pth (or .h5/.keras/.tflite where tensorflow is installed)")
    ap.add_argument("knx", help="the converted .knx")
    ap.add_argument("--input", help="input .npy (first axis: batch); default seeded standard-normal samples")
    ap.add_argument("--batch", type=int, default=64, help="samples of the random input (default 64)")
    ap.add_argument("--tol", type=float, default=1e-4, help="largest allowed relative error (default 1e-4)")
    a = ap.parse_args(argv)
    if a.batch < 1:
        ap.error("--batch must be at least 1")
    try:
        m = Model(a.knx)
    except (ValueError, OSError) as e:
        ap.error(str(e))
    if a.input:
        x = np.load(a.input)
        if x.ndim < 2 or tuple(x.shape[1:]) != m.in_shape:
            ap.error(f"--input shape {x.shape}: expected (batch, {', '.join(map(str, m.in_shape))})")
        x = np.ascontiguousarray(x, np.float32)
    else:
        x = np.random.default_rng(0).standard_normal((a.batch,) + tuple(m.in_shape)).astype(np.float32)
    try:
        name, original = load_original(a.original)
    except ImportError as e:
        ap.error(f"the original needs a package that is not installed ({e.name})")
    except ValueError as e:
        ap.error(str(e))
    try:
        want = original(x)
    except Exception as e:  # noqa: BLE001  the original's own failure, reported with its cause
        ap.error(f"the original failed: {type(e).__name__}: {e}")
    got = m(x)
    err, agree = compare(want, got)
    n = len(x)
    print(f"input: {a.input} ({n} samples)" if a.input else f"input: {n} standard-normal samples (seed 0)")
    print(f"{'':24}{name:>12}{'KERNIX-B200':>14}")
    print(f"{'largest relative error':24}{'':>12}{err:>14.1e}")
    print(f"{'argmax agreement':24}{'':>12}{'-' if agree is None else f'{agree * 100:.1f}%':>14}")
    for b in sorted({1, n}):
        print(f"{f'batch {b} time':24}{median_ms(original, x[:b]):>9.3f} ms{median_ms(m, x[:b]):>11.3f} ms")
    ok = err <= a.tol
    print(f"verdict: {'pass' if ok else 'FAIL'} (tolerance {a.tol:g})")
    m.close()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
