"""GPU: output-column sharding of wide dense layers (kernix_model_load_sharded). On one GPU the ranks are threads
of this process with a host-side all-gather (each rank waits for its slice, deposits it, and copies every
slice into its receive buffer); on two GPUs, tests/shard_worker.py runs under torchrun with NCCL. Each rank keeps
only its slice of every wide LINEAR's weights, yet every rank returns the full output, equal to the unsharded
model's."""
import os
import subprocess
import sys
import threading

import numpy as np
import pytest

from conftest import ROOT, rel_err
from oracle import knx_oracle as ko

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
F32 = np.float32


class ThreadGather:
    """All-gather among `world` threads of one process (one GPU), done on the host with stream syncs: no kernel
    waits on another."""

    def __init__(self, world):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots = [None] * world

    def fn(self, rank):
        from kernix_b200.shard import _DevArray

        def gather(send, recv, count, stream):
            torch.cuda.ExternalStream(stream).synchronize()  # the slice's GEMM has finished
            self.slots[rank] = torch.as_tensor(_DevArray(send, count), device="cuda").clone()
            torch.cuda.current_stream().synchronize()
            self.barrier.wait()
            dst = torch.as_tensor(_DevArray(recv, count * self.world), device="cuda")
            dst.copy_(torch.cat(self.slots))
            torch.cuda.current_stream().synchronize()
            self.barrier.wait()  # every rank has read the slots before they are reused

        return gather


def run_ranks(path, world, x):
    from kernix_b200 import Model
    tg = ThreadGather(world)
    models = [Model(path, shard=(r, world, tg.fn(r))) for r in range(world)]
    outs, errs = [None] * world, []

    def work(r):
        try:
            outs[r] = models[r](x)
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    th = [threading.Thread(target=work, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    for m in models:
        m.close()
    assert not errs, errs
    return outs


@pytest.fixture(scope="module")
def wide_mlp(model_dir):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import knx_writer
    rng = np.random.default_rng(11)
    p = os.path.join(model_dir, "shard_mlp.knx")
    dims = [512, 2048, 3072, 1024, 10]  # 2048 / 3072 / 1024 outputs shard (>= 1024, divisible); 10 runs whole
    s = knx_writer.Sequential()
    for i in range(4):
        w = (rng.standard_normal((dims[i], dims[i + 1])) * np.sqrt(2.0 / dims[i])).astype(F32)
        s.linear(w, np.full(dims[i + 1], 0.01, F32))
        if i < 3:
            s.act("relu")
    s.write(p)
    return p


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_ranks_equal_unsharded(wide_mlp, world):
    from kernix_b200 import Model
    x = np.random.default_rng(world).uniform(-1, 1, (37, 512)).astype(F32)
    full = Model(wide_mlp)(x)
    outs = run_ranks(wide_mlp, world, x)
    for r, y in enumerate(outs):
        assert y.shape == full.shape
        assert rel_err(y, full) <= 1e-6, f"rank {r}"
    assert rel_err(outs[0], ko.forward(ko.load(wide_mlp), x)) <= 1e-5


def test_sharded_chunked_and_repeated(wide_mlp):
    """Workspace chunking runs one all-gather per chunk and step, in the same order on every rank."""
    from kernix_b200 import Model
    x = np.random.default_rng(3).uniform(-1, 1, (300, 512)).astype(F32)
    full = Model(wide_mlp)(x)
    tg = ThreadGather(2)
    models = [Model(wide_mlp, workspace_mb=1, shard=(r, 2, tg.fn(r))) for r in range(2)]
    outs = [None, None]

    def work(r):
        outs[r] = [models[r](x), models[r](x[:5])]

    th = [threading.Thread(target=work, args=(r,)) for r in range(2)]
    [t.start() for t in th]
    [t.join(timeout=300) for t in th]
    for r in range(2):
        # the 1 MB workspace cuts the 300 rows into chunks of <= 128, whose sharded K = 2048 / 3072 layers split K over
        # the idle SMs (partial sums added in range order) where the whole batch runs CTA-pair tiles, and five rows
        # run the skinny (CUDA-core fp32) dense path: every form within 1e-5 of the exact product, so they agree to
        # ~1e-5
        assert rel_err(outs[r][0], full) <= 1e-5 and rel_err(outs[r][1], full[:5]) <= 1.5e-5
        models[r].close()


def test_sharded_bad_arguments(wide_mlp):
    from kernix_b200 import kernix
    L = kernix.lib()
    assert not L.kernix_model_load_sharded(wide_mlp.encode(), 2, 2, None, None)  # rank out of range
    assert not L.kernix_model_load_sharded(wide_mlp.encode(), 0, 2, None, None)  # no all-gather


def test_c5_two_gpus_nccl(model_dir):
    """c5 (8192-16384-16384-8192) split over two GPUs with NCCL: both ranks equal the unsharded forward."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, KERNIX_MODEL_DIR=model_dir, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(ROOT, "tests", "shard_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("SHARD_OK") == 2, r.stdout[-3000:]
