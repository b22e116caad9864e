"""CPU, two gloo ranks: the host-side logic of the multi-GPU paths.

  * output-column sharding (kernix_b200.shard, the rule the runtime applies in kernix_model_load_sharded): each
    rank computes its slice of every wide layer with the numpy oracle, the slices are all-gathered in rank-major
    [world][rows][slice] order and re-interleaved, and the result equals the unsharded oracle forward;
  * bench.py's weak-scaling plumbing: per-rank inputs differ, and the timed region is the max over ranks."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mlp(rng, dims):
    return [((rng.standard_normal((dims[i], dims[i + 1])) / np.sqrt(dims[i])).astype(np.float32),
             rng.standard_normal(dims[i + 1]).astype(np.float32)) for i in range(len(dims) - 1)]


def _worker(rank, world, port, out):
    try:
        _work(rank, world, port, out)
    except Exception:  # noqa: BLE001  (reported to the parent, which fails the test with it)
        import traceback
        out.put((rank, {"error": traceback.format_exc()}))


def _work(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from kernix_b200 import shard
    from oracle import knx_oracle as ko
    import bench
    res = {}
    # --- sharded MLP forward, oracle arithmetic per slice
    layers = _mlp(np.random.default_rng(0), [64, 2048, 1024, 10])
    x = np.random.default_rng(1).uniform(-1, 1, (5, 64)).astype(np.float32)
    h = x
    for i, (w, b) in enumerate(layers):
        act = 0 if i < len(layers) - 1 else ko.ACT_NONE
        sl = shard.column_slice(w.shape[1], rank, world)
        if sl is None:
            h = ko.dense(h, w, b, act, 0.0)
            continue
        c0, n = sl
        local = np.ascontiguousarray(ko.dense(h, np.ascontiguousarray(w[:, c0:c0 + n]), b[c0:c0 + n], act, 0.0))
        gathered = [torch.empty(local.size) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(local.ravel()))
        g = torch.cat(gathered).numpy().reshape(world, h.shape[0], n)  # [world][rows][slice]
        h = np.concatenate([g[r] for r in range(world)], axis=1)       # the re-interleave of kx_unshard_cols
    ref = x
    for i, (w, b) in enumerate(layers):
        ref = ko.dense(ref, w, b, 0 if i < len(layers) - 1 else ko.ACT_NONE, 0.0)
    res["shard_equal"] = bool(np.array_equal(h, ref))
    res["sliced"] = [shard.column_slice(w.shape[1], rank, world) for w, _ in layers]
    # --- bench plumbing
    res["batch0"] = float(bench.rank_batch(rank)[0, 0])
    res["max"] = bench.reduce_max(dist, float(rank + 1) * 1.5, "cpu")
    dist.barrier()
    dist.destroy_process_group()
    out.put((rank, res))


def test_two_gloo_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=180) for _ in ps)
    for r in range(2):
        assert "error" not in got[r], got[r].get("error")
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert got[r]["shard_equal"], "sharded forward differs from the whole one"
        assert got[r]["max"] == 3.0
    assert got[0]["sliced"] == [(0, 1024), (0, 512), None] and got[1]["sliced"] == [(1024, 1024), (512, 512), None]
    assert got[0]["batch0"] != got[1]["batch0"]  # every rank runs its own samples
