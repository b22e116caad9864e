"""torchrun worker of tests/test_gpu_shard.py: c5 split by output columns over the ranks, once with the runtime's
own NCCL all-gather (kernix_model_load_sharded_nccl: the id made on rank 0, shared through torch.distributed) and
once through the torch.distributed callback; every rank compares both with the unsharded model on its own GPU
(and the two sharded results with each other, bit for bit) and prints SHARD_OK."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from kernix_b200 import Model, configs, shard
    if rank == 0:
        configs.model_path("c5")  # written once (2.1 GB), then read by every rank
    dist.barrier()
    path = configs.model_path("c5")
    os.environ["KERNIX_DEVICE"] = str(local)
    x = configs.inputs("c5", 24)
    m_nccl = Model(path, shard=(rank, world, shard.share_nccl_id()))
    ys_nccl = m_nccl(x)
    ys_nccl2 = m_nccl(x[:5])  # a second call over the same communicator, a different row count
    x3 = configs.inputs("c5", 300, seed=7)  # more than 128 rows: the CTA-pair tiles, no K split
    ys_nccl3 = m_nccl(x3)
    m_nccl.close()
    ys_cb = Model(path, shard=(rank, world, shard.torch_allgather()))(x)
    y1 = Model(path)(x)
    err = float(np.abs(ys_nccl - y1).max() / np.abs(y1).max())
    err2 = float(np.abs(ys_nccl2 - y1[:5]).max() / np.abs(y1).max())
    m1 = Model(path)
    y3 = m1(x3)
    m1.close()
    err3 = float(np.abs(ys_nccl3 - y3).max() / np.abs(y3).max())
    same = np.array_equal(ys_nccl, ys_cb)
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: max rel diff sharded (C NCCL) vs whole {err:.2e}, 5 rows {err2:.2e}, 300 rows {err3:.2e}, "
          f"C NCCL == callback: {same}")
    if err <= 1e-6 and err2 <= 1.5e-5 and err3 <= 1e-5 and same:
        print("SHARD_OK")


if __name__ == "__main__":
    main()
