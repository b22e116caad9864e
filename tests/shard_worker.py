"""torchrun worker of tests/test_gpu_shard.py: c5 split by output columns over the ranks (NCCL all-gather);
every rank compares its output with the unsharded model on its own GPU and prints SHARD_OK."""
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
    ys = Model(path, shard=(rank, world, shard.torch_allgather()))(x)
    y1 = Model(path)(x)
    err = float(np.abs(ys - y1).max() / np.abs(y1).max())
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: max rel diff sharded vs whole {err:.2e}")
    if err <= 1e-6:
        print("SHARD_OK")


if __name__ == "__main__":
    main()
