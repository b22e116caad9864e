"""Output-column sharding of wide dense layers across the GPUs of one node (one process per GPU).

The runtime (kernix_model_load_sharded, include/kernix_cuda.h) keeps, on rank r of W, output columns
[out * r / W, out * (r + 1) / W) of every fp32 LINEAR step with at least KERNIX_SHARD_MIN_COLS outputs
(divisible by W), computes that slice, and calls an all-gather supplied by the host; every rank then
re-interleaves the gathered [W][rows][out / W] block into full rows and runs the next step whole.

    import torch.distributed as dist
    from kernix_b200 import Model, shard
    dist.init_process_group("nccl")                      # torchrun, one process per GPU
    uid = shard.share_nccl_id()                          # rank 0 makes an NCCL id, every rank receives it
    m = Model(path, shard=(dist.get_rank(), dist.get_world_size(), uid))   # the runtime all-gathers with NCCL
    y = m(x)                                             # every rank gets the full output

A host callback instead of the id (shard.torch_allgather()) routes each all-gather through torch.distributed.

This is the multi-GPU form of the reference's per-call row split of one sgemm between two devices
(src/kernix_metal.m:161-265): a layer too narrow in batch to split by samples is split by output columns, with
one collective per layer over NVLink.
"""

SHARD_MIN_COLS = 1024  # KERNIX_SHARD_MIN_COLS


def column_slice(out, rank, world):
    """(first column, width) of rank's slice of a sharded layer with `out` outputs, or None if it runs whole."""
    if world <= 1 or out < SHARD_MIN_COLS or out % world:
        return None
    n = out // world
    return n * rank, n


class _DevArray:
    """Zero-copy view of device floats for torch.as_tensor (CUDA array interface)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "stream": None}


def torch_allgather(group=None):
    """An all-gather for Model(shard=...) backed by torch.distributed (NCCL on GPUs): the collective is ordered on
    the runtime's stream, so it runs after the slice's GEMM and before the re-interleave kernel."""
    import torch
    import torch.distributed as dist

    def gather(send, recv, count, stream):
        world = dist.get_world_size(group)
        dev = torch.device("cuda", torch.cuda.current_device())
        src = torch.as_tensor(_DevArray(send, count), device=dev)
        dst = torch.as_tensor(_DevArray(recv, count * world), device=dev)
        with torch.cuda.stream(torch.cuda.ExternalStream(stream, device=dev)):
            dist.all_gather_into_tensor(dst, src, group=group)

    return gather


def nccl_unique_id():
    """A new 128-byte NCCL unique id (kernix_nccl_unique_id): make it on one rank and give it to all."""
    import ctypes

    from .kernix import lib
    buf = ctypes.create_string_buffer(128)
    if lib().kernix_nccl_unique_id(buf) != 0:
        raise RuntimeError("NCCL is not available")
    return buf.raw


def share_nccl_id(group=None):
    """nccl_unique_id() made on rank 0 of the torch.distributed group and broadcast to every rank (bytes)."""
    import torch
    import torch.distributed as dist
    obj = [nccl_unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]
