"""Multi-GPU plumbing of the path: one process per GPU, batch rows sharded across ranks, and the only collective
the path has -- the all-reduce of (loss sum, token count).  Streams are independent (every RunTimeSdm.forward
starts from an empty memory, track4_onesdm_models.py:249-258), so the mixer itself needs no communication.
"""
import datetime
import os

import torch
import torch.distributed as dist


def shard_rows(total_rows, rank, world):
    """Contiguous [start, stop) of the batch rows owned by `rank` (sizes differ by at most one)."""
    base, extra = divmod(total_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def init(backend=None, timeout_s=120, device=None):
    """init_process_group from the torchrun environment (RANK, WORLD_SIZE, MASTER_ADDR/PORT) with a short
    timeout, so a rank that waits for a peer that died ends with an error instead of hanging."""
    backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist.get_rank(), dist.get_world_size()


def reduce_loss(loss_sum, count, device=None):
    """Sum (loss, count) over all ranks in float64; returns (total loss, total count) as Python floats."""
    dev = device or (loss_sum.device if torch.is_tensor(loss_sum) else torch.device("cpu"))
    buf = torch.zeros(2, dtype=torch.float64, device=dev)
    buf[0] = loss_sum if not torch.is_tensor(loss_sum) else loss_sum.reshape(()).to(torch.float64)
    buf[1] = float(count)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(buf)
    return float(buf[0].item()), float(buf[1].item())


def env_world():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def world_size():
    return dist.get_world_size() if dist.is_initialized() else 1


def all_reduce_(buf):
    """In-place sum of a tensor over all ranks (the per-step (loss sum, token count) exchange); no-op alone."""
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(buf)
    return buf


def barrier():
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def max_over_ranks(x, device=None):
    """The largest of a per-rank float (a timed duration: the job takes as long as its slowest rank)."""
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def finalize():
    """Last barrier, then destroy the process group (after every CUDA graph holding collectives is released)."""
    if dist.is_initialized():
        if dist.get_world_size() > 1:
            dist.barrier()
        dist.destroy_process_group()
