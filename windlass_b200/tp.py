"""Host plumbing of tensor parallelism with one process per GPU (the layout torchrun gives).

The model itself splits and reduces inside libwindlass_cuda (wl_options.tp_size / tp_rank / tp_id, NCCL over NVLink).
What the processes have to do on the host is small, and it is here:

- agree on one group id: rank 0 makes it (wl_tp_unique_id) and the others receive it over any torch.distributed
  process group (gloo is enough; no device collective is involved);
- open the same model with the same options on every rank, then make the same calls with the same arguments;
- combine per-rank timings as the maximum over ranks.

The reference has no counterpart: it runs on one CPU (src/Transformer.cs:496-501 is its only parallelism).
"""
import os


def env_ranks():
    """(rank, world size, local rank) from the torchrun environment; (0, 1, 0) outside it."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def share_group_id(dist, make_id=None):
    """Rank 0's fresh group id, broadcast to every rank of the default process group; returns the 128 bytes."""
    if make_id is None:
        from ._lib import tp_unique_id as make_id
    obj = [make_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    gid = obj[0]
    if not isinstance(gid, (bytes, bytearray)) or len(gid) != 128:
        raise ValueError("the tensor-parallel group id must be 128 bytes")
    return bytes(gid)


def max_over_ranks(dist, value):
    """The largest of every rank's float `value` (host all-reduce; every rank gets it)."""
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64)
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def open_group_model(dist, device, make_id=None, **kw):
    """CudaTransformer of this rank's share of a tensor-parallel model over every rank of `dist`'s default group
    (one GPU per rank, `device` this rank's). Keyword arguments go to CudaTransformer and must be equal on every
    rank."""
    from .transformer import CudaTransformer
    world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
    if world == 1:
        return CudaTransformer(device=device, **kw)
    gid = share_group_id(dist, make_id)
    return CudaTransformer(device=device, tp_size=world, tp_rank=dist.get_rank(), tp_id=gid, **kw)
