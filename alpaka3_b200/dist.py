"""Sharding of the primitive path over one process per GPU (torch.distributed over NCCL; gloo for CPU tests).

alpaka3 itself has no multi-device layer; these are the exchange steps the sharded algorithms need, each on the
smallest data that has to move:

* :func:`shard_range`              contiguous 1/world block of a global index range (remainder to the first ranks)
* :func:`allreduce_partial`        reduce/dot/transformReduce: one 8-byte partial per rank, NCCL all-reduce, then the
                                   final rounding to the output dtype (same op order on every rank)
* :func:`scan_carry`               scan: all-gather of the per-rank totals, carry = sum of the totals of lower ranks
* :func:`nbody_allgather`          nBody: all-gather of the x/y/z shards into the full position arrays
* :func:`heat_exchange_halos`      heat: one boundary row to each neighbour (send/recv), into the neighbour's ghost row

The collectives are written for tensors on the rank's device; with the gloo backend they run on CPU tensors, which
is how the host-side logic is tested without a GPU.
"""
import datetime
import os

import torch
import torch.distributed as dist


def env_world():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(
        os.environ.get("LOCAL_RANK", "0"))


def init(backend=None, timeout_s=120):
    """Initialise the process group from the torchrun environment (no-op for a single process)."""
    world, rank, local = env_world()
    if world == 1:
        return 1, 0, local
    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.get_world_size(), dist.get_rank(), local


def shard_range(n, rank, world):
    """[begin, end) of rank's contiguous share of n items; the first n % world ranks get one extra item."""
    base, rem = divmod(n, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


def allreduce_partial(partial, op="plus"):
    """Combine the per-rank 8-byte partials in place (sum / min / max)."""
    if dist.is_initialized() and dist.get_world_size() > 1:
        rop = {"plus": dist.ReduceOp.SUM, "min": dist.ReduceOp.MIN, "max": dist.ReduceOp.MAX}[op]
        dist.all_reduce(partial, op=rop)
    return partial


def scan_carry(total, rank=None, world=None):
    """total: 1-element tensor with this rank's shard sum. Returns (carry for this rank, grand total), both 1-element
    tensors of total's dtype; integer sums wrap like the single-device scan."""
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        return torch.zeros_like(total), total.clone()
    world = dist.get_world_size()
    rank = dist.get_rank()
    gathered = torch.empty(world, dtype=total.dtype, device=total.device)
    dist.all_gather_into_tensor(gathered, total)
    if rank == 0:
        carry = torch.zeros_like(total)
    else:
        carry = gathered[:rank].sum(dtype=gathered.dtype).reshape(1).to(total.dtype)
    return carry, gathered.sum(dtype=gathered.dtype).reshape(1).to(total.dtype)


def nbody_allgather(full, local):
    """Gather every rank's equal-size shard `local` into `full` (rank-major)."""
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_gather_into_tensor(full, local)
    else:
        full.copy_(local)
    return full


def heat_exchange_halos(u, rank, world):
    """u: (rows+2, cols+2) local slab with ghost rows 0 and rows+1. Sends row 1 up and row `rows` down, receives the
    neighbours' boundary rows into the ghost rows. Global boundary ghost rows are left untouched (Dirichlet 0)."""
    if world == 1:
        return
    rows = u.shape[0] - 2
    ops = []
    if rank > 0:
        ops.append(dist.P2POp(dist.isend, u[1].contiguous() if not u[1].is_contiguous() else u[1], rank - 1))
        ops.append(dist.P2POp(dist.irecv, u[0], rank - 1))
    if rank < world - 1:
        ops.append(dist.P2POp(dist.isend, u[rows], rank + 1))
        ops.append(dist.P2POp(dist.irecv, u[rows + 1], rank + 1))
    for req in dist.batch_isend_irecv(ops):
        req.wait()
