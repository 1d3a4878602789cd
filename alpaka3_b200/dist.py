"""Sharding of the primitive path over one process per GPU (torch.distributed over NCCL; gloo for CPU tests).

alpaka3 itself has no multi-device layer; these are the exchange steps the sharded algorithms need, each on the
smallest data that has to move:

* :func:`shard_range`              contiguous 1/world block of a global index range (remainder to the first ranks)
* :func:`allreduce_partial`        reduce/dot/transformReduce: one 8-byte partial per rank, NCCL all-reduce, then the
                                   final rounding to the output dtype (same op order on every rank)
* :func:`scan_carry`               scan: all-gather of the per-rank totals, carry = sum of the totals of lower ranks
* :func:`nbody_allgather`          nBody: all-gather of the x/y/z shards into the full position arrays
* :func:`heat_exchange_halos`      heat: one boundary row to each neighbour (send/recv), into the neighbour's ghost row
* :class:`HeatSlab`                heat time steps on row slabs: fused stencil + halo exchange over NVLink (HaloMailbox)
                                   or stencil + NCCL send/recv

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
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(gathered, total)
    else:
        dist.all_gather(list(gathered.chunk(world)), total)
    if rank == 0:
        carry = torch.zeros_like(total)
    else:
        carry = gathered[:rank].sum(dtype=gathered.dtype).reshape(1).to(total.dtype)
    return carry, gathered.sum(dtype=gathered.dtype).reshape(1).to(total.dtype)


def nbody_allgather(full, local):
    """Gather every rank's equal-size shard `local` into `full` (rank-major)."""
    if dist.is_initialized() and dist.get_world_size() > 1:
        if dist.get_backend() == "nccl":
            dist.all_gather_into_tensor(full, local)
        else:
            dist.all_gather(list(full.chunk(dist.get_world_size())), local)
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


# ------------------------------------------------------------------------------------- sharded algorithms (GPU)
def _world():
    if dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def transform_reduce(neutral, reduce_fn, transform_fn, in0_local, in1_local=None, out=None):
    """onHost::transformReduce over data sharded across ranks: one kernel per rank (unrounded 8-byte partial), one
    all-reduce of the partials, final rounding to the input dtype. Returns a 1-element tensor on every rank."""
    from . import algo
    partial = algo.transform_reduce_partial(reduce_fn, transform_fn, in0_local, in1_local, neutral=neutral)
    allreduce_partial(partial, reduce_fn)
    res = partial.to(in0_local.dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res


def carry_to_dtype(carry, dtype):
    """Converts a carry computed as an 8-byte partial (float64, or int64 bits for integers) to the scan's element
    type; integer carries keep their low bits (two's-complement wrap, as the single-device scan)."""
    if dtype.is_floating_point:
        return carry.to(dtype)
    c = carry.view(torch.int64)
    if torch.empty(0, dtype=dtype).element_size() == 4:
        return (c & 0xFFFFFFFF).to(torch.int32).view(dtype)
    return c.view(dtype)


def _scan_sharded(inclusive, out_local, data_local):
    from . import algo
    world, rank = _world()
    carry = None
    if world > 1:
        total = algo.transform_reduce_partial("plus", "identity", data_local, neutral=0)
        if not data_local.dtype.is_floating_point:
            total = total.view(torch.int64)  # sums of integer shards wrap; int64 bits carry them exactly
        c, _ = scan_carry(total)
        carry = carry_to_dtype(c, data_local.dtype)
    return algo._scan(inclusive, out_local, data_local, None, carry)


def exclusive_scan(out_local, data_local):
    """Exclusive scan of a contiguously sharded array (rank r holds elements [begin_r, end_r)): shard total, all-gather
    of the totals, scan seeded with the sum of the lower ranks' totals (3N/G traffic per GPU)."""
    return _scan_sharded(False, out_local, data_local)


def inclusive_scan(out_local, data_local):
    return _scan_sharded(True, out_local, data_local)


class NBody:
    """All-pairs nBody with the bodies split across ranks: every rank keeps all positions (m, x, y, z of n bodies) and
    the velocities of its own bodies; a step is the local kick + drift followed by an all-gather of the positions."""

    def __init__(self, m, x, y, z, vx_local, vy_local, vz_local, i_begin):
        self.m, self.x, self.y, self.z = m, x, y, z
        self.v = (vx_local, vy_local, vz_local)
        self.i_begin = i_begin
        self.count = vx_local.numel()
        self.stage = [torch.empty(self.count, dtype=x.dtype, device=x.device) for _ in range(3)]

    def step(self, dt, eps):
        from . import algo
        algo.nbody_step(self.m, self.x, self.y, self.z, *self.v, dt, eps, i_begin=self.i_begin)
        world, _ = _world()
        if world > 1:
            b, e = self.i_begin, self.i_begin + self.count
            for full, st in zip((self.x, self.y, self.z), self.stage):
                st.copy_(full[b:e])
                nbody_allgather(full, st)


class HaloMailbox:
    """Halo mailbox of this rank (a3b_halo): a small device buffer that the neighbouring ranks map through CUDA IPC.
    The fused heat step stores its boundary rows straight into the neighbours' mailboxes over NVLink and reads its
    ghost rows from its own, with per-step flags instead of NCCL send/recv."""

    def __init__(self, cols):
        import ctypes
        from . import capi
        self.world, self.rank = _world()
        L = capi.lib()
        handle = (ctypes.c_char * L.a3b_ipc_handle_size())()
        self.h = ctypes.c_void_p()
        capi.call("a3b_halo_create", self.world, self.rank, cols, ctypes.byref(self.h), handle)
        mine = bytes(handle)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, mine)
        else:
            handles = [mine]
        blob = b"".join(handles)
        capi.call("a3b_halo_connect", self.h, (ctypes.c_char * len(blob)).from_buffer_copy(blob))
        if self.world > 1:
            dist.barrier()

    def close(self):
        from . import capi
        if self.h:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier()  # no neighbour writes into this mailbox any more
            capi.call("a3b_halo_destroy", self.h)
            self.h = None


class HeatSlab:
    """Row slab of the heat grid on one rank: `rows` interior rows (global rows row_offset+1 ... row_offset+rows) and
    one ghost row above and below.

    collective="fused" (default on several ranks): one kernel per step; its two boundary bands run first, wait for the
    neighbours' boundary rows of the previous step in this rank's halo mailbox, and store their own boundary rows into
    the neighbours' mailboxes over NVLink (a3b_heat_step_halo). The interior bands never wait.
    collective="nccl": the two boundary rows are updated first, sent to the neighbours with NCCL send/recv while the
    interior rows are updated, and the receives are waited for before the next step."""

    def __init__(self, cur, nxt, rX, rY, collective="fused"):
        self.cur, self.nxt, self.rX, self.rY = cur, nxt, rX, rY
        self.rows = cur.shape[0] - 2
        self.cols = cur.shape[1] - 2
        self.pending = []
        self.halo = None
        world, _ = _world()
        if world > 1 and collective == "fused":
            from . import algo, capi
            self.halo = HaloMailbox(self.cols)
            capi.call("a3b_heat_halo_publish", algo.stream_handle(), self.halo.h, algo._ptr(cur), self.rows, self.cols,
                      cur.stride(0))

    def step(self):
        from . import algo, capi
        if self.halo is not None:
            capi.call("a3b_heat_step_halo", algo.stream_handle(), self.halo.h, algo._ptr(self.cur),
                      algo._ptr(self.nxt), self.rows, self.cols, self.cur.stride(0), self.rX, self.rY)
            self.cur, self.nxt = self.nxt, self.cur
            return
        for r in self.pending:
            r.wait()
        self.pending = []
        world, rank = _world()
        rows = self.rows
        if world == 1 or rows < 3:
            algo.heat_step(self.cur, self.nxt, self.rX, self.rY)
            if world > 1:
                heat_exchange_halos(self.nxt, rank, world)
        else:
            algo.heat_step(self.cur, self.nxt, self.rX, self.rY, row_begin=1, row_end=2)
            algo.heat_step(self.cur, self.nxt, self.rX, self.rY, row_begin=rows, row_end=rows + 1)
            ops = []
            if rank > 0:
                ops.append(dist.P2POp(dist.isend, self.nxt[1], rank - 1))
                ops.append(dist.P2POp(dist.irecv, self.nxt[0], rank - 1))
            if rank < world - 1:
                ops.append(dist.P2POp(dist.isend, self.nxt[rows], rank + 1))
                ops.append(dist.P2POp(dist.irecv, self.nxt[rows + 1], rank + 1))
            self.pending = dist.batch_isend_irecv(ops)
            algo.heat_step(self.cur, self.nxt, self.rX, self.rY, row_begin=2, row_end=rows)
        self.cur, self.nxt = self.nxt, self.cur

    def finish(self):
        for r in self.pending:
            r.wait()
        self.pending = []

    def close(self):
        self.finish()
        if self.halo is not None:
            self.halo.close()
            self.halo = None


class PeerGroup:
    """The ranks of this node connected through mapped slot buffers (a3b_peer_group): the fused reduce + all-reduce
    stores each rank's partial straight into every peer's memory over NVLink from inside the reduction kernel."""

    def __init__(self):
        import ctypes
        from . import capi
        self.world, self.rank = _world()
        L = capi.lib()
        hsz = L.a3b_ipc_handle_size()
        handle = (ctypes.c_char * hsz)()
        self.g = ctypes.c_void_p()
        capi.call("a3b_peer_group_create", self.world, self.rank, ctypes.byref(self.g), handle)
        mine = bytes(handle)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, mine)
        else:
            handles = [mine]
        blob = b"".join(handles)
        arr = (ctypes.c_char * len(blob)).from_buffer_copy(blob)
        capi.call("a3b_peer_group_connect", self.g, arr)
        if self.world > 1:
            dist.barrier()

    def close(self):
        from . import capi
        if self.g:
            capi.call("a3b_peer_group_destroy", self.g)
            self.g = None

    def transform_reduce(self, neutral, reduce_fn, transform_fn, in0_local, in1_local=None, out=None):
        """Sharded onHost::transformReduce in one launch per rank (fused with the all-reduce); every rank gets the
        same bits. All ranks must make the same sequence of calls."""
        import ctypes
        from . import algo, capi
        code = algo.dtype_code(in0_local)
        if out is None:
            out = torch.empty(1, dtype=in0_local.dtype, device=in0_local.device)
        if neutral is None:
            neutral = algo._neutral(reduce_fn, code)
        keep, p = algo._host_scalar(neutral, code)
        capi.call("a3b_transform_reduce_allranks", algo.stream_handle(), self.g, code, algo.REDUCE[reduce_fn],
                  algo.XFORM[transform_fn], algo._ptr(in0_local), algo._ptr(in1_local), in0_local.numel(), p,
                  algo._ptr(out))
        return out

    def scan(self, inclusive, out_local, data_local, carry=None):
        """Scan of a contiguously sharded array in two launches per rank and no NCCL: the shard total and the
        exclusive carry over lower ranks come from one fused kernel (peer slots), then the carried single-pass scan."""
        from . import algo, capi
        if carry is None:
            carry = torch.empty(1, dtype=data_local.dtype, device=data_local.device)
        capi.call("a3b_reduce_lower_ranks", algo.stream_handle(), self.g, algo.dtype_code(data_local),
                  algo._ptr(data_local), data_local.numel(), algo._ptr(carry))
        return algo._scan(inclusive, out_local, data_local, None, carry)
