"""CPU: the host-side logic of the sharded algorithms (alpaka3_b200.dist) with world_size 2 over gloo.

Local compute uses the oracle; what is under test is the decomposition (shard ranges, carries, halo rows, gathers).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn_name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        res = globals()[fn_name](rank, world)
        q.put((rank, "ok", res))
    except Exception as e:  # noqa: BLE001 - reported to the parent test
        import traceback
        q.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(fn_name):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, fn_name, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(WORLD):
        rank, status, res = q.get(timeout=120)
        assert status == "ok", res
        out[rank] = res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


# ------------------------------------------------------------------------------------------------ workers
def _scan_worker(rank, world):
    from alpaka3_b200 import dist as ad
    from oracle.oracle import Port
    port = Port()
    n = 100003
    x = port.gen_u32(n, shift=1).view(np.int32)  # large values: the global sum wraps int32
    b, e = ad.shard_range(n, rank, world)
    local = x[b:e]
    total = torch.tensor([int(local.astype(np.int64).sum())], dtype=torch.int64)
    carry, grand = ad.scan_carry(total)
    c32 = ad.carry_to_dtype(carry, torch.int32).item()
    mine = (port.scan(local, False).astype(np.int64) + c32).astype(np.int64)
    want = port.scan(x, False)[b:e]
    return bool(((mine & 0xFFFFFFFF) == (want.astype(np.int64) & 0xFFFFFFFF)).all()), int(grand.item())


def _allreduce_worker(rank, world):
    from alpaka3_b200 import dist as ad
    vals = {"plus": torch.tensor([1.5 + rank], dtype=torch.float64), "min": torch.tensor([10 - rank], dtype=torch.int64),
            "max": torch.tensor([10 + rank], dtype=torch.int64)}
    return {op: ad.allreduce_partial(t, op).item() for op, t in vals.items()}


def _heat_worker(rank, world):
    from alpaka3_b200 import dist as ad
    from oracle.oracle import Port
    port = Port()
    n = 64
    dx = 1.0 / (n + 1)
    r = 0.2
    full0 = port.heat_init(n, dx, dx)
    b, e = ad.shard_range(n, rank, world)  # interior rows [b, e) -> storage rows b+1 .. e
    rows = e - b
    slab = full0[b:e + 2].copy()            # ghost row above (storage b) and below (storage e+1)
    cur = slab.copy()
    for _ in range(5):
        # local step over the slab (the oracle steps a square grid), in the reference's operation order
        k = 1.0 - 2.0 * r - 2.0 * r
        nxt = cur.copy()
        for i in range(1, rows + 1):
            nxt[i, 1:-1] = cur[i, 1:-1] * k + cur[i, :-2] * r + cur[i, 2:] * r + cur[i - 1, 1:-1] * r + cur[i + 1, 1:-1] * r
        t = torch.from_numpy(nxt)
        ad.heat_exchange_halos(t, rank, world)
        cur = t.numpy()
    want = port.heat_steps(full0, n, r, r, 5)[b + 1:e + 1]
    return bool((cur[1:rows + 1] == want).all())


def _gather_worker(rank, world):
    from alpaka3_b200 import dist as ad
    n = 12
    full = torch.zeros(n, dtype=torch.float32)
    local = torch.arange(rank * (n // world), (rank + 1) * (n // world), dtype=torch.float32)
    ad.nbody_allgather(full, local)
    return full.tolist()


# ------------------------------------------------------------------------------------------------ tests
def test_shard_range_covers_exactly():
    from alpaka3_b200 import dist as ad
    for n in (0, 1, 7, 8, 1 << 20, (1 << 30) + 3):
        for world in (1, 2, 3, 4, 8):
            parts = [ad.shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [e - b for b, e in parts]
            assert max(sizes) - min(sizes) <= 1


def test_scan_carry_two_ranks():
    out = _run("_scan_worker")
    assert out[0][0] and out[1][0]
    assert out[0][1] == out[1][1]


def test_allreduce_partials_two_ranks():
    out = _run("_allreduce_worker")
    for r in range(WORLD):
        assert out[r] == {"plus": 1.5 + 2.5, "min": 9, "max": 11}


def test_heat_halo_exchange_two_ranks():
    out = _run("_heat_worker")
    assert out[0] and out[1]


def test_nbody_allgather_two_ranks():
    out = _run("_gather_worker")
    assert out[0] == out[1] == [float(i) for i in range(12)]
