"""Worker for tests/test_gpu_multi.py, run under torchrun with one rank per GPU (NCCL): the sharded algorithms of
alpaka3_b200.dist on each rank's GPU against the oracle. Rank 0 prints one JSON line with the per-check results."""
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    from alpaka3_b200 import algo, dist as ad
    from oracle.oracle import SEED, Port
    world, rank, local = ad.init(timeout_s=120)
    dev = torch.device("cuda", local)
    port = Port()
    res = {}

    # transformReduce sum of squares, fp32, sharded; fp64 partials + all-reduce
    n = (1 << 24) + 5
    b, e = ad.shard_range(n, rank, world)
    x = torch.empty(e - b, dtype=torch.float32, device=dev)
    algo.random_f32(x, SEED, -1.0, 1.0, start=b)
    got = ad.transform_reduce(0.0, "plus", "square", x).item()
    exact = port.sumsq(port.gen_f32(n, -1.0, 1.0))
    res["sumsq_rel"] = abs(got - exact) / exact

    # the same reduction fused with the all-reduce over mapped peer slots
    group = ad.PeerGroup()
    fused = group.transform_reduce(0.0, "plus", "square", x).item()
    res["sumsq_fused_rel"] = abs(fused - exact) / exact
    res["fused_matches_nccl"] = abs(fused - got) <= 1e-6 * abs(got)
    for _ in range(5):  # consecutive calls reuse the slots through the epoch parity
        again = group.transform_reduce(0.0, "plus", "square", x).item()
    res["fused_repeat_ok"] = again == fused
    xi0 = torch.randint(-1000, 1000, (e - b,), dtype=torch.int32, device=dev)
    mx = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
    torch.distributed.all_gather(mx, xi0.max().reshape(1))
    res["fused_max_ok"] = group.transform_reduce(None, "max", "identity", xi0).item() == max(m.item() for m in mx)
    # scan carried through the peer slots (no NCCL)
    xs0 = torch.empty(e - b, dtype=torch.int32, device=dev)
    algo.random_u32(xs0, SEED, start=b, shift=1)  # large values: the carry wraps int32
    ys0 = torch.empty_like(xs0)
    for _ in range(3):
        group.scan(False, ys0, xs0)
    want0 = port.scan(port.gen_u32(n, shift=1), False)[b:e]
    res["peer_scan_ok"] = bool((ys0.cpu().numpy().view(np.uint32) == want0).all())
    torch.cuda.synchronize()
    group.close()

    # dot fp64 and int32 min/max
    a = torch.rand(e - b, dtype=torch.float64, device=dev)
    c = torch.rand(e - b, dtype=torch.float64, device=dev)
    d = ad.transform_reduce(0.0, "plus", "product", a, c).item()
    parts = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
    torch.distributed.all_gather(parts, (a * c).sum().reshape(1))
    res["dot_rel"] = abs(d - sum(p.item() for p in parts)) / abs(sum(p.item() for p in parts))
    xi = torch.randint(-1000, 1000, (e - b,), dtype=torch.int32, device=dev)
    mins = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
    torch.distributed.all_gather(mins, xi.min().reshape(1))
    res["min_ok"] = ad.transform_reduce(None, "min", "identity", xi).item() == min(m.item() for m in mins)

    # exclusive scan int32 [0,16) and inclusive scan uint64, bit-exact against the global oracle scan
    xs = torch.empty(e - b, dtype=torch.int32, device=dev)
    algo.random_u32(xs, SEED, start=b, shift=28)
    ys = torch.empty_like(xs)
    ad.exclusive_scan(ys, xs)
    want = port.scan(port.gen_u32(n, shift=28), False)[b:e]
    res["scan_i32_ok"] = bool((ys.cpu().numpy().view(np.uint32) == want).all())
    n64 = (1 << 22) + 3
    b6, e6 = ad.shard_range(n64, rank, world)
    xu = torch.empty(e6 - b6, dtype=torch.int64, device=dev)
    algo.random_u64(xu, SEED, start=b6)
    yu = torch.empty_like(xu)
    ad.inclusive_scan(yu, xu)
    want64 = port.scan(port.gen_u64(n64), True)[b6:e6]
    res["scan_u64_ok"] = bool((yu.cpu().numpy().view(np.uint64) == want64).all())

    # nBody: 4096 bodies split across ranks, 3 steps, against the oracle (eps^2 = 1e-3)
    nb = 4096
    m = port.gen_f32(nb, 0.5, 1.0, seed=SEED + 1)
    pos = [port.gen_f32(nb, 0.0, 1.0, seed=SEED + s) for s in (2, 3, 4)]
    zeros = np.zeros(nb, np.float32)
    wantb = port.nbody_steps(m, *pos, zeros, zeros, zeros, 1e-3, 1e-3, 3)
    bb, eb = ad.shard_range(nb, rank, world)
    T = [torch.from_numpy(t).to(dev) for t in (m, *pos)]
    V = [torch.zeros(eb - bb, dtype=torch.float32, device=dev) for _ in range(3)]
    sim = ad.NBody(T[0], T[1], T[2], T[3], *V, bb)
    for _ in range(3):
        sim.step(1e-3, 1e-3)
    torch.cuda.synchronize()
    res["nbody_rel"] = max(float(np.max(np.abs(T[k + 1].cpu().numpy() - wantb[k]))) / float(np.max(np.abs(wantb[k])))
                           for k in range(3))

    # heat: row slabs, bit-exact against the oracle, through the fused halo exchange (mailboxes over NVLink) and
    # through NCCL send/recv: 256 x 256 (two bands per slab) and 1000 x 1000 (eight bands per slab, a ragged last band)
    for nh, steps in ((256, 9), (1000, 7)):
        dx = 1.0 / (nh + 1)
        r = 0.2
        u0 = port.heat_init(nh, dx, dx)
        wanth = port.heat_steps(u0, nh, r, r, steps)
        hb, he = ad.shard_range(nh, rank, world)
        for collective in ("fused", "nccl"):
            cur = torch.from_numpy(u0[hb:he + 2].copy()).to(dev)
            nxt = cur.clone()
            slab = ad.HeatSlab(cur, nxt, r, r, collective=collective)
            for _ in range(steps):
                slab.step()
            slab.close()
            torch.cuda.synchronize()
            ok = bool((slab.cur[1:he - hb + 1].cpu().numpy() == wanth[hb + 1:he + 1]).all())
            key = "heat_ok" if collective == "fused" else "heat_nccl_ok"
            res[key] = res.get(key, True) and ok

    allres = [None] * world
    torch.distributed.all_gather_object(allres, res)
    if rank == 0:
        print(json.dumps({"world": world, "ranks": allres}), flush=True)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
