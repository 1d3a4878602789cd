"""GPU: the benchmark configurations at full size, checked through size-independent properties and sampled oracles
(the CPU oracle cannot replay 2^30-element scans or 262144-body steps quickly)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_sumsq_2e30_fp32(cuda, port):
    """transformReduce sum of squares over 2^30 seeded fp32 values vs the compensated fp64 oracle, rel <= 1e-5."""
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    n = 1 << 30
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    algo.random_f32(x, SEED, -1.0, 1.0)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    algo.transform_reduce(0.0, out, "plus", "square", x)
    got = out.item()
    exact = port.sumsq(x.cpu().numpy())
    assert abs(got - exact) / exact <= 1e-5


def test_exclusive_scan_2e30_int32_properties(cuda):
    """exclusive scan of 2^30 int32 in [0,16): out[0] = 0, out[i+1] - out[i] = in[i] (mod 2^32), last + in[-1] = total."""
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    n = 1 << 30
    x = torch.empty(n, dtype=torch.int32, device=cuda)
    algo.random_u32(x, SEED, shift=28)
    y = torch.empty_like(x)
    algo.exclusive_scan(y, x)
    assert y[0].item() == 0
    d = (y[1:] - y[:-1]).view(torch.int32)  # int32 arithmetic wraps like the unsigned scan
    assert torch.equal(d, x[:-1])
    tot = torch.empty(1, dtype=torch.int32, device=cuda)
    algo.reduce(0, tot, "plus", x)
    assert (y[-1] + x[-1]).item() == tot.item()


def test_inclusive_scan_2e28_uint64_properties(cuda, port):
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    n = 1 << 28
    x = torch.empty(n, dtype=torch.int64, device=cuda)
    algo.random_u64(x, SEED)
    y = torch.empty_like(x)
    algo.inclusive_scan(y, x)
    assert y[0].item() == x[0].item()
    assert torch.equal(y[1:] - y[:-1], x[1:])  # int64 wrap == uint64 wrap
    # the first 2^20 against the oracle
    k = 1 << 20
    assert (y[:k].cpu().numpy().view(np.uint64) == port.scan(port.gen_u64(k), True)).all()


def test_heat_32768_eigenmode(cuda):
    """32768^2 interior, 30 steps: the sin*sin field decays by lambda per step (discrete eigenmode), normwise 1e-12."""
    from alpaka3_b200 import algo
    n = 32768
    dx = 1.0 / (n + 1)
    r = 0.2
    u = torch.empty((n + 2, n + 2), dtype=torch.float64, device=cuda)
    algo.heat_init(u, dx, dx)
    v = u.clone()
    steps = 30
    lam = 1.0 - 4.0 * r * (1.0 - np.cos(np.pi * dx))
    ref_row = u[n // 3].clone()
    for _ in range(steps):
        algo.heat_step(u, v, r, r)
        u, v = v, u
    torch.cuda.synchronize()
    # compare a band of rows against lambda^steps * u0 (u0 rows are regenerated: v holds step steps-1)
    u0 = torch.empty_like(v)
    algo.heat_init(u0, dx, dx)
    err = 0.0
    for r0 in (1, n // 3, n // 2, n - 1):
        want = u0[r0] * lam ** steps
        err = max(err, (u[r0] - want).abs().max().item() / u0.abs().max().item())
    assert err <= 1e-12
    assert torch.equal(u0[n // 3], ref_row)


def test_nbody_262144_sampled(cuda, port):
    """One step of 262144 bodies: accelerations of 512 sampled bodies against an fp64 all-pairs sum (rel 1e-4
    normwise), and total momentum stays ~0 from rest."""
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    n = 262144
    m = port.gen_f32(n, 0.5, 1.0, seed=SEED + 1)
    pos = [port.gen_f32(n, 0.0, 1.0, seed=SEED + s) for s in (2, 3, 4)]
    M = torch.from_numpy(m).to(cuda)
    X, Y, Z = (torch.from_numpy(p).to(cuda) for p in pos)
    V = [torch.zeros(n, dtype=torch.float32, device=cuda) for _ in range(3)]
    dt = 1e-3
    algo.nbody_update_velocities(M, X, Y, Z, *V, dt, 1e-3)
    torch.cuda.synchronize()
    idx = np.random.default_rng(3).choice(n, 512, replace=False)
    acc = port.nbody_accel_sample(m, *pos, 1e-3, idx)
    got = np.stack([V[k].cpu().numpy()[idx] / dt for k in range(3)], axis=1)
    assert np.max(np.abs(got - acc)) / np.max(np.abs(acc)) <= 1e-4
    for c in V:
        p = (M.double() * c.double()).sum().item()
        scale = (M.double() * c.double().abs()).sum().item()
        assert abs(p) <= 1e-4 * scale


def test_nbody_262144_ten_steps_against_golden(cuda):
    """The nBody workload itself: 262144 bodies (unit cube, masses [0.5, 1), v = 0), eps^2 = 1e-3, dt = 1e-3, ten
    kick + drift steps through the C ABI; final positions within 1e-4 (normwise, max |error| / max |position| per
    component) of the oracle's trajectory (tests/golden/nbody_262144.npz; the oracle follows the reference kernel's
    operation order, pinned bit-exact to it by nbody.npz). The configuration collapses violently (peak speed ~7200,
    positions spread to ~65), which makes it sensitive to the order of the j sums."""
    import os

    import numpy as np
    from alpaka3_b200 import algo
    from conftest import GOLDEN
    from oracle.oracle import SEED
    g = np.load(os.path.join(GOLDEN, "nbody_262144.npz"))
    n, steps, dt, eps = int(g["n"]), int(g["steps"]), float(g["dt"]), float(g["eps"])
    m = torch.empty(n, dtype=torch.float32, device=cuda)
    algo.random_f32(m, SEED + 1, 0.5, 1.0)
    pos = [torch.empty(n, dtype=torch.float32, device=cuda) for _ in range(3)]
    for k, t in enumerate(pos):
        algo.random_f32(t, SEED + 2 + k, 0.0, 1.0)
    v = [torch.zeros(n, dtype=torch.float32, device=cuda) for _ in range(3)]
    for _ in range(steps):
        algo.nbody_step(m, *pos, *v, dt, eps)
    torch.cuda.synchronize()
    for t, key in zip(pos, "xyz"):
        want = g[key]
        got = t.cpu().numpy()
        rel = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
        assert rel <= 1e-4, (key, rel)
