"""GPU parity: nBody step against the reference kernel's golden output and the oracle restatement."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def _rel(a, b):
    return np.max(np.abs(a - b)) / np.max(np.abs(b))


def test_nbody_reference_golden(cuda):
    """alpaka3's UpdateVelocitiesKernel + UpdatePositions at its built-in EPS=4, 512 bodies, 3 steps."""
    from alpaka3_b200 import algo
    g = np.load(os.path.join(GOLDEN, "nbody.npz"))
    m = _t(g["m"], cuda)
    x, y, z = (_t(g[k], cuda) for k in ("x0", "y0", "z0"))
    vx, vy, vz = (torch.zeros_like(m) for _ in range(3))
    for _ in range(int(g["steps"])):
        algo.nbody_step(m, x, y, z, vx, vy, vz, float(g["dt"]), float(g["eps"]))
    torch.cuda.synchronize()
    for t, k in ((x, "x"), (y, "y"), (z, "z"), (vx, "vx"), (vy, "vy"), (vz, "vz")):
        assert _rel(t.cpu().numpy(), g[k]) <= 1e-4, k


@pytest.mark.parametrize("n,steps", [(256, 2), (1000, 3), (8192, 2)])
def test_nbody_config_softening_vs_oracle(cuda, port, n, steps):
    """the nBody workload's distributions (unit cube, masses [0.5,1), eps^2 = 1e-3, dt = 1e-3) at reduced N."""
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    m = port.gen_f32(n, 0.5, 1.0, seed=SEED + 1)
    pos = [port.gen_f32(n, 0.0, 1.0, seed=SEED + s) for s in (2, 3, 4)]
    zeros = np.zeros(n, np.float32)
    want = port.nbody_steps(m, *pos, zeros, zeros, zeros, 1e-3, 1e-3, steps)
    M = _t(m, cuda)
    X, Y, Z = (_t(p, cuda) for p in pos)
    V = [torch.zeros_like(M) for _ in range(3)]
    for _ in range(steps):
        algo.nbody_step(M, X, Y, Z, *V, 1e-3, 1e-3)
    torch.cuda.synchronize()
    for t, w in zip((X, Y, Z), want[:3]):
        assert _rel(t.cpu().numpy(), w) <= 1e-4
    for t, w in zip(V, want[3:]):
        assert _rel(t.cpu().numpy(), w) <= 1e-4


def test_nbody_split_i_range_matches_whole(cuda, port):
    """velocity kick for two i-ranges (as two ranks would) equals the kick over all bodies."""
    from alpaka3_b200 import algo
    n = 3000
    m = _t(port.gen_f32(n, 0.5, 1.0, seed=11), cuda)
    x, y, z = (_t(port.gen_f32(n, 0.0, 1.0, seed=s), cuda) for s in (12, 13, 14))
    va = [torch.zeros(n, dtype=torch.float32, device=cuda) for _ in range(3)]
    algo.nbody_update_velocities(m, x, y, z, *va, 1e-3, 1e-3)
    h = 1234
    vb = [torch.zeros(n, dtype=torch.float32, device=cuda) for _ in range(3)]
    algo.nbody_update_velocities(m, x, y, z, *(v[:h] for v in vb), 1e-3, 1e-3, i_begin=0)
    algo.nbody_update_velocities(m, x, y, z, *(v[h:] for v in vb), 1e-3, 1e-3, i_begin=h)
    torch.cuda.synchronize()
    for a, b in zip(va, vb):
        assert torch.equal(a, b)


@pytest.mark.parametrize("slice_len", [40000, 120000])
def test_nbody_large_ragged_i_range_matches_slices(cuda, port, slice_len):
    """A kick over 263181 bodies (ragged: neither a multiple of the j-tile nor of the block's group) equals the kicks
    over slices of 40000 bodies (the few-warps variant of the packed-i kernel) or 120000 bodies (the j-pair kernel):
    every body sums its j-bodies in index order whatever the launch shape, so the bits agree; two kicks in a row
    accumulate the same way."""
    from alpaka3_b200 import algo
    n = 262144 + 1000 + 37
    m = _t(port.gen_f32(n, 0.5, 1.0, seed=31), cuda)
    x, y, z = (_t(port.gen_f32(n, 0.0, 1.0, seed=s), cuda) for s in (32, 33, 34))
    va = [torch.zeros(n, dtype=torch.float32, device=cuda) for _ in range(3)]
    for _ in range(2):
        algo.nbody_update_velocities(m, x, y, z, *va, 1e-3, 1e-3)
    vb = [torch.zeros(n, dtype=torch.float32, device=cuda) for _ in range(3)]
    for _ in range(2):
        for b in range(0, n, slice_len):
            e = min(n, b + slice_len)
            algo.nbody_update_velocities(m, x, y, z, *(v[b:e] for v in vb), 1e-3, 1e-3, i_begin=b)
    torch.cuda.synchronize()
    from alpaka3_b200 import capi
    assert capi.device_error(algo.stream_handle()) == 0  # no hand-over wait gave up
    for a, b in zip(va, vb):
        assert torch.isfinite(a).all()
        assert torch.equal(a, b)


def test_nbody_momentum_conserved(cuda, port):
    """pairwise-antisymmetric kick: sum m_i v_i stays ~0 from rest (a size-independent property)."""
    from alpaka3_b200 import algo
    n = 16384
    m = _t(port.gen_f32(n, 0.5, 1.0, seed=21), cuda)
    x, y, z = (_t(port.gen_f32(n, 0.0, 1.0, seed=s), cuda) for s in (22, 23, 24))
    v = [torch.zeros_like(m) for _ in range(3)]
    algo.nbody_update_velocities(m, x, y, z, *v, 1e-3, 1e-3)
    torch.cuda.synchronize()
    for c in v:
        p = (m.double() * c.double()).sum().item()
        scale = (m.double() * c.double().abs()).sum().item()
        assert abs(p) <= 1e-4 * scale
