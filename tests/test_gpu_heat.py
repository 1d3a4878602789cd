"""GPU parity: heat stencil bit-exact against the reference StencilKernel (golden) and the oracle."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _steps(algo, u0, r, steps, dev, pitch=None):
    n2 = u0.shape[0]
    if pitch is None:
        cur = torch.from_numpy(u0).to(dev)
        nxt = cur.clone()
    else:
        big = torch.zeros((n2, pitch), dtype=torch.float64, device=dev)
        big2 = big.clone()
        cur, nxt = big[:, :n2], big2[:, :n2]
        cur.copy_(torch.from_numpy(u0))
        nxt.copy_(cur)
    for _ in range(steps):
        algo.heat_step(cur, nxt, r, r)
        cur, nxt = nxt, cur
    torch.cuda.synchronize()
    return cur.cpu().numpy()


def test_heat_reference_golden_bitexact(cuda):
    from alpaka3_b200 import algo
    g = np.load(os.path.join(GOLDEN, "heat.npz"))
    dx, dt = float(g["dx"]), float(g["dt"])
    r = dt / (dx * dx)
    out = _steps(algo, g["u0"], r, int(g["steps"]), cuda)
    assert (out == g["u25"]).all()


@pytest.mark.parametrize("n,pitch", [(64, None), (100, None), (129, None), (255, 300), (1000, None), (33, 41)])
def test_heat_vs_oracle_bitexact(cuda, port, n, pitch):
    from alpaka3_b200 import algo
    dx = 1.0 / (n + 1)
    dt = 0.2 * dx * dx
    r = dt / (dx * dx)
    u0 = port.heat_init(n, dx, dx)
    out = _steps(algo, u0, r, 7, cuda, pitch)
    assert (out == port.heat_steps(u0, n, r, r, 7)).all()


def test_heat_row_ranges_compose(cuda, port):
    """boundary rows first, then the interior (the overlap order of the multi-GPU step) == one full step."""
    from alpaka3_b200 import algo
    n = 200
    dx = 1.0 / (n + 1)
    r = 0.2
    u0 = port.heat_init(n, dx, dx)
    cur = torch.from_numpy(u0).to(cuda)
    a, b = cur.clone(), cur.clone()
    algo.heat_step(cur, a, r, r)
    algo.heat_step(cur, b, r, r, row_begin=1, row_end=2)
    algo.heat_step(cur, b, r, r, row_begin=n, row_end=n + 1)
    algo.heat_step(cur, b, r, r, row_begin=2, row_end=n)
    assert torch.equal(a, b)


def test_heat_eigenmode_decay(cuda):
    """sin*sin is a discrete eigenmode of the 5-point operator with zero Dirichlet walls: after s steps the field is
    lambda^s * u0, lambda = 1 - 4r(1 - cos(pi dx)) per axis pair -- a size-independent check used at full size."""
    from alpaka3_b200 import algo
    n = 2048
    dx = 1.0 / (n + 1)
    r = 0.2
    u = torch.empty((n + 2, n + 2), dtype=torch.float64, device=cuda)
    algo.heat_init(u, dx, dx)
    u0 = u.clone()
    v = torch.empty_like(u)
    v.copy_(u)
    steps = 50
    for _ in range(steps):
        algo.heat_step(u, v, r, r)
        u, v = v, u
    lam = 1.0 - 4.0 * r * (1.0 - np.cos(np.pi * dx))
    want = u0 * lam ** steps
    err = (u - want).abs().max().item() / want.abs().max().item()
    assert err <= 1e-12


def test_heat_example_problem_reference_golden(cuda):
    """The heatEquation2D example end to end at its defaults (64 x 64, 4000 steps, tMax 0.1): exact initial field and
    time-dependent Dirichlet ring (BoundaryKernel). Against the reference's own output (normwise 1e-12: the ring values
    come from the device's exp/sin instead of the host's) and the example's own analytical check
    (max error < 1e-4, example/heatEquation2D/src/analyticalSolution.hpp:31-56)."""
    from alpaka3_b200 import algo
    g = np.load(os.path.join(GOLDEN, "heat_problem.npz"))
    n, steps, t_max = int(g["n"]), int(g["steps"]), float(g["t_max"])
    u = algo.heat_problem(n, steps, t_max, cuda).cpu().numpy()
    ref = g["u"]
    assert np.max(np.abs(u - ref)) <= 1e-12 * np.max(np.abs(ref))
    dx = 1.0 / (n + 1)
    j, i = np.meshgrid(np.arange(n + 2), np.arange(n + 2))
    exact = np.exp(-np.pi ** 2 * t_max) * (np.sin(np.pi * j * dx) + np.sin(np.pi * i * dx))
    err = np.max(np.abs(u[1:-1, 1:-1] - exact[1:-1, 1:-1]))
    assert err < 1e-4
    assert abs(err - float(g["err"])) <= 1e-9


@pytest.mark.parametrize("rows,cols,pad", [(1000, 1000, 0), (130, 64, 0), (64, 130, 0), (200, 999, 1), (7, 12, 0),
                                           (97, 2046, 0)])
def test_halo_step_one_rank_matches_plain_step(cuda, rows, cols, pad):
    """The fused halo step (a3b_heat_step_halo) on a one-rank mailbox: the slab is the whole grid, so it must give the
    plain stencil's bits step after step. Even widths run the boundary bands on the register march and the interior
    on the shared-memory ring; odd widths (pitch padded to even) run the register march everywhere."""
    import ctypes

    from alpaka3_b200 import algo, capi
    L = capi.lib()
    pitch = cols + 2 + pad
    store = torch.zeros((rows + 2, pitch), dtype=torch.float64, device=cuda)
    u = store[:, :cols + 2]
    dx = 1.0 / (cols + 1)
    algo.heat_init(u, dx, 1.0 / (rows + 1))
    a = [store.clone(), store.clone()]
    b = [store.clone(), store.clone()]
    handle = (ctypes.c_char * L.a3b_ipc_handle_size())()
    h = ctypes.c_void_p()
    capi.call("a3b_halo_create", 1, 0, cols, ctypes.byref(h), handle)
    try:
        capi.call("a3b_halo_connect", h, handle)
        s = algo.stream_handle()
        capi.call("a3b_heat_halo_publish", s, h, ctypes.c_void_p(a[0].data_ptr()), rows, cols, pitch)
        for k in range(5):
            src, dst = a[k % 2], a[(k + 1) % 2]
            capi.call("a3b_heat_step_halo", s, h, ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()),
                      rows, cols, pitch, 0.2, 0.2)
            algo.heat_step(b[k % 2][:, :cols + 2], b[(k + 1) % 2][:, :cols + 2], 0.2, 0.2)
        torch.cuda.synchronize()
        assert capi.device_error(s) == 0
        assert torch.equal(a[1][1:rows + 1, :cols + 2], b[1][1:rows + 1, :cols + 2])
    finally:
        torch.cuda.synchronize()
        capi.call("a3b_halo_destroy", h)
