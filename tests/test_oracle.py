"""CPU: the C restatement (oracle/oracle.c) pinned against alpaka3's own host backend and the golden fixtures."""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_philox_known_answer(port):
    # Random123 known-answer vector for Philox4x32-10 with counter 0 and key 0
    assert [hex(v) for v in port.philox(0, 0)] == ["0x6627e8d5", "0xe169c58d", "0xbc57ac4c", "0x9b00dbd8"]


@pytest.mark.parametrize("n", [12, 1024, 654321, 20971520])
@pytest.mark.parametrize("kind", ["excl", "incl"])
def test_scan_iota_golden(port, n, kind):
    g = json.load(open(os.path.join(GOLDEN, "scan_iota.json")))[f"{n}_{kind}"]
    y = port.scan(np.arange(n, dtype=np.int64).astype(np.int32), kind == "incl")
    assert _sha(y) == g["sha256"]
    assert y[:4].tolist() == g["head"] and y[-4:].tolist() == g["tail"]


def test_scan_matches_reference_random(port, ref):
    x = port.gen_u32(300001, shift=28)
    for incl in (0, 1):
        assert (port.scan(x, incl) == ref.scan(x, incl)).all()
    u = port.gen_u64(100003)
    for incl in (0, 1):
        assert (port.scan(u, incl) == ref.scan(u, incl)).all()


def test_reduce_iota_golden(port):
    g = json.load(open(os.path.join(GOLDEN, "reduce_iota.json")))
    for key, want in g.items():
        n = int(np.prod([int(v) for v in key.split("x")]))
        x = np.arange(n, dtype=np.int32)
        for op, v in want.items():
            assert int(port.reduce_int(op, x)) == v, (key, op)


def test_babelstream_golden_bitexact(port):
    g = json.load(open(os.path.join(GOLDEN, "babelstream.json")))
    for name, dt in (("f64", np.float64), ("f32", np.float32)):
        n, runs = g[name]["n"], g[name]["runs"]
        a, b, c = (np.empty(n, dt) for _ in range(3))
        port.stream("init", a, b, c)
        for _ in range(runs):
            for k in ("copy", "mul", "add", "triad"):
                port.stream(k, a, b, c)
        for arr, key in ((a, "a_hex"), (b, "b_hex"), (c, "c_hex")):
            assert (arr == arr[0]).all()
            assert np.array(arr[0]).tobytes().hex() == g[name][key]
        # dot: reference sums in its own order; the gold check of babelStreamMainTest.cpp:419-431
        assert abs(port.dot(a, b) - g[name]["dot"]) / abs(g[name]["dot"]) < (1e-12 if dt == np.float64 else 1e-5)


def test_babelstream_matches_reference(port, ref):
    a, b, c, dot, _ = ref.babelstream(4099, 3, exec_kind=1)
    A, B, C = (np.empty(4099) for _ in range(3))
    port.stream("init", A, B, C)
    for _ in range(3):
        for k in ("copy", "mul", "add", "triad"):
            port.stream(k, A, B, C)
    assert (A == a).all() and (B == b).all() and (C == c).all()


def test_heat_golden_bitexact(port):
    g = np.load(os.path.join(GOLDEN, "heat.npz"))
    n, dx, dt, steps = int(g["n"]), float(g["dx"]), float(g["dt"]), int(g["steps"])
    u0 = port.heat_init(n, dx, dx)
    assert (u0 == g["u0"]).all()
    r = dt / (dx * dx)
    u = port.heat_steps(u0, n, r, r, steps)
    assert (u == g["u25"]).all()


def test_nbody_golden_bitexact(port):
    g = np.load(os.path.join(GOLDEN, "nbody.npz"))
    z0 = np.zeros_like(g["m"])
    out = port.nbody_steps(g["m"], g["x0"], g["y0"], g["z0"], z0, z0, z0, float(g["dt"]), float(g["eps"]),
                           int(g["steps"]))
    for arr, key in zip(out, ("x", "y", "z", "vx", "vy", "vz")):
        assert (arr == g[key]).all(), key


def test_sumsq_golden(port):
    g = json.load(open(os.path.join(GOLDEN, "sumsq.json")))
    x = port.gen_f32(g["n"], -1.0, 1.0, seed=g["seed"])
    assert _sha(x) == g["input_sha256"]
    exact = port.sumsq(x)
    # the reference's own fp32 transformReduce lands within the fp32 tolerance of the compensated fp64 sum
    assert abs(g["ref_fp32"] - exact) / exact < 1e-5


def test_reduce_matches_reference_nd(port, ref):
    for ext in ((5, 7, 3, 11), (93, 7, 123), (7, 3)):
        x = port.gen_u32(int(np.prod(ext)), shift=1).astype(np.int32).reshape(ext)
        for op in ("plus", "min", "max"):
            assert ref.reduce(op, x) == port.reduce_int(op, x.ravel())


def test_heat_example_problem_golden(ref):
    """The heatEquation2D example's own problem through alpaka3's host backend reproduces the fixture and passes the
    example's analytical check (max error < 1e-4)."""
    g = np.load(os.path.join(GOLDEN, "heat_problem.npz"))
    u, err = ref.heat_problem(int(g["n"]), int(g["steps"]), float(g["t_max"]))
    assert (u == g["u"]).all()
    assert err < 1e-4 and err == float(g["err"])


def test_haccmk_restatement_matches_reference_gold(port, ref):
    """oracle.c's HACCmk step equals the benchmark's own CPU gold (benchmark/HACCmk/src/helper.hpp:19-66) bit for bit,
    at the benchmark's default size (15000 particles, 784 active) and two others."""
    import numpy as np
    for n2, n1 in ((15000, 784), (1000, 1000), (4096, 100)):
        xx, yy, zz, m = port.haccmk_init(n2)
        a = port.haccmk_step10(n1, xx, yy, zz, m)
        b = ref.haccmk_gold(n1, xx, yy, zz, m)
        for x, y in zip(a, b):
            assert (x.view(np.uint32) == y.view(np.uint32)).all()
