"""Generates the golden fixtures of tests/golden/ by running alpaka3's OWN host backend (oracle/_ref, built from the
reference headers by oracle/build_ref.sh) on the inputs the reference's unit tests and examples use.

Run here (where the reference tree exists):  python tests/golden/gen_golden.py
The fixtures are small (hashes, scalars, a few KB of arrays) and are committed; the tests never read the reference.

  scan_iota.json      test/unit/algorithm/scan.cpp:158-197: int iota 0..n-1, n in {12, 1024, 654321, 20971520},
                      exclusive and inclusive (int wraps at 20 Mi): sha256 of the int32 output + head/tail values
  reduce_iota.json    test/unit/algorithm/reduce.cpp:135-152: int iota over the reference's extents, plus/min/max
  babelstream.json    babelStreamMainTest.cpp:285-366 on exec::cpuSerial: 2^18 doubles and floats, 10 runs: final
                      a/b/c values (uniform arrays) and the dot result
  heat.npz            StencilKernel on a 64x64 interior, sin*sin start, 25 steps (dt = 0.2 dx^2)
  nbody.npz           UpdateVelocitiesKernel + UpdatePositions (built-in EPS = 4), 512 bodies, 3 steps, dt = 1e-3
  sumsq.json          transformReduce(plus, x*x) over 2^20 seeded fp32 in [-1, 1) (reference fp32 value)
  heat_problem.npz    the heatEquation2D example's own problem at its defaults (64 x 64, 4000 steps, tMax 0.1: exact
                      initial field, time-dependent Dirichlet ring): final field and the example's validation error
  nbody_262144.npz    the nBody workload itself: 262144 bodies (positions uniform in the unit cube, masses uniform in
                      [0.5, 1), velocities 0, seeded Philox streams), eps^2 = 1e-3, dt = 1e-3, 10 kick + drift steps:
                      final positions. The reference kernel hard-codes EPS = 4 (example/nBody/src/common.hpp:41), so
                      these come from the oracle restatement (oracle.c), which nbody.npz pins bit-exact to the
                      reference kernel at EPS = 4 (about a minute on 8 cores).

usage: python tests/golden/gen_golden.py [fixture-name ...]   (default: all)
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.oracle import Port, Ref, SEED  # noqa: E402

SCAN_SIZES = (12, 1024, 654321, 20971520)
REDUCE_EXTENTS = ((5, 7, 3, 11), (93, 7, 123), (5, 7, 4111), (5, 7, 3), (7, 3), (3,))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def nbody_full(port):
    n, steps, dt, eps = 262144, 10, 1e-3, 1e-3
    m = port.gen_f32(n, 0.5, 1.0, seed=SEED + 1)
    pos = [port.gen_f32(n, 0.0, 1.0, seed=SEED + s) for s in (2, 3, 4)]
    zeros = np.zeros(n, np.float32)
    out = port.nbody_steps(m, *pos, zeros, zeros, zeros, dt, eps, steps)
    np.savez_compressed(os.path.join(HERE, "nbody_262144.npz"), x=out[0], y=out[1], z=out[2], n=n, steps=steps, dt=dt,
                        eps=eps, vmax=max(float(np.max(np.abs(v))) for v in out[3:]),
                        input_sha256=sha(np.stack([m, *pos])))


def main():
    port = Port()
    only = set(sys.argv[1:])
    if only:
        if "nbody_262144" in only:
            nbody_full(port)
        print("written:", sorted(only))
        return
    ref = Ref()
    scan = {}
    for n in SCAN_SIZES:
        x = np.arange(n, dtype=np.int64).astype(np.int32)
        for incl in (0, 1):
            y = ref.scan(x, incl)
            scan[f"{n}_{'incl' if incl else 'excl'}"] = {"sha256": sha(y), "head": y[:4].tolist(),
                                                           "tail": y[-4:].tolist()}
    json.dump(scan, open(os.path.join(HERE, "scan_iota.json"), "w"), indent=1)

    red = {}
    for ext in REDUCE_EXTENTS:
        x = np.arange(int(np.prod(ext)), dtype=np.int32).reshape(ext)
        red["x".join(map(str, ext))] = {op: int(ref.reduce(op, x)) for op in ("plus", "min", "max")}
    json.dump(red, open(os.path.join(HERE, "reduce_iota.json"), "w"), indent=1)

    bs = {}
    for dt, name in ((np.float64, "f64"), (np.float32, "f32")):
        a, b, c, dot, _ = ref.babelstream(1 << 18, 10, dtype=dt, exec_kind=0)
        assert (a == a[0]).all() and (b == b[0]).all() and (c == c[0]).all()
        bs[name] = {"n": 1 << 18, "runs": 10, "a": float(a[0]), "b": float(b[0]), "c": float(c[0]),
                    "dot": float(dot), "a_hex": np.array(a[0]).tobytes().hex(), "b_hex": np.array(b[0]).tobytes().hex(),
                    "c_hex": np.array(c[0]).tobytes().hex()}
    json.dump(bs, open(os.path.join(HERE, "babelstream.json"), "w"), indent=1)

    n = 64
    dx = 1.0 / (n + 1)
    dt = 0.2 * dx * dx
    u0 = port.heat_init(n, dx, dx)
    u = ref.heat_steps(u0, n, dx, dx, dt, 25)
    np.savez_compressed(os.path.join(HERE, "heat.npz"), u0=u0, u25=u, n=n, dx=dx, dt=dt, steps=25)

    N = 512
    m = port.gen_f32(N, 0.5, 1.0, seed=SEED + 1)
    pos = [port.gen_f32(N, 0.0, 1.0, seed=SEED + s) for s in (2, 3, 4)]
    vel = [np.zeros(N, np.float32) for _ in range(3)]
    out = ref.nbody_steps(m, *pos, *vel, 1e-3, 3)
    np.savez_compressed(os.path.join(HERE, "nbody.npz"), m=m, x0=pos[0], y0=pos[1], z0=pos[2], x=out[0], y=out[1],
                        z=out[2], vx=out[3], vy=out[4], vz=out[5], dt=1e-3, eps=4.0, steps=3)

    x = port.gen_f32(1 << 20, -1.0, 1.0)
    json.dump({"n": 1 << 20, "seed": SEED, "ref_fp32": float(ref.sumsq(x)), "input_sha256": sha(x)},
              open(os.path.join(HERE, "sumsq.json"), "w"), indent=1)
    u, err = ref.heat_problem(64, 4000, 0.1)
    np.savez_compressed(os.path.join(HERE, "heat_problem.npz"), u=u, err=err, n=64, steps=4000, t_max=0.1)
    nbody_full(port)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
