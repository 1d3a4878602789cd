"""numpy bindings of the CPU oracle (test infrastructure only).

Two back ends:

* :class:`Port`  -- ``liboracle.so``, the C restatement in ``oracle.c`` (always available once built);
* :class:`Ref`   -- ``_ref/libalpaka_ref.so``, alpaka3's own host backend (``exec::cpuSerial`` = 0,
  ``exec::cpuOmpBlocks`` = 1) driven through its public onHost API by ``ref_harness.cpp``.

Only the test suite, the smoke check and the CPU-baseline / reference arm of ``bench.py`` import this module. The
product library never does.
"""
import ctypes
import os

import numpy as np

from . import build as _build

_P = ctypes.c_void_p
_U64 = ctypes.c_uint64
_U32 = ctypes.c_uint32

SEED = 0x5EED0001


def _p(a):
    return a.ctypes.data_as(_P)


class Port:
    """The C restatement (``oracle.c``)."""

    def __init__(self, path=None):
        path = path or _build.ORACLE_SO
        if not os.path.exists(path):
            _build.build_oracle()
        self.lib = ctypes.CDLL(path)
        L = self.lib
        for name in ("orc_sumsq_f32", "orc_sumsq_f64", "orc_sum_f32", "orc_sum_f64"):
            getattr(L, name).restype = ctypes.c_double
            getattr(L, name).argtypes = [_P, _U64]
        for name in ("orc_dot_f64", "orc_dot_f32"):
            getattr(L, name).restype = ctypes.c_double
            getattr(L, name).argtypes = [_P, _P, _U64]
        L.orc_reduce_i32.restype = ctypes.c_int32
        L.orc_reduce_i32.argtypes = [ctypes.c_int, _P, _U64, ctypes.c_int32]
        L.orc_reduce_u32.restype = ctypes.c_uint32
        L.orc_reduce_u32.argtypes = [ctypes.c_int, _P, _U64, ctypes.c_uint32]
        L.orc_reduce_i64.restype = ctypes.c_int64
        L.orc_reduce_i64.argtypes = [ctypes.c_int, _P, _U64, ctypes.c_int64]
        L.orc_reduce_u64.restype = ctypes.c_uint64
        L.orc_reduce_u64.argtypes = [ctypes.c_int, _P, _U64, ctypes.c_uint64]
        L.orc_gen_u32.argtypes = [_U64, _U64, _U64, ctypes.c_int, _P]
        L.orc_gen_u64.argtypes = [_U64, _U64, _U64, _P]
        L.orc_gen_f32.argtypes = [_U64, _U64, _U64, ctypes.c_float, ctypes.c_float, _P]
        L.orc_stream_f64.argtypes = [ctypes.c_int, _P, _P, _P, _U64] + [ctypes.c_double] * 4
        L.orc_stream_f32.argtypes = [ctypes.c_int, _P, _P, _P, _U64] + [ctypes.c_float] * 4
        for name in ("orc_scan_u32", "orc_scan_u64", "orc_scan_f32", "orc_scan_f64"):
            getattr(L, name).argtypes = [ctypes.c_int, _P, _P, _U64]
        L.orc_heat_init.argtypes = [_P, _U32, ctypes.c_double, ctypes.c_double]
        L.orc_heat_step.argtypes = [_P, _P, _U32, ctypes.c_double, ctypes.c_double]
        L.orc_nbody_step.argtypes = [_P] * 7 + [_U64, ctypes.c_float, ctypes.c_float]
        L.orc_nbody_accel_sample.argtypes = [_P] * 4 + [_U64, ctypes.c_float, _P, _U64, _P]
        L.orc_philox.argtypes = [_U64, _U64, _P]
        L.orc_haccmk_init.argtypes = [ctypes.c_int, _P, _P, _P, _P]
        L.orc_haccmk_step10.argtypes = [ctypes.c_int, ctypes.c_int] + [_P] * 4 + [ctypes.c_float] * 3 + [_P] * 3
        L.orc_num_threads.restype = ctypes.c_int

    # ---- seeded inputs (Philox4x32-10, counter = element index) ----
    def gen_u32(self, n, seed=SEED, start=0, shift=0):
        out = np.empty(n, dtype=np.uint32)
        self.lib.orc_gen_u32(seed, start, n, shift, _p(out))
        return out

    def gen_u64(self, n, seed=SEED, start=0):
        out = np.empty(n, dtype=np.uint64)
        self.lib.orc_gen_u64(seed, start, n, _p(out))
        return out

    def gen_f32(self, n, lo=-1.0, hi=1.0, seed=SEED, start=0):
        out = np.empty(n, dtype=np.float32)
        self.lib.orc_gen_f32(seed, start, n, lo, hi, _p(out))
        return out

    def philox(self, seed, i):
        out = np.empty(4, dtype=np.uint32)
        self.lib.orc_philox(seed, i, _p(out))
        return out

    # ---- BabelStream ----
    KINDS = {"init": 0, "copy": 1, "mul": 2, "add": 3, "triad": 4, "nstream": 5}

    def stream(self, kind, a, b, c, scalar=0.4, init=(0.1, 0.2, 0.0)):
        f = self.lib.orc_stream_f64 if a.dtype == np.float64 else self.lib.orc_stream_f32
        f(self.KINDS[kind], _p(a), _p(b), _p(c), a.size, scalar, *init)

    # ---- reductions ----
    def sumsq(self, x):
        return (self.lib.orc_sumsq_f32 if x.dtype == np.float32 else self.lib.orc_sumsq_f64)(_p(x), x.size)

    def sum(self, x):
        return (self.lib.orc_sum_f32 if x.dtype == np.float32 else self.lib.orc_sum_f64)(_p(x), x.size)

    def dot(self, x, y):
        return (self.lib.orc_dot_f32 if x.dtype == np.float32 else self.lib.orc_dot_f64)(_p(x), _p(y), x.size)

    def reduce_int(self, op, x, neutral=None):
        """op: 'plus' | 'min' | 'max' over an integer array (plus wraps)."""
        x = np.ascontiguousarray(x)
        code = {"plus": 0, "min": 1, "max": 2}[op]
        info = np.iinfo(x.dtype)
        if neutral is None:
            neutral = {"plus": 0, "min": info.max, "max": info.min}[op]
        f = {np.dtype(np.int32): self.lib.orc_reduce_i32, np.dtype(np.uint32): self.lib.orc_reduce_u32,
             np.dtype(np.int64): self.lib.orc_reduce_i64, np.dtype(np.uint64): self.lib.orc_reduce_u64}[x.dtype]
        return x.dtype.type(f(code, _p(x), x.size, int(neutral)))

    # ---- scans ----
    def scan(self, x, inclusive):
        x = np.ascontiguousarray(x)
        out = np.empty_like(x)
        view = x
        if x.dtype in (np.int32, np.uint32):
            f, view, outv = self.lib.orc_scan_u32, x.view(np.uint32), out.view(np.uint32)
        elif x.dtype in (np.int64, np.uint64):
            f, view, outv = self.lib.orc_scan_u64, x.view(np.uint64), out.view(np.uint64)
        elif x.dtype == np.float32:
            f, outv = self.lib.orc_scan_f32, out
        else:
            f, outv = self.lib.orc_scan_f64, out
        f(int(bool(inclusive)), _p(view), _p(outv), x.size)
        return out

    # ---- heat ----
    def heat_init(self, n, dx, dy):
        u = np.empty((n + 2, n + 2), dtype=np.float64)
        self.lib.orc_heat_init(_p(u), n, dx, dy)
        return u

    def heat_steps(self, u, n, rX, rY, steps):
        cur = u.copy()
        nxt = u.copy()
        for _ in range(steps):
            self.lib.orc_heat_step(_p(cur), _p(nxt), n, rX, rY)
            cur, nxt = nxt, cur
        return cur

    # ---- nBody ----
    def nbody_steps(self, m, x, y, z, vx, vy, vz, dt, eps, steps):
        arrs = [np.ascontiguousarray(a, dtype=np.float32).copy() for a in (x, y, z, vx, vy, vz)]
        m = np.ascontiguousarray(m, dtype=np.float32)
        for _ in range(steps):
            self.lib.orc_nbody_step(_p(m), *[_p(a) for a in arrs], m.size, dt, eps)
        return arrs

    def nbody_accel_sample(self, m, x, y, z, eps, idx):
        idx = np.ascontiguousarray(idx, dtype=np.int64)
        out = np.empty((idx.size, 3), dtype=np.float64)
        self.lib.orc_nbody_accel_sample(_p(m), _p(x), _p(y), _p(z), m.size, eps, _p(idx), idx.size, _p(out))
        return out

    def haccmk_init(self, n2):
        """HACCmk's input (main_alpaka.cpp:254-272): xx, yy, zz, mass of n2 particles."""
        arrs = [np.empty(n2, dtype=np.float32) for _ in range(4)]
        self.lib.orc_haccmk_init(n2, *[_p(a) for a in arrs])
        return arrs

    def haccmk_step10(self, n1, xx, yy, zz, mass, fsrrmax2=0.5, mp_rsm2=0.03, fcoeff=0.23):
        out = [np.zeros(n1, dtype=np.float32) for _ in range(3)]
        self.lib.orc_haccmk_step10(n1, xx.size, _p(xx), _p(yy), _p(zz), _p(mass), fsrrmax2, mp_rsm2, fcoeff,
                                   *[_p(a) for a in out])
        return out

    def num_threads(self):
        return self.lib.orc_num_threads()


class Ref:
    """alpaka3's own host backend (``exec::cpuSerial`` = 0, ``exec::cpuOmpBlocks`` = 1)."""

    def __init__(self, path=None):
        path = path or _build.REF_SO
        if not os.path.exists(path):
            built = _build.build_ref()
            if not built or not os.path.exists(built):
                raise FileNotFoundError("oracle/_ref/libalpaka_ref.so is not built (reference tree absent)")
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.ref_babelstream_f64.argtypes = [ctypes.c_int, _P, _P, _P, _U32, ctypes.c_int, ctypes.c_int, _P, _P]
        L.ref_babelstream_f32.argtypes = [ctypes.c_int, _P, _P, _P, _U32, ctypes.c_int, ctypes.c_int, _P, _P]
        L.ref_sumsq_f32.argtypes = [ctypes.c_int, _P, _U64, _P]
        L.ref_sumsq_f64.argtypes = [ctypes.c_int, _P, _U64, _P]
        L.ref_dot_f64.argtypes = [ctypes.c_int, _P, _P, _U64, _P]
        L.ref_reduce_i32.argtypes = [ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int, _P]
        L.ref_reduce_f64.argtypes = [ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int, _P]
        for t in ("i32", "u32", "u64", "i64", "f64"):
            getattr(L, "ref_scan_" + t).argtypes = [ctypes.c_int, ctypes.c_int, _P, _P, _U64]
        L.ref_heat_steps.argtypes = [ctypes.c_int, _P, _P, _U32, _U32, ctypes.c_double, ctypes.c_double,
                                     ctypes.c_double]
        L.ref_nbody_steps.argtypes = [ctypes.c_int] + [_P] * 7 + [_U32, _U32, ctypes.c_float]
        L.ref_heat_problem.argtypes = [ctypes.c_int, _U32, _U32, ctypes.c_double, _P]
        L.ref_heat_problem.restype = ctypes.c_double
        L.ref_num_threads.restype = ctypes.c_int
        L.ref_set_num_threads.argtypes = [ctypes.c_int]
        L.ref_haccmk_gold.argtypes = [ctypes.c_int, ctypes.c_int] + [_P] * 4 + [ctypes.c_float] * 3 + [_P] * 3

    def haccmk_gold(self, n1, xx, yy, zz, mass, fsrrmax2=0.5, mp_rsm2=0.03, fcoeff=0.23):
        """HACCmk's own CPU gold (helper.hpp) for the first n1 particles."""
        out = [np.zeros(n1, dtype=np.float32) for _ in range(3)]
        assert self.lib.ref_haccmk_gold(n1, xx.size, _p(xx), _p(yy), _p(zz), _p(mass), fsrrmax2, mp_rsm2, fcoeff,
                                        *[_p(a) for a in out]) == 0
        return out

    def set_num_threads(self, n):
        """OpenMP threads of alpaka3's host backend for every later call."""
        self.lib.ref_set_num_threads(int(n))

    KERNELS = {"copy": 1, "mul": 2, "add": 4, "triad": 8, "dot": 16, "nstream": 32}

    def babelstream(self, n, runs, dtype=np.float64, kernels=("copy", "mul", "add", "triad", "dot"), exec_kind=1):
        """Runs the reference BabelStream sequence; returns (a, b, c, dot, per-run times[runs, 5])."""
        a = np.empty(n, dtype=dtype)
        b = np.empty(n, dtype=dtype)
        c = np.empty(n, dtype=dtype)
        dot = np.zeros(1, dtype=dtype)
        times = np.zeros((runs, 5), dtype=np.float64)
        mask = sum(self.KERNELS[k] for k in kernels)
        f = self.lib.ref_babelstream_f64 if dtype == np.float64 else self.lib.ref_babelstream_f32
        rc = f(exec_kind, _p(a), _p(b), _p(c), n, runs, mask, _p(dot), _p(times))
        assert rc == 0
        return a, b, c, dot[0], times

    def sumsq(self, x, exec_kind=1):
        out = np.zeros(1, dtype=x.dtype)
        f = self.lib.ref_sumsq_f32 if x.dtype == np.float32 else self.lib.ref_sumsq_f64
        f(exec_kind, _p(x), x.size, _p(out))
        return out[0]

    def dot(self, x, y, exec_kind=1):
        out = np.zeros(1, dtype=np.float64)
        self.lib.ref_dot_f64(exec_kind, _p(x), _p(y), x.size, _p(out))
        return out[0]

    def reduce(self, op, x, exec_kind=1):
        """x: contiguous int32 or float64 array of dimension 1..4 (alpaka extents, slowest first)."""
        code = {"plus": 0, "min": 1, "max": 2}[op]
        ext = np.array(x.shape, dtype=np.uint64)
        out = np.zeros(1, dtype=x.dtype)
        f = self.lib.ref_reduce_i32 if x.dtype == np.int32 else self.lib.ref_reduce_f64
        rc = f(exec_kind, code, _p(np.ascontiguousarray(x)), _p(ext), x.ndim, _p(out))
        assert rc == 0
        return out[0]

    def scan(self, x, inclusive, exec_kind=1):
        x = np.ascontiguousarray(x)
        out = np.empty_like(x)
        name = {np.dtype(np.int32): "i32", np.dtype(np.uint32): "u32", np.dtype(np.uint64): "u64",
                np.dtype(np.int64): "i64", np.dtype(np.float64): "f64"}[x.dtype]
        getattr(self.lib, "ref_scan_" + name)(exec_kind, int(bool(inclusive)), _p(x), _p(out), x.size)
        return out

    def heat_steps(self, u, n, dx, dy, dt, steps, exec_kind=1):
        cur = np.ascontiguousarray(u, dtype=np.float64).copy()
        nxt = cur.copy()
        rc = self.lib.ref_heat_steps(exec_kind, _p(cur), _p(nxt), n, steps, dx, dy, dt)
        assert rc == 0
        return cur

    def heat_problem(self, n, steps, t_max, exec_kind=1):
        """The heatEquation2D example's own problem; returns (final (n+2)^2 field, its validation error)."""
        out = np.empty((n + 2, n + 2), dtype=np.float64)
        err = self.lib.ref_heat_problem(exec_kind, n, steps, t_max, _p(out))
        return out, err

    def nbody_steps(self, m, x, y, z, vx, vy, vz, dt, steps, exec_kind=1):
        """Reference step with its built-in softening EPS = 4 (example/nBody/src/common.hpp:41)."""
        arrs = [np.ascontiguousarray(a, dtype=np.float32).copy() for a in (m, x, y, z, vx, vy, vz)]
        rc = self.lib.ref_nbody_steps(exec_kind, *[_p(a) for a in arrs], m.size, steps, dt)
        assert rc == 0
        return arrs[1:]

    def num_threads(self):
        return self.lib.ref_num_threads()
