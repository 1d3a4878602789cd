"""Python mirror of alpaka3's onHost algorithm entry points for the primitive path, over the C ABI.

Device buffers are torch CUDA tensors (plumbing only: allocation, streams); every computation is one call into
``libalpaka3_b200.so``. Names and argument meaning follow include/alpaka/onHost/algo/*.hpp:

* :func:`transform`           onHost::transform            (algo/transform.hpp:50-88)
* :func:`transform_reduce`    onHost::transformReduce      (algo/transformReduce.hpp:59-114)
* :func:`reduce`              onHost::reduce               (algo/reduce.hpp:28-79)
* :func:`inclusive_scan` / :func:`exclusive_scan` (+ ``in_place``), :func:`get_scan_buffer_size`
                              onHost::*Scan[InPlace], getScanBufferSize (algo/scan.hpp:26-218)
* :func:`fill`, :func:`iota`  onHost::fill (Queue.hpp:346), onHost::iota (algo/iota.hpp:29-85)
* :func:`babelstream`         the BabelStream kernels (benchmark/babelstream/src/babelStreamMainTest.cpp:78-141)
* :func:`nbody_step`, :func:`nbody_update_velocities`, :func:`nbody_update_positions`  (example/nBody)
* :func:`heat_step`, :func:`heat_init`  (example/heatEquation2D)

Errors raise :class:`alpaka3_b200.capi.A3BError` (the reference throws std::runtime_error on backend errors).
"""
import ctypes

import numpy as np
import torch

from . import capi

_DT = {torch.int32: capi.I32, torch.uint32: capi.U32, torch.int64: capi.I64, torch.uint64: capi.U64,
       torch.float32: capi.F32, torch.float64: capi.F64}
_NP = {capi.I32: np.int32, capi.U32: np.uint32, capi.I64: np.int64, capi.U64: np.uint64, capi.F32: np.float32,
       capi.F64: np.float64}
REDUCE = {"plus": capi.PLUS, "min": capi.MIN, "max": capi.MAX}
XFORM = {"identity": capi.IDENTITY, "square": capi.SQUARE, "product": capi.PRODUCT}
STREAM = {"init": capi.INIT, "copy": capi.COPY, "mul": capi.MUL, "add": capi.ADD, "triad": capi.TRIAD,
          "nstream": capi.NSTREAM}
MAP = {"copy": capi.MAP_COPY, "scale": capi.MAP_SCALE, "add": capi.MAP_ADD, "mul": capi.MAP_MUL,
       "axpy": capi.MAP_AXPY, "square": capi.MAP_SQUARE}


def dtype_code(t):
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def stream_handle(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return ctypes.c_void_p(t.data_ptr())


def _host_scalar(value, code):
    arr = np.array([value], dtype=_NP[code])
    return arr, arr.ctypes.data_as(ctypes.c_void_p)


def _neutral(op, code):
    dt = np.dtype(_NP[code])
    if op == "plus":
        return 0
    if dt.kind == "f":
        return np.inf if op == "min" else -np.inf
    info = np.iinfo(dt)
    return info.max if op == "min" else info.min


# ------------------------------------------------------------------------------------------------ element-wise
def babelstream(kind, a, b, c, scalar=0.4, init=(0.1, 0.2, 0.0), stream=None):
    code = dtype_code(a)
    ini = (ctypes.c_double * 3)(*init)
    capi.call("a3b_babelstream", stream_handle(stream), STREAM[kind], code, _ptr(a), _ptr(b), _ptr(c), a.numel(),
              float(scalar), ini)


def transform(kind, out, in0, in1=None, alpha=1.0, stream=None):
    capi.call("a3b_transform", stream_handle(stream), MAP[kind], dtype_code(out), _ptr(out), _ptr(in0), _ptr(in1),
              out.numel(), float(alpha))
    return out


def fill(out, value, stream=None):
    code = dtype_code(out)
    keep, p = _host_scalar(value, code)
    capi.call("a3b_fill", stream_handle(stream), code, _ptr(out), out.numel(), p)
    return out


def iota(out, start=0, stream=None):
    code = dtype_code(out)
    keep, p = _host_scalar(start, code)
    capi.call("a3b_iota", stream_handle(stream), code, _ptr(out), out.numel(), p)
    return out


def random_u32(out, seed, start=0, shift=0, stream=None):
    capi.call("a3b_random_u32", stream_handle(stream), _ptr(out), out.numel(), seed, start, shift)
    return out


def random_u64(out, seed, start=0, stream=None):
    capi.call("a3b_random_u64", stream_handle(stream), _ptr(out), out.numel(), seed, start)
    return out


def random_f32(out, seed, lo=-1.0, hi=1.0, start=0, stream=None):
    capi.call("a3b_random_f32", stream_handle(stream), _ptr(out), out.numel(), seed, start, lo, hi)
    return out


# -------------------------------------------------------------------------------------------------- reductions
def set_early_start(enable=True, stream=None):
    """Let the reductions on `stream` start while the previous kernel of the stream still runs (programmatic
    dependent launch; off by default). Enable it only when no kernel on the stream signals its dependents early
    (griddepcontrol.launch_dependents) before writing its output."""
    capi.call("a3b_set_early_start", stream_handle(stream), 1 if enable else 0)


def transform_reduce(neutral, out, reduce_fn, transform_fn, in0, in1=None, stream=None):
    """onHost::transformReduce(queue, neutral, out, reduceFn, transformFn, in0[, in1]); out: 1-element tensor."""
    code = dtype_code(in0)
    if out.dtype != in0.dtype or out.numel() < 1:
        raise ValueError("out must hold one element of the input dtype")
    if neutral is None:
        neutral = _neutral(reduce_fn, code)
    keep, p = _host_scalar(neutral, code)
    capi.call("a3b_transform_reduce", stream_handle(stream), code, REDUCE[reduce_fn], XFORM[transform_fn], _ptr(in0),
              _ptr(in1), in0.numel(), p, _ptr(out))
    return out


def transform_reduce_partial(reduce_fn, transform_fn, in0, in1=None, partial=None, neutral=None, stream=None):
    """Un-rounded 8-byte partial (float64 for float inputs, int64/uint64 for integers) for cross-GPU combination."""
    code = dtype_code(in0)
    if partial is None:
        pdt = torch.float64 if code in (capi.F32, capi.F64) else (torch.int64 if code in (capi.I32, capi.I64)
                                                                   else torch.uint64)
        partial = torch.empty(1, dtype=pdt, device=in0.device)
    if neutral is None:
        neutral = _neutral(reduce_fn, code)
    keep, p = _host_scalar(neutral, code)
    capi.call("a3b_transform_reduce_partial", stream_handle(stream), code, REDUCE[reduce_fn], XFORM[transform_fn],
              _ptr(in0), _ptr(in1), in0.numel(), p, _ptr(partial))
    return partial


def reduce(neutral, out, reduce_fn, data, stream=None):
    """onHost::reduce over a 1-D..N-D tensor; a tensor whose rows (last dim) are strided by a constant pitch is
    passed as a pitched 2-D view without copying."""
    code = dtype_code(data)
    if neutral is None:
        neutral = _neutral(reduce_fn, code)
    keep, p = _host_scalar(neutral, code)
    if data.is_contiguous():
        rows, row_len, pitch = 1, data.numel(), data.numel() * data.element_size()
    else:
        if data.dim() != 2 or data.stride(1) != 1:
            raise ValueError("non-contiguous input must be a 2-D view with unit stride in the last dimension")
        rows, row_len, pitch = data.shape[0], data.shape[1], data.stride(0) * data.element_size()
    capi.call("a3b_reduce_2d", stream_handle(stream), code, REDUCE[reduce_fn], ctypes.c_void_p(data.data_ptr()),
              rows, row_len, pitch, p, _ptr(out))
    return out


# -------------------------------------------------------------------------------------------------------- scan
def get_scan_buffer_size(dtype, n):
    code = _DT[dtype]
    return capi.lib().a3b_scan_buffer_size(code, n)


def _scan(inclusive, out, data, buffer=None, carry=None, stream=None):
    code = dtype_code(data)
    if out.dtype != data.dtype or out.numel() != data.numel():
        raise ValueError("output must match the input's dtype and size")
    bp = _ptr(buffer) if buffer is not None else None
    bb = buffer.numel() * buffer.element_size() if buffer is not None else 0
    capi.call("a3b_scan", stream_handle(stream), code, 1 if inclusive else 0, _ptr(data), _ptr(out), data.numel(),
              _ptr(carry), bp, bb)
    return out


def inclusive_scan(out, data, buffer=None, carry=None, stream=None):
    return _scan(True, out, data, buffer, carry, stream)


def exclusive_scan(out, data, buffer=None, carry=None, stream=None):
    return _scan(False, out, data, buffer, carry, stream)


def inclusive_scan_in_place(data, buffer=None, stream=None):
    return _scan(True, data, data, buffer, None, stream)


def exclusive_scan_in_place(data, buffer=None, stream=None):
    return _scan(False, data, data, buffer, None, stream)


# ------------------------------------------------------------------------------------------------------- nBody
def nbody_update_velocities(m, x, y, z, vx, vy, vz, dt, eps, i_begin=0, stream=None):
    capi.call("a3b_nbody_update_velocities", stream_handle(stream), _ptr(m), _ptr(x), _ptr(y), _ptr(z), m.numel(),
              i_begin, vx.numel(), _ptr(vx), _ptr(vy), _ptr(vz), float(dt), float(eps))


def nbody_update_positions(x, y, z, vx, vy, vz, dt, stream=None):
    capi.call("a3b_nbody_update_positions", stream_handle(stream), _ptr(x), _ptr(y), _ptr(z), _ptr(vx), _ptr(vy),
              _ptr(vz), x.numel(), float(dt))


def nbody_step(m, x, y, z, vx, vy, vz, dt, eps, i_begin=0, stream=None):
    capi.call("a3b_nbody_step", stream_handle(stream), _ptr(m), _ptr(x), _ptr(y), _ptr(z), m.numel(), i_begin,
              vx.numel(), _ptr(vx), _ptr(vy), _ptr(vz), float(dt), float(eps))


# -------------------------------------------------------------------------------------------------------- heat
def haccmk_step10(xx, yy, zz, mass, vx2, vy2, vz2, n1, fsrrmax2, mp_rsm2, fcoeff, stream=None):
    """HACCmk's Step10 short-range force for the first n1 particles against all of xx/yy/zz/mass (float32)."""
    capi.call("a3b_haccmk_step10", stream_handle(stream), _ptr(xx), _ptr(yy), _ptr(zz), _ptr(mass), int(n1),
              xx.numel(), float(fsrrmax2), float(mp_rsm2), float(fcoeff), _ptr(vx2), _ptr(vy2), _ptr(vz2))


def heat_step(cur, nxt, rX, rY, row_begin=1, row_end=None, stream=None):
    """cur/nxt: (rows+2, cols+2) float64 tensors (rows may be pitched: stride(0) >= cols + 2)."""
    rows, cols = cur.shape[0] - 2, cur.shape[1] - 2
    if row_end is None:
        row_end = rows + 1
    if cur.stride(1) != 1 or nxt.stride() != cur.stride():
        raise ValueError("grids must share a row pitch and be contiguous within rows")
    capi.call("a3b_heat_step", stream_handle(stream), ctypes.c_void_p(cur.data_ptr()),
              ctypes.c_void_p(nxt.data_ptr()), rows, cols, cur.stride(0), row_begin, row_end, float(rX), float(rY))


def heat_init(u, dx, dy, row_offset=0, global_rows=None, stream=None):
    rows, cols = u.shape[0] - 2, u.shape[1] - 2
    if global_rows is None:
        global_rows = rows
    capi.call("a3b_heat_init", stream_handle(stream), ctypes.c_void_p(u.data_ptr()), rows, cols, u.stride(0),
              row_offset, global_rows, float(dx), float(dy))


def heat_exact(u, t, dx, dy, ring_only=False, row_offset=0, global_rows=None, stream=None):
    """The heatEquation2D example's exact solution at time t on every cell, or on the global ring only."""
    rows, cols = u.shape[0] - 2, u.shape[1] - 2
    if global_rows is None:
        global_rows = rows
    capi.call("a3b_heat_exact", stream_handle(stream), ctypes.c_void_p(u.data_ptr()), rows, cols, u.stride(0),
              row_offset, global_rows, float(t), float(dx), float(dy), 1 if ring_only else 0)


def heat_problem(n, steps, t_max, device, stream=None):
    """Runs the heatEquation2D example's own problem (heatEquation2D.cpp:97-196) on the device: exact initial field,
    `steps` Jacobi steps with the exact solution re-imposed on the ring after each; returns the final field."""
    extent = n + 2
    dx = 1.0 / (extent - 1)
    dy = 1.0 / (extent - 1)
    dt = t_max / steps
    rX = dt / (dx * dx)
    rY = dt / (dy * dy)
    cur = torch.empty((extent, extent), dtype=torch.float64, device=device)
    heat_exact(cur, 0.0, dx, dy, stream=stream)
    nxt = cur.clone()
    for step in range(1, steps + 1):
        heat_step(cur, nxt, rX, rY, stream=stream)
        heat_exact(nxt, float(step) * dt, dx, dy, ring_only=True, stream=stream)
        cur, nxt = nxt, cur
    return cur
