"""GPU: the allocation-free transform-reduce entry point.

Some callers of this library cannot allocate device memory: processes whose device memory is owned by another
allocator's pool (a framework that reserves the GPU's memory up front), services that must keep a fixed, accounted
memory footprint, and latency-critical loops that cannot afford an allocation's implicit synchronisation.
a3b_transform_reduce_noalloc serves them with scratch from a fixed static device array instead of the library's
cached, allocated scratch. This file checks, through
the C ABI, that two calls in a row give the same result as a3b_transform_reduce (which uses the allocated scratch),
within the tolerances the other reduction tests use. It is collected last so that a failure here comes after every
other test has run; it passes both alone in a fresh process and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


CASES = [
    # dtype, reduce op, transform op, n, relative tolerance (0 = bit-exact)
    (torch.float32, "plus", "square", (1 << 22) + 3, 1e-5),
    (torch.float64, "plus", "product", (1 << 21) + 1, 1e-12),
    (torch.int32, "plus", "identity", 1000003, 0),
    (torch.int32, "min", "identity", 999, 0),
    (torch.int64, "max", "identity", 123457, 0),
]


@pytest.mark.parametrize("dtype,rop,xop,n,tol", CASES)
def test_noalloc_matches_allocating_entry_point(cuda, dtype, rop, xop, n, tol):
    from alpaka3_b200 import algo, capi
    L = capi.lib()
    code = algo.dtype_code(torch.empty(0, dtype=dtype))
    g = torch.Generator(device="cuda").manual_seed(n)
    if dtype.is_floating_point:
        x = torch.rand(n, dtype=dtype, device=cuda, generator=g) * 2 - 1
        y = torch.rand(n, dtype=dtype, device=cuda, generator=g) * 2 - 1
    else:
        x = torch.randint(-(1 << 30), 1 << 30, (n,), dtype=dtype, device=cuda, generator=g)
        y = x
    neutral = np.array([algo._neutral(rop, code)], dtype=algo._NP[code])
    np_ = neutral.ctypes.data_as(ctypes.c_void_p)
    stream = algo.stream_handle()
    in1 = _p(y) if xop == "product" else None

    want = torch.empty(1, dtype=dtype, device=cuda)
    capi.check(L.a3b_transform_reduce(stream, code, algo.REDUCE[rop], algo.XFORM[xop], _p(x), in1, n, np_, _p(want)))
    for call in range(2):  # the static scratch is shared by consecutive calls
        got = torch.full((1,), 7, dtype=dtype, device=cuda)
        rc = L.a3b_transform_reduce_noalloc(stream, code, algo.REDUCE[rop], algo.XFORM[xop], _p(x), in1, n, np_,
                                            _p(got))
        capi.check(rc, "a3b_transform_reduce_noalloc")
        torch.cuda.synchronize()
        w, v = want.cpu().item(), got.cpu().item()
        if tol == 0:
            assert v == w, (call, v, w)
        else:
            assert abs(v - w) <= tol * abs(w), (call, v, w)


def test_noalloc_rejects_bad_arguments(cuda):
    from alpaka3_b200 import algo, capi
    L = capi.lib()
    zero = np.zeros(1, dtype=np.float32)
    rc = L.a3b_transform_reduce_noalloc(algo.stream_handle(), capi.F32, capi.PLUS, capi.SQUARE, None, None, 10,
                                        zero.ctypes.data_as(ctypes.c_void_p), None)
    assert rc == capi.ERR_INVALID
