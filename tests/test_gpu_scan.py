"""GPU parity: single-pass scan against the reference's own pins (test/unit/algorithm/scan.cpp:74-197) and the
oracle, bit-exact for integers; bounded wait timeout (failure detection without a GPU fault)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _h(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("n", [12, 1024, 654321, 20971520])
def test_scan_iota_pins_all_variants(cuda, n):
    """exclusive/inclusive x out-of-place/in-place x with/without a getScanBufferSize buffer, int iota input."""
    from alpaka3_b200 import algo
    g = json.load(open(os.path.join(GOLDEN, "scan_iota.json")))
    iota = torch.arange(n, dtype=torch.int32, device=cuda)
    out = torch.empty_like(iota)
    buf = torch.empty(algo.get_scan_buffer_size(torch.int32, n), dtype=torch.uint8, device=cuda)
    for kind, fn, fn_ip in (("excl", algo.exclusive_scan, algo.exclusive_scan_in_place),
                            ("incl", algo.inclusive_scan, algo.inclusive_scan_in_place)):
        want = g[f"{n}_{kind}"]["sha256"]
        for use_buf in (False, True):
            b = buf if use_buf else None
            out.fill_(-7)
            fn(out, iota, buffer=b)
            assert _sha(_h(out)) == want, (kind, "out-of-place", use_buf)
            data = iota.clone()
            fn_ip(data, buffer=b)
            assert _sha(_h(data)) == want, (kind, "in-place", use_buf)


@pytest.mark.parametrize("n", [1, 2, 31, 33, 4095, 4096, 4097, 8193, 1 << 20, (1 << 20) + 5])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_scan_random_sizes(cuda, port, n, dtype):
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    x = torch.empty(n, dtype=torch.int32, device=cuda)
    algo.random_u32(x, SEED, shift=28)
    if dtype == torch.int64:
        w = torch.empty(n, dtype=torch.int64, device=cuda)
        algo.random_u64(w, SEED)
        x = w
    h = _h(x)
    out = torch.empty_like(x)
    for incl in (False, True):
        (algo.inclusive_scan if incl else algo.exclusive_scan)(out, x)
        assert (_h(out) == port.scan(h, incl)).all()


def test_scan_u32_config_shape(cuda, port):
    """the exclusive-scan workload's input distribution (values in [0, 16)), 2^24 elements, unsigned wrap."""
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    n = 1 << 24
    x = torch.empty(n, dtype=torch.int32, device=cuda)
    algo.random_u32(x, SEED, shift=28)
    out = torch.empty_like(x)
    algo.exclusive_scan(out, x)
    assert (_h(out).view(np.uint32) == port.scan(port.gen_u32(n, shift=28), False)).all()


def test_scan_unaligned_and_carry(cuda, port):
    from alpaka3_b200 import algo
    n = 70001
    base = torch.randint(0, 100, (n + 3,), dtype=torch.int32, device=cuda)
    x = base[3:]  # 12-byte offset: scalar path
    out = torch.empty(n + 1, dtype=torch.int32, device=cuda)[1:]
    carry = torch.tensor([1000], dtype=torch.int32, device=cuda)
    algo.exclusive_scan(out, x, carry=carry)
    assert (_h(out) == port.scan(_h(x), False) + 1000).all()
    algo.inclusive_scan(out, x, carry=carry)
    assert (_h(out) == port.scan(_h(x), True) + 1000).all()


def test_scan_float(cuda, port):
    from alpaka3_b200 import algo
    n = 300007
    for dtype in (torch.float32, torch.float64):
        x = torch.rand(n, dtype=dtype, device=cuda)
        out = torch.empty_like(x)
        algo.inclusive_scan(out, x)
        want = np.cumsum(_h(x).astype(np.float64))
        tol = 1e-5 if dtype == torch.float32 else 1e-12
        assert np.max(np.abs(_h(out) - want)) <= tol * want[-1]


def test_repeated_calls_epochs(cuda, port):
    """many calls on one stream reuse the cached scratch through its epoch counter without clearing."""
    from alpaka3_b200 import algo
    x = torch.randint(0, 16, (123457,), dtype=torch.int32, device=cuda)
    out = torch.empty_like(x)
    want = port.scan(_h(x), False)
    for _ in range(50):
        algo.exclusive_scan(out, x)
    assert (_h(out) == want).all()
    y = torch.randint(0, 16, (1 << 21,), dtype=torch.int32, device=cuda)  # scratch grows
    out2 = torch.empty_like(y)
    algo.exclusive_scan(out2, y)
    algo.exclusive_scan(out, x)
    assert (_h(out2) == port.scan(_h(y), False)).all() and (_h(out) == want).all()


def test_aggregate_wait_timeout_reports_error(cuda):
    """A tile whose aggregate is never published (host-requested stall) makes the bounded waits of the tiles after it
    give up: the device error word reports a timeout, the kernel returns, and the context keeps working."""
    import ctypes
    from alpaka3_b200 import algo, capi
    s = algo.stream_handle()
    capi.device_error(s, clear=True)
    capi.call("a3b_set_wait_timeout_ns", 20_000_000)  # 20 ms
    try:
        n = 1 << 18  # at least 8 tiles for every tile size; tile 2 stalls
        x = torch.ones(n, dtype=torch.int32, device=cuda)
        out = torch.empty_like(x)
        capi.call("a3b_scan_debug_stall", s, capi.I32, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                  n, 2)
        assert capi.device_error(s, clear=True) & capi.ERR_BIT_TIMEOUT
    finally:
        capi.call("a3b_set_wait_timeout_ns", 1_000_000_000)
    # the context is still usable and the next scan on the same stream is exact
    algo.exclusive_scan(out, x)
    assert (_h(out) == np.arange(n)).all()
    assert capi.device_error(s, clear=True) == 0
