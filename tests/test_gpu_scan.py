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


# The scan runs one block per SM (G = 148 on B200) over 36 KB tiles (9216 x 4-byte, 4608 x 8-byte elements) in rounds;
# a tile's aggregate is taken two rounds before its scan. These sizes sit on the edges of that structure: one tile,
# G tiles, G tiles + 1 element, more than the two-round lag, and ragged last tiles.
_G = 148


def _edge_sizes(tile):
    return [tile - 1, tile, tile + 1, _G * tile, _G * tile + 1, 3 * _G * tile + 7, 5 * _G * tile - 3]


@pytest.mark.parametrize("dtype,tile", [(torch.int32, 9216), (torch.int64, 4608)])
def test_scan_round_structure_sizes(cuda, port, dtype, tile):
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    for n in _edge_sizes(tile):
        if dtype == torch.int32:
            x = torch.empty(n, dtype=torch.int32, device=cuda)
            algo.random_u32(x, SEED, shift=28)
        else:
            x = torch.empty(n, dtype=torch.int64, device=cuda)
            algo.random_u64(x, SEED)
        h = _h(x)
        out = torch.empty_like(x)
        for incl in (False, True):
            (algo.inclusive_scan if incl else algo.exclusive_scan)(out, x)
            assert (_h(out) == port.scan(h, incl)).all(), (n, incl)


def test_scan_in_place_with_exact_buffer_multi_round(cuda, port):
    """in place over several rounds with a ragged last tile, scratch in a caller buffer of exactly
    a3b_scan_buffer_size bytes"""
    from alpaka3_b200 import algo
    n = 4 * _G * 9216 + 4097
    x = torch.randint(-1000, 1000, (n,), dtype=torch.int32, device=cuda)
    want = port.scan(_h(x), True)
    buf = torch.empty(algo.get_scan_buffer_size(torch.int32, n), dtype=torch.uint8, device=cuda)
    algo.inclusive_scan_in_place(x, buffer=buf)
    assert (_h(x) == want).all()


def test_scan_unaligned_multi_round(cuda, port):
    """4-byte offset input and output (no 16-byte packs, no TMA) over several rounds, with a carry"""
    from alpaka3_b200 import algo
    n = 3 * _G * 9216 + 11
    base = torch.randint(0, 16, (n + 1,), dtype=torch.int32, device=cuda)
    x = base[1:]
    out = torch.empty(n + 3, dtype=torch.int32, device=cuda)[3:]
    carry = torch.tensor([-5], dtype=torch.int32, device=cuda)
    algo.exclusive_scan(out, x, carry=carry)
    assert (_h(out) == port.scan(_h(x), False) - 5).all()


def test_float_scan_is_deterministic(cuda):
    """tile aggregates are combined in a fixed order, so repeated floating-point scans give identical bits"""
    from alpaka3_b200 import algo
    for dtype in (torch.float32, torch.float64):
        x = torch.rand(2 * _G * 9216 + 333, dtype=dtype, device=cuda) - 0.5
        a = torch.empty_like(x)
        b = torch.empty_like(x)
        algo.inclusive_scan(a, x)
        for _ in range(3):
            algo.inclusive_scan(b, x)
            assert torch.equal(a, b)


def test_early_started_reduce_after_scan(cuda):
    """Reductions with the early start enabled right after a scan on the same stream: one of the scan's output (out of
    place or in place) must see every element the scan wrote, one of the scan's input stays correct. int32 sums wrap,
    so the checks are bit-exact."""
    from alpaka3_b200 import algo
    n = (1 << 26) + 5
    x = torch.empty(n, dtype=torch.int32, device=cuda)
    algo.random_u32(x, 0x5EED, shift=28)
    xl = x.long()
    excl = torch.cumsum(xl, 0) - xl
    want_scan = int(((excl.sum() + (1 << 31)) % (1 << 32)) - (1 << 31))
    want_x = int(((xl.sum() + (1 << 31)) % (1 << 32)) - (1 << 31))
    del xl, excl
    y = torch.empty_like(x)
    z = torch.empty_like(x)
    s1, s2, s3 = (torch.empty(1, dtype=torch.int32, device=cuda) for _ in range(3))
    algo.set_early_start(True)
    try:
        for _ in range(4):
            algo.exclusive_scan(y, x)               # out of place
            algo.reduce(None, s1, "plus", y)        # reads the scan's output
            z.copy_(x)
            algo.exclusive_scan(z, z)               # in place
            algo.reduce(None, s2, "plus", z)        # reads the in-place output
            algo.exclusive_scan(y, x)
            algo.reduce(None, s3, "plus", x)        # the scan's input
            torch.cuda.synchronize()
            assert int(s1.item()) == want_scan
            assert int(s2.item()) == want_scan
            assert int(s3.item()) == want_x
    finally:
        algo.set_early_start(False)
