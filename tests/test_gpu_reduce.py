"""GPU parity: transformReduce / reduce / dot against the reference pins and the compensated fp64 oracle."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _val(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()[0]


def test_reduce_iota_pins(cuda):
    """test/unit/algorithm/reduce.cpp:135-152: int iota over the reference's extents, plus/min/max."""
    from alpaka3_b200 import algo
    g = json.load(open(os.path.join(GOLDEN, "reduce_iota.json")))
    out = torch.empty(1, dtype=torch.int32, device=cuda)
    for key, want in g.items():
        ext = [int(v) for v in key.split("x")]
        x = torch.arange(int(np.prod(ext)), dtype=torch.int32, device=cuda).reshape(ext)
        for op, v in want.items():
            algo.reduce(None, out, op, x)
            assert int(_val(out)) == v, (key, op)


@pytest.mark.parametrize("n", [0, 1, 3, 31, 33, 4097, 100003, 1 << 22])
def test_sumsq_f32_vs_fp64(cuda, port, n):
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    if n:
        algo.random_f32(x, SEED, -1.0, 1.0)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    algo.transform_reduce(0.0, out, "plus", "square", x)
    exact = port.sumsq(port.gen_f32(n, -1.0, 1.0)) if n else 0.0
    got = float(_val(out))
    if n == 0:
        assert got == 0.0
    else:
        assert abs(got - exact) / exact <= 1e-5


def test_sumsq_golden_input(cuda, port):
    from alpaka3_b200 import algo
    g = json.load(open(os.path.join(GOLDEN, "sumsq.json")))
    x = torch.from_numpy(port.gen_f32(g["n"], -1.0, 1.0, seed=g["seed"])).to(cuda)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    algo.transform_reduce(0.0, out, "plus", "square", x)
    got = float(_val(out))
    assert abs(got - g["ref_fp32"]) / g["ref_fp32"] <= 1e-5


@pytest.mark.parametrize("n", [5, 1 << 16, (1 << 21) + 3])
def test_dot_f64(cuda, port, n):
    from alpaka3_b200 import algo
    rng = np.random.default_rng(7)
    A, B = rng.uniform(-1, 1, n), rng.uniform(-1, 1, n)
    out = torch.empty(1, dtype=torch.float64, device=cuda)
    algo.transform_reduce(0.0, out, "plus", "product", torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda))
    exact = port.dot(A, B)
    assert abs(float(_val(out)) - exact) <= 1e-12 * np.abs(A * B).sum()


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64, torch.uint32])
@pytest.mark.parametrize("op", ["plus", "min", "max"])
def test_integer_reduce_bitexact(cuda, port, dtype, op):
    from alpaka3_b200 import algo
    n = 1000003
    x = torch.empty(n, dtype=torch.int32, device=cuda)
    algo.random_u32(x, 99)  # full 32-bit range: the plus overflows and wraps
    xh = x.cpu().numpy().view(np.uint32)
    if dtype == torch.int64:
        xh = xh.astype(np.int64) * 3 - (1 << 31)
        x = torch.from_numpy(xh).to(cuda)
    elif dtype == torch.int32:
        xh = xh.view(np.int32)
    else:
        x = x.view(torch.uint32)
    out = torch.empty(1, dtype=dtype, device=cuda)
    algo.reduce(None, out, op, x)
    got = out.cpu().numpy()[0]
    assert got == port.reduce_int(op, xh)


def test_float_min_max_and_f64_sum(cuda):
    from alpaka3_b200 import algo
    x = torch.randn(300007, dtype=torch.float64, device=cuda)
    out = torch.empty(1, dtype=torch.float64, device=cuda)
    algo.reduce(None, out, "min", x)
    assert _val(out) == x.min().item()
    algo.reduce(None, out, "max", x)
    assert _val(out) == x.max().item()
    algo.reduce(0.0, out, "plus", x)
    h = x.cpu().numpy()
    assert abs(_val(out) - np.sum(h.astype(np.longdouble))) <= 1e-12 * np.abs(h).sum()


def test_pitched_2d_reduce(cuda):
    from alpaka3_b200 import algo
    full = torch.arange(37 * 130, dtype=torch.int32, device=cuda).reshape(37, 130)
    view = full[:, 3:120]  # rows 520 bytes apart, row start offset 12 bytes
    out = torch.empty(1, dtype=torch.int32, device=cuda)
    for op in ("plus", "min", "max"):
        algo.reduce(None, out, op, view)
        want = {"plus": view.sum(), "min": view.min(), "max": view.max()}[op].item()
        assert int(_val(out)) == want
    view2 = full[:, 0:128]  # aligned rows, packed path
    algo.reduce(None, out, "plus", view2)
    assert int(_val(out)) == view2.sum().item()


def test_deterministic_bits(cuda):
    from alpaka3_b200 import algo
    x = torch.randn(1 << 22, dtype=torch.float32, device=cuda)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    vals = set()
    for _ in range(5):
        algo.transform_reduce(0.0, out, "plus", "square", x)
        vals.add(out.cpu().numpy().tobytes())
    assert len(vals) == 1


def test_partial_is_unrounded(cuda, port):
    from alpaka3_b200 import algo
    x = torch.from_numpy(port.gen_f32(1 << 20, -1.0, 1.0)).to(cuda)
    p = algo.transform_reduce_partial("plus", "square", x)
    assert p.dtype == torch.float64
    exact = port.sumsq(x.cpu().numpy())
    assert abs(p.item() - exact) / exact < 1e-9


def test_fused_reduce_one_rank_back_to_back_and_chained(cuda, port):
    """The fused reduce + all-reduce on a one-rank peer group: consecutive calls overlap on the stream (the next call
    reads its input while the previous one finishes), so repeated calls must give the same bits, and a call whose
    input starts with the previous call's output must see that output (it is launched without the early start)."""
    from alpaka3_b200 import algo, dist as adist
    from oracle.oracle import SEED
    n = (1 << 24) + 7
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    algo.random_f32(x, SEED, -1.0, 1.0)
    want = port.sumsq(port.gen_f32(n, -1.0, 1.0))
    g = adist.PeerGroup()
    algo.set_early_start(True)
    try:
        outs = [torch.empty(1, dtype=torch.float32, device=cuda) for _ in range(8)]
        for o in outs:
            g.transform_reduce(0.0, "plus", "square", x, out=o)
        vals = [float(o.item()) for o in outs]
        assert all(v == vals[0] for v in vals)
        assert abs(vals[0] - want) / want <= 1e-5
        # chain: buf[0] receives a sum, the next call reduces buf (identity), whose other elements are 0
        buf = torch.zeros(64, dtype=torch.float32, device=cuda)
        total = torch.empty(1, dtype=torch.float32, device=cuda)
        for _ in range(4):
            g.transform_reduce(0.0, "plus", "square", x, out=buf[0:1])
            g.transform_reduce(0.0, "plus", "identity", buf, out=total)
            torch.cuda.synchronize()
            assert float(total.item()) == float(buf[0].item()) == vals[0]
    finally:
        algo.set_early_start(False)
        g.close()


def test_plain_reduce_back_to_back_and_chained(cuda, port):
    """Consecutive transformReduce calls on a stream overlap (the next call reads its input while the previous one
    combines its partials): repeated calls give the same bits, and a call whose input starts with the previous call's
    output sees that output, for the dense and the pitched kernel."""
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    n = (1 << 24) + 7
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    algo.random_f32(x, SEED, -1.0, 1.0)
    want = port.sumsq(port.gen_f32(n, -1.0, 1.0))
    algo.set_early_start(True)
    try:
        _plain_chained(algo, x, want, cuda)
    finally:
        algo.set_early_start(False)


def _plain_chained(algo, x, want, cuda):
    outs = [torch.empty(1, dtype=torch.float32, device=cuda) for _ in range(8)]
    for o in outs:
        algo.transform_reduce(0.0, o, "plus", "square", x)
    vals = [float(o.item()) for o in outs]
    assert all(v == vals[0] for v in vals) and abs(vals[0] - want) / want <= 1e-5
    buf = torch.zeros(64, dtype=torch.float32, device=cuda)
    grid = torch.zeros((4, 40), dtype=torch.float32, device=cuda)  # pitched rows of 32 columns
    total = torch.empty(1, dtype=torch.float32, device=cuda)
    for _ in range(4):
        algo.transform_reduce(0.0, buf[0:1], "plus", "square", x)
        algo.transform_reduce(0.0, total, "plus", "identity", buf)
        torch.cuda.synchronize()
        assert float(total.item()) == float(buf[0].item()) == vals[0]
        algo.transform_reduce(0.0, grid[1, 3:4], "plus", "square", x)
        algo.reduce(0.0, total, "plus", grid[:, :32])
        torch.cuda.synchronize()
        assert float(total.item()) == vals[0]


def test_early_start_three_call_chain(cuda, port):
    """A writes buf[0], an unrelated call B (early start) follows, then C reduces buf: C must see A's output although
    A may still run while B starts (the guard remembers every early-started call since the last ordered launch)."""
    from alpaka3_b200 import algo
    from oracle.oracle import SEED
    n = (1 << 24) + 7
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    algo.random_f32(x, SEED, -1.0, 1.0)
    ref = torch.empty(1, dtype=torch.float32, device=cuda)
    algo.transform_reduce(0.0, ref, "plus", "square", x)
    torch.cuda.synchronize()
    want = float(ref.item())
    buf = torch.zeros(64, dtype=torch.float32, device=cuda)
    other = torch.empty(1, dtype=torch.float32, device=cuda)
    total = torch.empty(1, dtype=torch.float32, device=cuda)
    algo.set_early_start(True)
    try:
        for _ in range(6):
            algo.transform_reduce(0.0, buf[0:1], "plus", "square", x)   # A
            algo.transform_reduce(0.0, other, "plus", "square", x)      # B: input x, not A's output
            algo.transform_reduce(0.0, total, "plus", "identity", buf)  # C: reads A's output
            torch.cuda.synchronize()
            assert float(total.item()) == float(buf[0].item()) == want
            assert float(other.item()) == want
    finally:
        algo.set_early_start(False)


def test_early_start_history_overflow_then_dependent(cuda):
    """More than 64 early-started calls (the guard's history limit), then a call reading the output of one of them."""
    from alpaka3_b200 import algo
    n = (1 << 20) + 3
    x = torch.rand(n, dtype=torch.float32, device=cuda) * 2 - 1
    ref = torch.empty(1, dtype=torch.float32, device=cuda)
    algo.transform_reduce(0.0, ref, "plus", "square", x)
    torch.cuda.synchronize()
    want = float(ref.item())
    outs = torch.zeros(100, dtype=torch.float32, device=cuda)
    total = torch.empty(1, dtype=torch.float32, device=cuda)
    algo.set_early_start(True)
    try:
        for k in range(100):
            algo.transform_reduce(0.0, outs[k:k + 1], "plus", "square", x)
        algo.transform_reduce(0.0, total, "plus", "identity", outs)
        torch.cuda.synchronize()
        assert (outs.cpu() == want).all()
        assert abs(float(total.item()) - 100 * want) <= 1e-5 * 100 * want
    finally:
        algo.set_early_start(False)


def test_early_start_off_by_default_is_ordered(cuda):
    """Without a3b_set_early_start the reductions are plain launches: a torch kernel writing the input just before
    the call is complete before the call reads it (here trivially, but the default must stay ordered)."""
    from alpaka3_b200 import algo
    x = torch.empty((1 << 22) + 5, dtype=torch.float32, device=cuda)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    for v in (1.0, 2.0, 3.0):
        x.fill_(v)
        algo.transform_reduce(0.0, out, "plus", "identity", x)
        torch.cuda.synchronize()
        assert float(out.item()) == v * x.numel()
