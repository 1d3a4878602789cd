"""GPU: alpaka3's own algorithm tests (scan.cpp / reduce.cpp / transformReduce.cpp / transform.cpp / concurrent.cpp /
iota.cpp pins, BabelStream dot) through alpaka3's public onHost API on a CUDA queue with the alpaka3_b200 binding:
every call runs on the C ABI or on a B200 engine compiled with the test's functors, none on alpaka3's CUDA backend."""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cpp", "_build", "test_alpaka_backend")


def test_alpaka_api_through_binding(cuda):
    if not os.path.exists(BIN):
        pytest.skip("binding test binary not built (it is compiled where the alpaka3 headers are available)")
    p = subprocess.run([BIN], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-4000:] + p.stderr[-2000:]
    m = re.search(r"PASS routed=(\d+) engine=(\d+) forwarded=(\d+)", p.stdout)
    assert m, p.stdout
    routed, engine, forwarded = int(m.group(1)), int(m.group(2)), int(m.group(3))
    # nothing runs on alpaka3's own CUDA backend
    assert forwarded == 0, p.stdout
    # C ABI: 4 sizes x 8 scan variants, 6 extents x std::plus reduce, iota into one buffer and fill;
    # element-wise engine: 6 extents x 4 transforms (std::minus, std::plus, ScalarFunc, up-cast) and the large one;
    # SIMD engine: 6 extents x (ScalarFunc min / max reduce, generator reduce, 3 transforms with StencilFunc or an
    # accelerator, 6 transformReduce pins, 2 concurrent pins, iota into two buffers), the dot, the cube, x*|x| and
    # 4 cross stencils
    assert engine >= 6 * (3 + 3 + 6 + 2 + 1) + 3 + 4, p.stdout
    assert routed >= engine + 4 * 8 + 6 + 6 * 4 + 1, p.stdout
    m = re.search(r"iota/fill routed=(\d+)", p.stdout)
    assert m and int(m.group(1)) >= 3 * 6, p.stdout
