"""GPU: alpaka3's own algorithm tests (scan.cpp / reduce.cpp / transform.cpp pins, BabelStream dot) through alpaka3's
public onHost API on a CUDA queue with the alpaka3_b200 binding: covered calls go to the C ABI or the element-wise
engine, the others to alpaka3's CUDA backend."""
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
    m = re.search(r"PASS routed=(\d+) forwarded=(\d+)", p.stdout)
    assert m, p.stdout
    routed, forwarded = int(m.group(1)), int(m.group(2))
    # routed: 4 sizes x 8 scan variants, 6 extents x 3 reduce ops, the dot, 6 extents x 4 transforms (std::minus,
    # std::plus, ScalarFunc, up-cast) and the large in-place transform; forwarded to alpaka3's own backend: the 6
    # generator reductions, the unrecognised transformReduce and 6 extents x 3 transforms (StencilFunc and the two
    # functors that take an accelerator)
    assert routed >= 4 * 8 + 6 * 3 + 1 + 6 * 4 + 1, p.stdout
    assert forwarded >= 6 + 1 + 6 * 3, p.stdout
    # iota into one dense buffer and fill go to the C ABI (at least the 1-D extent is dense); iota into two buffers
    # stays on alpaka3's kernel
    m = re.search(r"iota/fill routed=(\d+)", p.stdout)
    assert m and int(m.group(1)) >= 2, p.stdout
