"""GPU: the reference GPU comparator (alpaka3's own CUDA backend on the benchmark workloads, oracle/_ref/ref_cuda_bench)
runs on small sizes and every workload passes its own result check. The comparator is measurement infrastructure; the
library under test is not involved."""
import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
BIN = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "ref_cuda_bench")


def test_reference_cuda_backend_small():
    if not os.path.exists(BIN):
        pytest.skip("oracle/_ref/ref_cuda_bench not built (needs the reference tree at build time)")
    res = subprocess.run([BIN, "--small", "--steps", "2", "--warmup", "1"], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr
    lines = [json.loads(l) for l in res.stdout.splitlines() if l.startswith("{")]
    names = {l["workload"] for l in lines}
    assert names == {"sumsq", "babelstream_copy", "babelstream_mul", "babelstream_add", "babelstream_triad",
                     "babelstream_dot", "scan_i32", "scan_u64", "heat", "nbody"}
    for l in lines:
        assert l["check"] == "ok", l
        assert l["value"] > 0
