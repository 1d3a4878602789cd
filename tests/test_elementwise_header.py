"""CPU: the header-only element-wise engine (include/alpaka3_b200/elementwise.cuh) compiles on its own, without
alpaka3, for sm_100a, used directly as a library user would (nvcc cross-compiles without a GPU; the engine itself runs
on the GPU in the alpaka3 binding test)."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SOURCE = r"""
#include <alpaka3_b200/elementwise.cuh>

struct Axpy
{
    float s;
    __device__ float operator()(float x, float y) const { return s * x + y; }
};

struct ToDouble
{
    __device__ double operator()(int v) const { return 0.5 * v; }
};

cudaError_t run(cudaStream_t stream, float* out, float const* x, float const* y, double* d, int const* v, unsigned long n)
{
    cudaError_t e = alpaka3_b200::elementwise::transform(stream, out, n, Axpy{2.f}, x, y);
    if(e != cudaSuccess)
        return e;
    return alpaka3_b200::elementwise::transform(stream, d, n, ToDouble{}, v);
}
"""


def test_elementwise_header_compiles_standalone():
    nvcc = shutil.which("nvcc")
    if nvcc is None:
        pytest.skip("nvcc not available")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "use_engine.cu")
        with open(src, "w") as f:
            f.write(SOURCE)
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
               "-I" + os.path.join(ROOT, "include"), "-c", src, "-o", os.path.join(d, "use_engine.o")]
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
        assert p.returncode == 0, p.stderr[-3000:]
