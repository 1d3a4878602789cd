"""Builds tests/cpp/_build/test_alpaka_backend: alpaka3's own algorithm tests (re-expressed without Catch2) compiled
against the reference's headers with the alpaka3_b200 binding included, linked to libalpaka3_b200.so. Built only where
the reference tree exists; the binary travels with the repository snapshot (the tests never read the reference)."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "_build", "test_alpaka_backend")
REFERENCE_ROOT = os.environ.get("ALPAKA_REFERENCE_ROOT")  # the alpaka3 source tree; no default


def build(force=False, reference_root=None):
    root = reference_root or REFERENCE_ROOT
    src = os.path.join(HERE, "test_alpaka_backend.cpp")
    hdr = os.path.join(ROOT, "include", "alpaka3_b200", "alpaka_backend.hpp")
    lib = os.path.join(ROOT, "alpaka3_b200", "lib", "libalpaka3_b200.so")
    if not root or not os.path.isdir(os.path.join(root, "include", "alpaka")):
        return OUT if os.path.exists(OUT) else None
    if not force and os.path.exists(OUT) and all(os.path.getmtime(OUT) >= os.path.getmtime(p) for p in (src, hdr, lib)):
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = ["nvcc", "-x", "cu", "-std=c++20", "-O2", "--expt-relaxed-constexpr", "--extended-lambda",
           # the benchmark's SIMD for-each kernel runs on the B200 SIMD engine (alpaka3_b200::IsSimdForEachKernel)
           '-DALPAKA3_B200_SIMD_FOR_EACH_KERNELS="SimdForEachKernel"',
           "-gencode", "arch=compute_100a,code=sm_100a", "-I" + os.path.join(root, "include"),
           "-I" + os.path.join(ROOT, "include"), src, "-o", OUT + ".tmp", "-L" + os.path.dirname(lib), "-lalpaka3_b200",
           "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN/../../../alpaka3_b200/lib"]
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    roots = [a for a in sys.argv[1:] if not a.startswith("--")]
    print(build("--force" in sys.argv, roots[0] if roots else None))
