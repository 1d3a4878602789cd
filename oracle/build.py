"""Build recipe for the CPU oracle (test infrastructure, never the product path).

* ``oracle/liboracle.so``     -- the plain-C restatement in ``oracle.c`` (always built).
* ``oracle/_ref/libalpaka_ref.so`` -- alpaka3's own host backend behind ``ref_harness.cpp``; built only where the
  reference tree exists (``build_ref.sh``).
* ``oracle/_ref/ref_cuda_bench`` -- alpaka3's own CUDA backend on the benchmark workloads (``ref_cuda_bench.cpp``,
  nvcc for sm_100a), the reference GPU comparator; built with it.
The built files travel with the repository snapshot; the source tree they are compiled from does not.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libalpaka_ref.so")
REF_CUDA_BENCH = os.path.join(HERE, "_ref", "ref_cuda_bench")
# where the alpaka3 source tree lies; the build script passes it explicitly (no default: without it, _ref is not built)
REFERENCE_ROOT = os.environ.get("ALPAKA_REFERENCE_ROOT")


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_oracle(force=False):
    src = os.path.join(HERE, "oracle.c")
    if force or _stale(ORACLE_SO, [src, __file__]):
        cmd = ["gcc", "-std=c11", "-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fno-math-errno", "-fPIC", "-shared",
               "-o", ORACLE_SO + ".tmp", src, "-lm"]
        subprocess.check_call(cmd)
        os.replace(ORACLE_SO + ".tmp", ORACLE_SO)
    return ORACLE_SO


def build_ref(force=False, reference_root=None):
    """Builds oracle/_ref from the alpaka3 tree at `reference_root` (or $ALPAKA_REFERENCE_ROOT); without one, or
    where it does not exist, keeps whatever was built before."""
    root = reference_root or REFERENCE_ROOT
    if not root or not os.path.isdir(os.path.join(root, "include", "alpaka")):
        return REF_SO if os.path.exists(REF_SO) else None
    srcs = [os.path.join(HERE, f) for f in ("ref_harness.cpp", "ref_ops.hpp", "ref_cuda_bench.cpp", "build_ref.sh")]
    if force or _stale(REF_SO, srcs) or _stale(REF_CUDA_BENCH, srcs):
        subprocess.check_call(["bash", os.path.join(HERE, "build_ref.sh"), root])
    return REF_SO


if __name__ == "__main__":
    force = "--force" in sys.argv
    roots = [a for a in sys.argv[1:] if not a.startswith("--")]
    print(build_oracle(force))
    print(build_ref(force, roots[0] if roots else None))
