"""Build recipe of the CUDA library ``alpaka3_b200/lib/libalpaka3_b200.so`` (sm_100a only).

Each ``csrc/*.cu`` is compiled by nvcc for ``-gencode arch=compute_100a,code=sm_100a`` and the objects are linked
into one shared library with the CUDA runtime linked statically, so the library needs only the driver at run time.
The build is in-tree: the ``.so`` sits next to the package and is found by ``alpaka3_b200.capi``.
"""
import concurrent.futures
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJDIR = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libalpaka3_b200.so")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")) + [__file__]


def compile_one(src, verbose=False, extra=()):
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()) or extra:
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
    return obj


def build(verbose=False, ptxas_verbose=False):
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ("-Xptxas", "-v") if ptxas_verbose else ()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, verbose, extra), srcs))
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB + ".tmp", *objs]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
