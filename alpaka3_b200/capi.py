"""ctypes binding of the C ABI declared in ``include/alpaka3_b200.h`` (and the test hooks of
``include/alpaka3_b200_testing.h``).

This module only loads ``lib/libalpaka3_b200.so`` and declares the signatures; it has no fallback. If the library is
missing, :func:`lib` raises :class:`LibraryNotBuilt` (run ``python -m alpaka3_b200.build`` or
``__graft_entry__.build()``).
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# A3B_LIBRARY selects another build of the same library (e.g. a tuning variant); default: the in-tree build
LIB_PATH = os.environ.get("A3B_LIBRARY") or os.path.join(_HERE, "lib", "libalpaka3_b200.so")

# status codes
OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_TIMEOUT, ERR_NOMEM, ERR_TOO_LARGE = range(7)
# dtypes
I32, U32, I64, U64, F32, F64 = range(6)
# reduce / transform functors
PLUS, MIN, MAX = range(3)
IDENTITY, SQUARE, PRODUCT = range(3)
# BabelStream kernels
INIT, COPY, MUL, ADD, TRIAD, NSTREAM = range(6)
# element-wise maps
MAP_COPY, MAP_SCALE, MAP_ADD, MAP_MUL, MAP_AXPY, MAP_SQUARE = range(6)

ERR_BIT_TIMEOUT = 1

_P = ctypes.c_void_p
_U64 = ctypes.c_uint64
_I = ctypes.c_int
_D = ctypes.c_double
_F = ctypes.c_float

# name -> argtypes (all return int unless listed in _RESTYPES)
SIGNATURES = {
    "a3b_version": [],
    "a3b_last_error": [],
    "a3b_device_count": [_P],
    "a3b_device_info_get": [_I, _P],
    "a3b_malloc_async": [_P, ctypes.c_size_t, _P],
    "a3b_free_async": [_P, _P],
    "a3b_memcpy_async": [_P, _P, ctypes.c_size_t, _P],
    "a3b_stream_synchronize": [_P],
    "a3b_get_device_error": [_P, _P, _I],
    "a3b_set_wait_timeout_ns": [_U64],
    "a3b_engine_scratch": [_P, ctypes.c_size_t, _P],
    "a3b_babelstream": [_P, _I, _I, _P, _P, _P, _U64, _D, _P],
    "a3b_transform": [_P, _I, _I, _P, _P, _P, _U64, _D],
    "a3b_fill": [_P, _I, _P, _U64, _P],
    "a3b_iota": [_P, _I, _P, _U64, _P],
    "a3b_nbody_update_positions": [_P, _P, _P, _P, _P, _P, _P, _U64, _F],
    "a3b_random_u32": [_P, _P, _U64, _U64, _U64, _I],
    "a3b_random_u64": [_P, _P, _U64, _U64, _U64],
    "a3b_random_f32": [_P, _P, _U64, _U64, _U64, _F, _F],
    "a3b_transform_reduce": [_P, _I, _I, _I, _P, _P, _U64, _P, _P],
    "a3b_transform_reduce_partial": [_P, _I, _I, _I, _P, _P, _U64, _P, _P],
    "a3b_transform_reduce_noalloc": [_P, _I, _I, _I, _P, _P, _U64, _P, _P],
    "a3b_reduce_2d": [_P, _I, _I, _P, _U64, _U64, _U64, _P, _P],
    "a3b_set_early_start": [_P, _I],
    "a3b_ipc_handle_size": [],
    "a3b_peer_group_create": [_I, _I, _P, _P],
    "a3b_peer_group_connect": [_P, _P],
    "a3b_peer_group_destroy": [_P],
    "a3b_transform_reduce_allranks": [_P, _P, _I, _I, _I, _P, _P, _U64, _P, _P],
    "a3b_reduce_lower_ranks": [_P, _P, _I, _P, _U64, _P],
    "a3b_scan_buffer_size": [_I, _U64],
    "a3b_scan": [_P, _I, _I, _P, _P, _U64, _P, _P, ctypes.c_size_t],
    "a3b_nbody_update_velocities": [_P, _P, _P, _P, _P, _U64, _U64, _U64, _P, _P, _P, _F, _F],
    "a3b_nbody_step": [_P, _P, _P, _P, _P, _U64, _U64, _U64, _P, _P, _P, _F, _F],
    "a3b_haccmk_step10": [_P, _P, _P, _P, _P, _I, _I, _F, _F, _F, _P, _P, _P],
    "a3b_heat_step": [_P, _P, _P, _U64, _U64, _U64, _U64, _U64, _D, _D],
    "a3b_heat_init": [_P, _P, _U64, _U64, _U64, _U64, _U64, _D, _D],
    "a3b_heat_exact": [_P, _P, _U64, _U64, _U64, _U64, _U64, _D, _D, _D, _I],
    "a3b_halo_bytes": [_U64],
    "a3b_halo_create": [_I, _I, _U64, _P, _P],
    "a3b_halo_connect": [_P, _P],
    "a3b_halo_destroy": [_P],
    "a3b_heat_halo_publish": [_P, _P, _P, _U64, _U64, _U64],
    "a3b_heat_step_halo": [_P, _P, _P, _P, _U64, _U64, _U64, _D, _D],
    # test hooks (include/alpaka3_b200_testing.h)
    "a3b_scan_debug_stall": [_P, _I, _P, _P, _U64, _U64],
    "a3b_debug_early_start_enable": [_I, _P, _I],
    "a3b_debug_early_start_probe": [_I, _P, _P, _P, _U64, _P, _P],
}
_RESTYPES = {"a3b_last_error": ctypes.c_char_p, "a3b_scan_buffer_size": ctypes.c_size_t,
             "a3b_ipc_handle_size": ctypes.c_size_t, "a3b_halo_bytes": ctypes.c_size_t}


class LibraryNotBuilt(RuntimeError):
    pass


class A3BError(RuntimeError):
    def __init__(self, status, message, call):
        super().__init__(f"{call} failed with status {status}: {message}")
        self.status = status


_lib = None


def lib():
    """Load the CUDA library (once). Raises LibraryNotBuilt when the .so is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryNotBuilt(f"{LIB_PATH} is missing: build the CUDA extension first")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = L
    return _lib


def check(rc, call="a3b call"):
    if rc != OK:
        msg = lib().a3b_last_error()
        raise A3BError(rc, msg.decode() if msg else "", call)
    return rc


def call(name, *args):
    """Invoke ``name`` and raise A3BError on a non-zero status."""
    return check(getattr(lib(), name)(*args), name)


def last_error():
    m = lib().a3b_last_error()
    return m.decode() if m else ""


class DeviceInfo(ctypes.Structure):
    _fields_ = [("ordinal", ctypes.c_int), ("sm_count", ctypes.c_int), ("cc_major", ctypes.c_int),
                ("cc_minor", ctypes.c_int), ("global_mem_bytes", ctypes.c_uint64), ("l2_bytes", ctypes.c_uint64),
                ("max_threads_per_block", ctypes.c_int), ("warp_size", ctypes.c_int), ("name", ctypes.c_char * 128)]


def device_info(ordinal=0):
    info = DeviceInfo()
    call("a3b_device_info_get", ordinal, ctypes.byref(info))
    return info


def device_error(stream, clear=True):
    bits = ctypes.c_uint32(0)
    call("a3b_get_device_error", stream, ctypes.byref(bits), 1 if clear else 0)
    return bits.value


def exported_symbols():
    return list(SIGNATURES)
