"""CPU: the C-ABI library loads and exports every entry point the public header declares (no GPU calls)."""
import ctypes
import os
import re

from conftest import ROOT


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(a3b_[a-z0-9_]+)\s*\(", src))
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert {"a3b_transform_reduce", "a3b_scan", "a3b_babelstream", "a3b_heat_step",
            "a3b_nbody_update_velocities"} <= names


def test_library_exports_every_declared_symbol():
    from alpaka3_b200 import capi
    lib = ctypes.CDLL(capi.LIB_PATH)
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    from alpaka3_b200 import capi
    assert _declared() == set(capi.SIGNATURES)


def test_version_and_scan_buffer_size():
    from alpaka3_b200 import capi
    L = capi.lib()
    assert L.a3b_version() == 100
    # 64-byte header + one 8-byte status word per 32 value bits per 36 KB tile (9216 x 4-byte or 4608 x 8-byte
    # elements), rounded up to 256 bytes
    tiles32 = -(-(1 << 30) // 9216)
    assert L.a3b_scan_buffer_size(capi.U32, 1 << 30) == 64 + -(-tiles32 * 8 // 256) * 256
    tiles64 = -(-(1 << 28) // 4608)
    assert L.a3b_scan_buffer_size(capi.U64, 1 << 28) == 64 + -(-tiles64 * 16 // 256) * 256
    assert L.a3b_scan_buffer_size(capi.U32, 1) == 64 + 256
    assert L.a3b_scan_buffer_size(99, 10) == 0


def test_invalid_arguments_rejected_without_gpu():
    from alpaka3_b200 import capi
    L = capi.lib()
    rc = L.a3b_babelstream(None, capi.TRIAD, capi.I32, None, None, None, 10, 0.4, None)
    assert rc == capi.ERR_INVALID
    assert "null" in capi.last_error()


def test_halo_mailbox_layout_and_argument_checks_without_gpu():
    """heat halo mailbox: 16 KB of step flags (2 sides x 2 parities x 1024 column blocks) + 4 ghost rows of cols + 2
    doubles padded to 256 bytes; steps and publications on a missing or unconnected mailbox are rejected up front."""
    from alpaka3_b200 import capi
    L = capi.lib()
    for cols in (1, 1000, 32768):
        row = -(-(cols + 2) // 32) * 32
        assert L.a3b_halo_bytes(cols) == 2 * 2 * 1024 * 4 + 4 * row * 8
    assert L.a3b_heat_step_halo(None, None, None, None, 10, 10, 12, 0.2, 0.2) == capi.ERR_INVALID
    assert "halo" in capi.last_error()
    assert L.a3b_heat_halo_publish(None, None, None, 10, 10, 12) == capi.ERR_INVALID
    assert L.a3b_halo_destroy(None) == capi.OK
