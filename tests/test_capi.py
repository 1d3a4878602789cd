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


def test_early_start_guard_host_bookkeeping_without_gpu():
    """The reductions' early-start guard (host only): off by default; once enabled, a call reading the output of any
    reduction started early since the last fully ordered launch is launched fully ordered (which clears the history),
    repeated outputs are remembered once, and a history past 64 outputs forces one ordered launch."""
    from alpaka3_b200 import capi
    L = capi.lib()
    s = ctypes.c_void_p(0x5000)  # stands for a stream; the hooks never pass it to CUDA
    x, y = 0x10000000, 0x20000000
    o = [0x30000000 + 256 * k for k in range(80)]
    flag = ctypes.c_int(-1)

    def probe(in0, out, in1=None, nbytes=4096):
        capi.call("a3b_debug_early_start_probe", 7, s, ctypes.c_void_p(in0), ctypes.c_void_p(in1) if in1 else None,
                  nbytes, ctypes.c_void_p(out), ctypes.byref(flag))
        return flag.value

    assert probe(x, o[0]) == 0  # not enabled: ordered
    capi.call("a3b_debug_early_start_enable", 7, s, 1)
    try:
        assert probe(x, o[0]) == 1            # A
        assert probe(y, o[1]) == 1            # B, unrelated
        assert probe(o[0], o[2], nbytes=256) == 0  # C reads A's output: ordered, history cleared
        assert probe(o[0], o[3], nbytes=256) == 1  # A completed before C started
        assert probe(x, o[4], in1=o[3] - 8, nbytes=16) == 0  # second input overlapping an early output
        for _ in range(100):                  # one repeated output: remembered once
            assert probe(x, o[5]) == 1
        for k in range(6, 68):                # with o[4] and o[5]: 64 distinct outputs in the history now
            assert probe(x, o[k]) == 1
        assert probe(x, o[70]) == 0           # past the limit: ordered
        assert probe(x, o[71]) == 1
    finally:
        capi.call("a3b_debug_early_start_enable", 7, s, 0)
    assert probe(x, o[0]) == 0
