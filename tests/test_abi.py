"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/voltattn.h declares, and its host-only entry points behave."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "voltattn.h")).read()
    return sorted(set(re.findall(r"VA_API\s+[\w\s\*]+?\b(va_\w+)\s*\(", txt)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ["va_decode", "va_quantize", "va_probe_ceiling", "va_combine_partials", "va_workspace_bytes",
              "va_status_string", "va_decode_gqa", "va_decode_partial"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    import voltattn_b200 as va
    lib = va.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_format_names_and_sizes():
    import voltattn_b200 as va
    names = ["f16", "f16+", "q8", "q8+", "q4", "q4+", "q3+"]  # src/voltattn.cu:677-686
    assert [va.fmt_name(i) for i in range(7)] == names
    for i, n in enumerate(names):
        assert va.Fmt.parse(n) == i
    with pytest.raises(ValueError):
        va.Fmt.parse("q5")
    n = 32 * 16384 * 128
    assert va.payload_bytes("f16+", n) == 2 * n
    assert va.payload_bytes("q8+", n) == n
    assert va.payload_bytes("q4+", n) == n // 2
    assert va.payload_bytes("q3+", n) == 3 * n // 8
    assert [va.lib().va_fmt_bits(i) for i in range(7)] == [16, 16, 8, 8, 4, 4, 3]


def test_workspace_layout():
    import voltattn_b200 as va
    for H, D, S in [(32, 128, 37), (8, 64, 1), (40, 128, 2)]:
        slots = H * S * (D + 2) * 4
        wb = va.workspace_bytes(H, D, S)
        assert wb >= slots + H * 4 and wb % 256 == 0
    assert va.workspace_bytes(0, 128, 1) == 0


def test_argument_errors_without_gpu():
    """Invalid arguments are rejected before any CUDA call."""
    import voltattn_b200 as va
    lib = va.lib()
    b = va.VaBufs(16, 16, 16, 16, 16, 16)
    ws, wb = C.c_void_p(256), 1 << 20
    assert lib.va_decode(99, C.byref(b), 1, 1, 128, 1, ws, wb, None) == 1       # bad format
    assert lib.va_decode(1, C.byref(b), 1, 1, 96, 1, ws, wb, None) == 5         # D unsupported
    assert lib.va_decode(1, C.byref(b), 0, 1, 128, 1, ws, wb, None) == 1        # H < 1
    assert lib.va_decode(1, C.byref(b), 1, 0, 128, 1, ws, wb, None) == 1        # L < 1
    assert lib.va_decode(1, C.byref(b), 1, 8, 128, 70000, ws, wb, None) == 1    # S too large
    nb = va.VaBufs(16, 16, None, None, 16, 16)
    assert lib.va_decode(3, C.byref(nb), 1, 8, 128, 1, ws, wb, None) == 1       # q8+ without scales
    mb = va.VaBufs(24, 16, 16, 16, 16, 16)
    assert lib.va_decode(3, C.byref(mb), 1, 8, 128, 1, ws, wb, None) == 2       # misaligned K
    assert lib.va_decode(3, C.byref(b), 1, 8, 128, 1, ws, 16, None) == 3        # workspace too small
    assert lib.va_decode(3, C.byref(b), 1, 8, 128, 1, None, wb, None) == 3      # no workspace
    assert lib.va_quantize(5, 16, 16, 16, 1, 1, 128, None) == 1
    assert lib.va_quantize(8, 16, 16, 16, 1, 1, 80, None) == 5
    assert lib.va_quantize(8, 24, 16, 16, 1, 1, 128, None) == 2
    for st in range(8):
        assert lib.va_status_string(st)
    assert lib.va_combine_partials(None, 1, 1, 1, 128, 16, None) == 1
