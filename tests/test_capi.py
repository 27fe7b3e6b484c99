"""The C-ABI library loads on the host and exports every entry point include/psgd_b200.h declares (no GPU)."""
import ctypes
import os
import re

from psgd_pro_b200 import _capi

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "psgd_b200.h")


def declared_symbols():
    src = open(HDR).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|void|unsigned long long)\s+(psgd_\w+)\s*\(", src, re.M)))


def test_header_declares_entry_points():
    assert len(declared_symbols()) >= 6


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_capi.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    bound = {name for name, _, _ in _capi.SIGNATURES}
    assert set(declared_symbols()) <= bound


def test_spec_struct_size_matches_header():
    # PsgdGemmSpec: 17 pointers/long longs before M (see header order) ... checked via field offsets
    s = _capi.GemmSpec
    assert s.M.offset == 6 * 8 and s.alpha.offset == s.mode.offset + 4
    assert ctypes.sizeof(s) % 8 == 0


def test_header_constants_match_binding():
    """Work-list geometry the host encodes (row blocks, chunks) must be the one the kernels assume."""
    text = open(HDR).read()
    defs = dict(re.findall(r"#define (PSGD_\w+) (\d+)", text))
    assert int(defs["PSGD_PREP_ROWS"]) == _capi.PREP_ROWS
    assert int(defs["PSGD_ROT_ROWS"]) == _capi.ROT_ROWS
    assert int(defs["PSGD_SKEW_TILE"]) == _capi.SKEW_TILE
    assert int(defs["PSGD_TRACE_ROWS"]) == _capi.TRACE_ROWS
    assert int(defs["PSGD_FAC_SCRATCH"]) == _capi.FAC_SCRATCH
    assert int(defs["PSGD_APPLY_CHUNK"]) == _capi.APPLY_CHUNK


def test_struct_layout_matches_bindings():
    """The library's struct sizes (psgd_struct_sizes) equal the ctypes mirrors: a stale build is refused at load."""
    L = _capi.lib()
    n = L.psgd_struct_sizes(None, 0)
    sizes = (ctypes.c_longlong * n)()
    L.psgd_struct_sizes(sizes, n)
    assert list(sizes) == [ctypes.sizeof(c) for c in _capi.STRUCTS]
