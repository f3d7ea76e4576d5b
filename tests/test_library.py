"""The C-ABI library loads and exports every entry point its header declares (no GPU calls)."""
from __future__ import annotations

import ctypes
import re

from conftest import REPO


def header_symbols() -> set[str]:
    names = set()
    for h in (REPO / 'include').glob('*.h'):
        text = re.sub(r'/\*.*?\*/', '', h.read_text(), flags=re.S)
        names |= set(re.findall(r'\b(musc_b200_\w+)\s*\(', text))
    return names


def test_header_declares_the_abi():
    names = header_symbols()
    assert {'musc_b200_lnamd', 'musc_b200_nearest', 'musc_b200_trimmed_mean', 'musc_b200_msm',
            'musc_b200_score_maps', 'musc_b200_prep_bank'} <= names


def test_library_exports_every_declared_symbol():
    from musc_b200 import _lib
    handle = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(header_symbols()) if not hasattr(handle, n)]
    assert not missing, f'declared in include/*.h but not exported: {missing}'


def test_binding_covers_header_exactly():
    from musc_b200 import _lib
    assert set(_lib.SIGNATURES) == header_symbols()


def test_host_only_queries():
    """Size queries and argument validation run without a device."""
    from musc_b200 import _lib
    lib = _lib.lib()
    assert lib.musc_b200_abi_version() == 1
    assert lib.musc_b200_lnamd_workspace_bytes(0) == 0
    assert lib.musc_b200_lnamd_workspace_bytes(4) == 4 * 8 * 2 * 8
    assert lib.musc_b200_bank_bytes(1369, 1024) >= 1369 * 1024 * 4
    assert lib.musc_b200_bank_bytes(1369, 1024) % 1024 == 0
    assert lib.musc_b200_msm_workspace_bytes(16, 1369, 1024) > 16 * 1369 * 16 * 4
    # contract violations are reported before any CUDA call
    st = lib.musc_b200_trimmed_mean(None, 10, 5, 0, 1, None, None)
    assert st == _lib.ERR_INVALID and 'null' in _lib.last_error()
    st = lib.musc_b200_msm(ctypes.c_void_p(16), 1, 10, 8, 0, 1, ctypes.c_void_p(16), ctypes.c_void_p(1024),
                           1 << 30, None)
    assert st == _lib.ERR_INVALID and 'N>=2' in _lib.last_error()
    st = lib.musc_b200_msm(ctypes.c_void_p(16), 10, 10, 8, 3, 3, ctypes.c_void_p(16), ctypes.c_void_p(1024),
                           1 << 30, None)
    assert st == _lib.ERR_INVALID and 'trimmed ranks' in _lib.last_error()
    radii = (ctypes.c_int * 1)(2)
    outs = (ctypes.c_void_p * 1)(1024)
    st = lib.musc_b200_lnamd(ctypes.c_void_p(1024), 0, 2, 1370, 64, 1, radii, outs, 1369 * 64, 64, 1,
                             ctypes.c_void_p(1024), 1024, None)
    assert st == _lib.ERR_INVALID and 'radius' in _lib.last_error()
    st = lib.musc_b200_lnamd(ctypes.c_void_p(1024), 0, 2, 1371, 64, 1, radii, outs, 1369 * 64, 64, 1,
                             ctypes.c_void_p(1024), 1024, None)
    assert st == _lib.ERR_INVALID and 'square' in _lib.last_error()
