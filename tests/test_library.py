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
    assert lib.musc_b200_abi_version() == 3
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


def test_score_pool_and_rscin_validate_before_any_cuda_call():
    """The one-call pool entry point and RsCIN reject contract violations on the host."""
    from musc_b200 import _lib
    lib = _lib.lib()
    vp = ctypes.c_void_p
    # workspace of the one-call pool path: the sum of its parts, and 0 for nonsense sizes
    n, c = 16, 1024
    need = lib.musc_b200_score_pool_bytes(n, 1370, c, 3)
    assert need >= lib.musc_b200_bank_bytes(n * 1369, c) + 3 * n * 1369 * c * 4
    assert lib.musc_b200_score_pool_bytes(0, 1370, c, 3) == 0
    assert lib.musc_b200_score_pool_bytes(n, 1, c, 3) == 0
    toks = (vp * 4)(*[1024] * 4)
    radii = (ctypes.c_int * 3)(1, 3, 5)
    out = vp(1 << 20)
    ws = vp(1 << 30)

    def pool(n_images, tokens_per_image, n_radii, lo, hi, ws_bytes, workspace=ws):
        return lib.musc_b200_score_pool(toks, 0, n_images, tokens_per_image, c, 4, n_radii, radii, lo, hi, 518,
                                        out, out, out, workspace, ws_bytes, None)

    assert pool(n, 1371, 3, 0.0, 0.3, need) == _lib.ERR_INVALID and 'square' in _lib.last_error()
    assert pool(n, 1370, 4, 0.0, 0.3, need) == _lib.ERR_INVALID and 'radii' in _lib.last_error()
    assert pool(n, 1370, 3, 0.5, 0.5, need) == _lib.ERR_INVALID and 'trimmed ranks' in _lib.last_error()
    assert pool(1, 1370, 3, 0.0, 0.3, need) == _lib.ERR_INVALID and 'trimmed ranks' in _lib.last_error()
    assert pool(n, 1370, 3, 0.0, 0.3, need - 1) == _lib.ERR_WORKSPACE
    assert pool(n, 1370, 3, 0.0, 0.3, need, vp((1 << 30) + 16)) == _lib.ERR_INVALID
    assert 'aligned' in _lib.last_error()
    # RsCIN: sizes and k values
    ks = (ctypes.c_int * 9)(*range(1, 10))
    st = lib.musc_b200_rscin(vp(1024), 10, 768, vp(2048), 9, ks, vp(4096), None)
    assert st == _lib.ERR_INVALID and 'at most 8' in _lib.last_error()
    st = lib.musc_b200_rscin(vp(1024), 0, 768, vp(2048), 3, ks, vp(4096), None)
    assert st == _lib.ERR_INVALID
    st = lib.musc_b200_rscin(vp(1024), 10, 768, None, 3, ks, vp(4096), None)
    assert st == _lib.ERR_INVALID and 'null' in _lib.last_error()


def test_rscin_passthrough_rule_without_a_device():
    """backend.RsCIN keeps the reference's passthrough (_RsCIN.py:23-24): no class tokens or a
    0 in k_list return the very input, with no device work."""
    import numpy as np
    from musc_b200 import backend
    s = np.array([1.0, 2.0, 3.0])
    assert backend.RsCIN(s) is s
    assert backend.RsCIN(s, None, k_list=[1, 2, 3]) is s
    assert backend.RsCIN(s, [np.ones(4)] * 3, k_list=[1, 0]) is s
