"""ctypes binding of the C-ABI library ``libmusc_b200.so`` (see include/musc_b200.h).

The shared library is built in-tree by ``musc-gpu_b200/build.py`` and loaded
from this package directory.  There is no fallback: if the library is missing
every entry point raises.  Status codes map onto the reference's exception
types -- contract violations raise ``ValueError`` (as
``models/modules/_MSM_gpu.py:702-711`` does), CUDA and driver failures raise
``RuntimeError`` (as ``models/modules/_cuda_runtime.py:47-55`` does).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name('libmusc_b200.so')

OK, ERR_INVALID, ERR_CUDA, ERR_DEVICE, ERR_WORKSPACE, ERR_TIMEOUT = range(6)
F32, F16, BF16 = 0, 1, 2
BICUBIC, BILINEAR = 0, 1

_vp, _ll, _int, _sz, _f = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_size_t, ctypes.c_float

# name -> (restype, argtypes); the exact set declared in include/musc_b200.h.
SIGNATURES = {
    'musc_b200_abi_version': (_int, []),
    'musc_b200_last_error': (ctypes.c_char_p, []),
    'musc_b200_take_device_error': (_int, [ctypes.POINTER(_int)]),
    'musc_b200_selftest_wait': (_int, [_ll, _int, _vp]),
    'musc_b200_lnamd_workspace_bytes': (_sz, [_int]),
    'musc_b200_lnamd': (_int, [_vp, _int, _int, _int, _int, _int, ctypes.POINTER(_int),
                               ctypes.POINTER(_vp), _ll, _ll, _int, _vp, _sz, _vp]),
    'musc_b200_lnamd_noalloc': (_int, [_vp, _int, _int, _int, _int, _int, ctypes.POINTER(_int),
                                       ctypes.POINTER(_vp), _ll, _ll, _int, _vp]),
    'musc_b200_lnamd_super_fast': (_int, [_vp, _int, _int, _int, _int, _int, _vp, _ll, _ll, _int,
                                          _vp, _sz, _vp]),
    'musc_b200_bank_bytes': (_sz, [_ll, _int]),
    'musc_b200_prep_bank': (_int, [_vp, _ll, _int, _vp, _sz, _vp]),
    'musc_b200_center_stats_bytes': (_sz, [_int]),
    'musc_b200_center_stats': (_int, [_vp, _ll, _int, _vp, _vp, _sz, _vp]),
    'musc_b200_prep_bank_centered': (_int, [_vp, _ll, _int, _vp, _int, _ll, _vp, _sz, _vp]),
    'musc_b200_nearest': (_int, [_vp, _ll, _ll, _vp, _ll, _int, _int, _vp, _vp]),
    'musc_b200_nearest_pool_bytes': (_sz, [_ll, _int, _ll]),
    'musc_b200_nearest_pool': (_int, [_vp, _ll, _ll, _int, _int, _int, _int, _ll, _int, _vp, _vp]),
    'musc_b200_bank_layout': (_int, [_ll, _int, ctypes.POINTER(_sz)]),
    'musc_b200_screen_pool': (_int, [_vp, _ll, _ll, _int, _int, _int, _int, _ll, _int, _vp, _vp, _vp, _vp]),
    'musc_b200_refine_bytes': (_sz, [_int, _ll, _int]),
    'musc_b200_refine_min_bytes': (_sz, [_int, _ll, _int]),
    'musc_b200_refine_launches': (_int, [_int, _ll, _int, _sz]),
    'musc_b200_refine': (_int, [_vp, _ll, _ll, _int, _int, _ll, _ll, _int, _vp, _vp, _int, _ll, _ll, _vp, _vp,
                                _sz, _vp]),
    'musc_b200_trimmed_mean': (_int, [_vp, _ll, _int, _int, _int, _vp, _vp]),
    'musc_b200_msm_workspace_bytes': (_sz, [_int, _int, _int]),
    'musc_b200_msm': (_int, [_vp, _int, _int, _int, _int, _int, _vp, _vp, _sz, _vp]),
    'musc_b200_attention_fwd': (_int, [_vp, _vp, _vp, _vp, _int, _int, _int, _int, _int, _ll, _ll, _f, _vp]),
    'musc_b200_add_layernorm': (_int, [_vp, _vp, _int, _vp, _vp, ctypes.c_float, _vp, _int, _ll, _int, _vp]),
    'musc_b200_preprocess_workspace_bytes': (_sz, [_int, _int, _int, _int, _int]),
    'musc_b200_preprocess_images': (_int, [_vp, _int, _int, _int, _ll, _int, _int, _int,
                                           ctypes.POINTER(_f), ctypes.POINTER(_f), _int, _vp, _vp, _sz, _vp]),
    'musc_b200_rscin': (_int, [_vp, _int, _int, _vp, _int, ctypes.POINTER(_int), _vp, _vp]),
    'musc_b200_score_pool_bytes': (_sz, [_int, _int, _int, _int]),
    'musc_b200_score_pool': (_int, [ctypes.POINTER(_vp), _int, _int, _int, _int, _int, _int,
                                    ctypes.POINTER(_int), ctypes.c_double, ctypes.c_double, _int, _vp, _vp,
                                    _vp, _vp, _sz, _vp]),
    'musc_b200_score_maps': (_int, [_vp, _int, _int, _int, _int, _int, _vp, _vp, _vp, _vp]),
    'musc_b200_ipc_get': (_int, [_vp, _vp, ctypes.POINTER(_sz)]),
    'musc_b200_ipc_open': (_int, [_vp, _sz, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    'musc_b200_ipc_close': (_int, [_vp]),
    'musc_b200_stream_signal': (_int, [_vp, ctypes.c_uint, _vp]),
    'musc_b200_stream_wait': (_int, [_vp, ctypes.c_uint, _vp]),
    'musc_b200_copy_async': (_int, [_vp, _vp, _sz, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class LibraryMissing(RuntimeError):
    """The sm_100a library has not been built; there is no CPU fallback."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise LibraryMissing(
                        f'{LIB_PATH} is missing: build it with `python musc-gpu_b200/build.py` '
                        '(the b200 backend has no CPU fallback)')
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().musc_b200_last_error()
    return msg.decode() if msg else ''


def check(status: int, what: str) -> None:
    """Raise the reference's exception type for a non-zero status."""
    if status == OK:
        return
    msg = f'{what}: {last_error()}'
    if status in (ERR_INVALID, ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def take_device_error() -> int:
    code = _int(0)
    check(lib().musc_b200_take_device_error(ctypes.byref(code)), 'take_device_error')
    return code.value
