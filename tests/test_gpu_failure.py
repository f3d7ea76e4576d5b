"""Failure detection on the GPU without a fault: the bounded-wait path.

Every pipelined kernel in the library (the nearest-neighbour GEMM, the attention kernel)
waits on mbarriers with a time limit; when a limit expires the kernel records
MUSC_B200_ERR_TIMEOUT in the device error word, drains and returns, and the host reads the
word.  ``musc_b200_selftest_wait`` runs that exact wait on a barrier nothing arrives at, with
a 50 ms limit, so the test sees the timeout reported and the context still working after it.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_context_survives(cuda_device):
    from musc_b200 import _lib, ops
    lib = _lib.lib()
    assert _lib.take_device_error() == _lib.OK
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    _lib.check(lib.musc_b200_selftest_wait(50_000_000, 0, stream), 'selftest_wait')
    assert _lib.take_device_error() == _lib.ERR_TIMEOUT
    assert _lib.take_device_error() == _lib.OK          # reading clears it
    _lib.check(lib.musc_b200_selftest_wait(50_000_000, 1, stream), 'selftest_wait')
    assert _lib.take_device_error() == _lib.OK          # an arrival completes the wait
    z = torch.nn.functional.normalize(torch.randn(8, 49, 64, device=cuda_device), dim=-1)
    assert torch.isfinite(ops.msm(z)).all()              # the context still runs work
    assert _lib.take_device_error() == _lib.OK


def test_selftest_rejects_bad_limits():
    from musc_b200 import _lib
    assert _lib.lib().musc_b200_selftest_wait(0, 0, None) == _lib.ERR_INVALID
