"""The allocation-free LNAMD entry point against the workspace entry point.

``musc_b200_lnamd_noalloc`` serves callers that cannot allocate device memory
(a plug-in that may only use the tensors its host hands it, a service that
forbids allocation after start-up, a foreign-language caller without a CUDA
allocator): its scratch is a static device array inside the library.  This
test calls it through the C ABI twice in a row -- with different batches, so
the second call runs on the scratch the first one left behind -- and checks
each result against ``musc_b200_lnamd`` with a caller-provided workspace.  It
lives in its own file, named to be collected last, and needs no state from the
other tests.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(tokens: torch.Tensor, radii, outs, l2_normalize: bool) -> None:
    from musc_b200 import _lib
    b, length, c = tokens.shape
    dtype = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}[tokens.dtype]
    radii_arr = (ctypes.c_int * len(radii))(*radii)
    out_arr = (ctypes.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
    stream = ctypes.c_void_p(torch.cuda.current_stream(tokens.device).cuda_stream)
    st = _lib.lib().musc_b200_lnamd_noalloc(ctypes.c_void_p(tokens.data_ptr()), dtype, b, length, c,
                                            len(radii), radii_arr, out_arr, (length - 1) * c, c,
                                            int(l2_normalize), stream)
    _lib.check(st, 'musc_b200_lnamd_noalloc')


def test_noalloc_lnamd_matches_workspace_entry_point(cuda_device):
    from musc_b200 import ops
    gen = torch.Generator().manual_seed(2024)
    radii = (1, 3, 5)
    batches = [(torch.randn(5, 1370, 128, generator=gen) * 3.0 + 0.7, True),
               (torch.randn(3, 1370, 64, generator=gen).to(torch.bfloat16), False)]
    for tokens, l2 in batches:  # two calls in a row on the shared scratch
        tokens = tokens.to(cuda_device)
        want = ops.lnamd(tokens, radii, l2_normalize=l2)
        got = [torch.full_like(w, float('nan')) for w in want]
        _noalloc(tokens, radii, got, l2)
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            torch.testing.assert_close(g, w, rtol=1e-5, atol=2e-5)


def test_noalloc_lnamd_fp16_and_the_image_limit(cuda_device):
    """fp16 tokens, and one call at exactly the 2048-image limit (a 4 x 4 patch grid,
    C = 64), so the last scratch slots are written and read; each against the
    workspace entry point, twice in a row."""
    from musc_b200 import ops
    gen = torch.Generator().manual_seed(77)
    radii = (1, 3, 5)
    batches = [((torch.randn(4, 1370, 96, generator=gen) * 2.0 - 0.3).to(torch.float16), True),
               (torch.randn(2048, 1 + 16, 64, generator=gen) * 1.5 + 0.2, True),
               ((torch.randn(2048, 1 + 16, 64, generator=gen) + 1.0).to(torch.float16), False)]
    for tokens, l2 in batches:
        tokens = tokens.to(cuda_device)
        want = ops.lnamd(tokens, radii, l2_normalize=l2)
        got = [torch.full_like(w, float('nan')) for w in want]
        _noalloc(tokens, radii, got, l2)
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            torch.testing.assert_close(g, w, rtol=1e-5, atol=2e-5)


def test_noalloc_rejects_batches_beyond_the_scratch(cuda_device):
    from musc_b200 import _lib
    radii = (ctypes.c_int * 1)(3)
    outs = (ctypes.c_void_p * 1)(1024)
    st = _lib.lib().musc_b200_lnamd_noalloc(ctypes.c_void_p(1024), _lib.F32, 2049, 1370, 64, 1, radii,
                                            outs, 1369 * 64, 64, 1, None)
    assert st == _lib.ERR_INVALID and '2048' in _lib.last_error()
