"""GPU numerics of the fused tcgen05 attention kernel.

Reference: a plain PyTorch fp32 evaluation of ``softmax(q k^T * scale) v`` on the same bf16
inputs (and the numpy oracle for one small case).  Tolerance: the kernel rounds P and the
output to the 16-bit input type (bf16: 2^-9 relative), so outputs are compared at 1e-2
relative + 2e-3 absolute.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, heads, scale):
    b, length, width = q.shape
    d = width // heads
    qf, kf, vf = (t.float().reshape(b, length, heads, d).transpose(1, 2) for t in (q, k, v))
    p = torch.softmax(qf @ kf.transpose(-1, -2) * scale, dim=-1)
    return (p @ vf).transpose(1, 2).reshape(b, length, width)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('b,length,heads', [(2, 200, 2), (1, 1, 1), (3, 128, 1), (1, 129, 3),
                                            (2, 1370, 16)])
def test_attention_matches_fp32_reference(cuda_device, b, length, heads, dtype):
    from musc_b200 import ops
    g = torch.Generator(device=cuda_device).manual_seed(b * 1000 + length + heads)
    width = heads * 64
    qkv = torch.randn(b, length, 3 * width, generator=g, device=cuda_device).to(dtype)
    q, k, v = qkv[..., :width], qkv[..., width:2 * width], qkv[..., 2 * width:]
    out = ops.attention(q, k, v, heads)
    want = _ref(q, k, v, heads, 64 ** -0.5)
    torch.testing.assert_close(out.float(), want, rtol=1e-2, atol=2e-3)


def test_attention_peaked_logits(cuda_device):
    """Large logits (near one-hot rows) exercise the running-max rescaling across tiles."""
    from musc_b200 import ops
    g = torch.Generator(device=cuda_device).manual_seed(7)
    b, length, heads, width = 2, 700, 4, 256
    q = (torch.randn(b, length, width, generator=g, device=cuda_device) * 4).to(torch.bfloat16)
    k = (torch.randn(b, length, width, generator=g, device=cuda_device) * 4).to(torch.bfloat16)
    v = torch.randn(b, length, width, generator=g, device=cuda_device).to(torch.bfloat16)
    out = ops.attention(q, k, v, heads)
    torch.testing.assert_close(out.float(), _ref(q, k, v, heads, 0.125), rtol=1e-2, atol=3e-3)


def test_attention_against_oracle(cuda_device):
    from musc_b200 import ops
    from oracle import attention as oattn
    g = torch.Generator(device=cuda_device).manual_seed(3)
    b, length, heads = 1, 300, 2
    q, k, v = (torch.randn(b, length, heads * 64, generator=g, device=cuda_device).to(torch.bfloat16)
               for _ in range(3))
    out = ops.attention(q, k, v, heads).float().cpu().numpy()
    qh, kh, vh = (t.float().cpu().numpy().reshape(length, heads, 64).transpose(1, 0, 2) for t in (q, k, v))
    want = oattn.attention(qh, kh, vh, 0.125).transpose(1, 0, 2).reshape(1, length, heads * 64)
    np.testing.assert_allclose(out, want, rtol=1e-2, atol=2e-3)
