"""Block softmax attention oracle (numpy) -- test infrastructure only.

Restates the attention of one ViT block as the reference runs it:
``nn.MultiheadAttention(d, h)`` called from
``models/backbone/open_clip/transformer.py:221-234`` computes, per batch item
and head, ``softmax(q k^T / sqrt(d_head)) v`` over the full 1370-token
sequence (no mask on the scoring path); the reference's softmax kernel does the
row softmax in fp32 (``models/modules/_attention_gpu.py:41-81``).  This oracle
evaluates it in float64.
"""
from __future__ import annotations

import numpy as np


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """``q, k, v``: ``(BH, L, d)`` -> ``(BH, L, d)`` float64."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    s = np.einsum('bld,bmd->blm', q, k) * scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum('blm,bmd->bld', p, v)
