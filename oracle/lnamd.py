"""LNAMD aggregation oracle (numpy) -- test infrastructure only.

Restates the reference's neighbourhood aggregation:

* ``LNAMD._embed`` (``models/modules/_LNAMD.py:72-129``): drop the CLS token
  (``:78``), view the tokens as ``(B, C, side, side)`` (``:79-83``), apply a
  fresh ``LayerNorm([C, side, side])`` -- weight 1, bias 0, eps 1e-5, biased
  variance over the whole image (``:84-85``) -- then the r x r ``Unfold`` with
  padding ``(r-1)/2`` followed by the channel mean (``:16-35, 54-61``).  The
  reference's own GPU path shows this equals
  ``avg_pool2d(r, stride 1, padding r//2, count_include_pad=True)``
  (``models/modules/_encoder_gpu.py:33-37``): zero padding, divisor r^2.
* ``features /= features.norm(dim=-1)`` (``models/musc.py:238``).
* The super-fast profile (``models/modules/_super_fast.py:17-27``): r = 3, then
  ``adaptive_avg_pool2d`` from 37x37 to 28x28 in float32 (``:23-26``); the L2
  normalisation of ``musc.py:238`` follows the pooling.
"""
from __future__ import annotations

import math

import numpy as np


def layer_norm_image(tokens: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """``(B, 1+P, C)`` tokens -> ``(B, C, side, side)`` float32 LayerNorm output."""
    x = np.asarray(tokens, dtype=np.float32)[:, 1:, :]
    b, p, c = x.shape
    side = math.isqrt(p)
    if side * side != p:
        raise ValueError('token count minus CLS must be a square')
    x = x.reshape(b, side, side, c).transpose(0, 3, 1, 2).astype(np.float64)
    mean = x.mean(axis=(1, 2, 3), keepdims=True)
    var = ((x - mean) ** 2).mean(axis=(1, 2, 3), keepdims=True)
    return ((x - mean) / np.sqrt(var + eps)).astype(np.float32)


def box_mean(spatial: np.ndarray, r: int) -> np.ndarray:
    """Zero-padded r x r mean, divisor r^2, stride 1 (``_encoder_gpu.py:35-37``)."""
    if r == 1:
        return spatial
    h = r // 2
    b, c, s, _ = spatial.shape
    padded = np.zeros((b, c, s + 2 * h, s + 2 * h), dtype=np.float64)
    padded[:, :, h:h + s, h:h + s] = spatial
    out = np.zeros((b, c, s, s), dtype=np.float64)
    for dy in range(r):
        for dx in range(r):
            out += padded[:, :, dy:dy + s, dx:dx + s]
    return (out / (r * r)).astype(np.float32)


def to_patches(spatial: np.ndarray) -> np.ndarray:
    """``(B, C, s, s)`` -> ``(B, s*s, C)`` (row-major patch order, ``_LNAMD.py:126``)."""
    b, c, s, _ = spatial.shape
    return spatial.reshape(b, c, s * s).transpose(0, 2, 1)


def l2_normalize(features: np.ndarray) -> np.ndarray:
    """``features / ||features||`` over the channel axis (``models/musc.py:238``)."""
    f = np.asarray(features, dtype=np.float32)
    return (f / np.linalg.norm(f.astype(np.float64), axis=-1, keepdims=True)).astype(np.float32)


def lnamd(tokens: np.ndarray, r: int) -> np.ndarray:
    """``(B, 1+P, C)`` -> ``(B, P, C)`` LayerNorm + neighbourhood mean (no L2 norm)."""
    return to_patches(box_mean(layer_norm_image(tokens), r))


def adaptive_avg_pool(spatial: np.ndarray, out_side: int) -> np.ndarray:
    """``adaptive_avg_pool2d``: window ``[floor(i*S/O), ceil((i+1)*S/O))`` per axis."""
    b, c, s, _ = spatial.shape
    starts = [(i * s) // out_side for i in range(out_side)]
    ends = [-(-((i + 1) * s) // out_side) for i in range(out_side)]
    x = spatial.astype(np.float64)
    out = np.empty((b, c, out_side, out_side), dtype=np.float64)
    for i in range(out_side):
        for j in range(out_side):
            out[:, :, i, j] = x[:, :, starts[i]:ends[i], starts[j]:ends[j]].mean(axis=(2, 3))
    return out.astype(np.float32)


def lnamd_super_fast(tokens: np.ndarray, out_side: int = 28) -> np.ndarray:
    """r=3 LNAMD then adaptive pooling to ``out_side``^2 patches (``_super_fast.py:17-27``)."""
    return to_patches(adaptive_avg_pool(box_mean(layer_norm_image(tokens), 3), out_side))


def bank(tokens: np.ndarray, r: int) -> np.ndarray:
    """One MSM input bank ``Z`` = L2-normalised LNAMD features ``(B, P, C)``."""
    return l2_normalize(lnamd(tokens, r))
