"""Score-reduction oracle (numpy) -- test infrastructure only.

Restates ``models/musc.py:248-288`` of the reference:

* mean of the per-layer MSM maps (``:259``), then mean over radii (``:263``),
  both in float64;
* bilinear up-sampling of the ``(N, side, side)`` map to ``image_size`` with
  ``align_corners=True`` (``:269-272``), float64;
* per-image score = maximum of the up-sampled map (``:288``).
"""
from __future__ import annotations

import math

import numpy as np


def mean_maps(scores: np.ndarray) -> np.ndarray:
    """``(R, L, N, P)`` float64 -> ``(N, P)``: layer mean then radius mean."""
    s = np.asarray(scores, dtype=np.float64)
    return s.mean(axis=1).mean(axis=0)


def bilinear_align_corners(maps: np.ndarray, out_size: int) -> np.ndarray:
    """``(N, s, s)`` -> ``(N, out, out)`` bilinear, align_corners=True, float64."""
    m = np.asarray(maps, dtype=np.float64)
    n, s, _ = m.shape
    if out_size == 1:
        pos = np.zeros(1)
    else:
        pos = np.arange(out_size, dtype=np.float64) * ((s - 1) / (out_size - 1))
    i0 = np.clip(np.floor(pos).astype(np.int64), 0, s - 1)
    i1 = np.minimum(i0 + 1, s - 1)
    w = pos - i0
    rows = m[:, i0, :] * (1 - w)[None, :, None] + m[:, i1, :] * w[None, :, None]
    return rows[:, :, i0] * (1 - w)[None, None, :] + rows[:, :, i1] * w[None, None, :]


def image_scores(scores: np.ndarray, image_size: int = 518) -> tuple[np.ndarray, np.ndarray]:
    """Returns ``(maps (N, side, side), image_max (N,))`` for ``(R, L, N, P)`` scores."""
    mean = mean_maps(scores)
    n, p = mean.shape
    side = math.isqrt(p)
    maps = mean.reshape(n, side, side)
    up = bilinear_align_corners(maps, image_size)
    return maps, up.reshape(n, -1).max(axis=1)
