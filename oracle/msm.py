"""MSM mutual scoring oracle (numpy) -- test infrastructure only.

Restates ``models/modules/_MSM.py`` of the reference:

* ``compute_scores_fast`` (``_MSM.py:10-30``): for query image ``i`` the
  Euclidean distance from each of its patches to every patch of the other
  ``N-1`` images (``torch.cdist``, ``_MSM.py:16``), the minimum over each
  reference image's patches (``_MSM.py:17``), then the mean of ranks
  ``[k_min, k_max)`` of those ``N-1`` minima (``_MSM.py:19-30``);
* ``MSM`` (``_MSM.py:53-59``): the loop over query images, stacked to an
  ``(N, P)`` float64 matrix.

``torch.cdist`` in its default mode evaluates large Euclidean distances with
the matrix-product identity ``|x|^2 + |y|^2 - 2 x.y`` clamped at 1e-30 before
the square root; this file uses the same identity in float32 so its rounding
behaviour matches the reference.
"""
from __future__ import annotations

import numpy as np


def trimmed_ranks(n_images: int, topmin_min: float = 0, topmin_max: float = 0.3) -> tuple[int, int]:
    """Rank interval ``[k_min, k_max)`` exactly as ``_MSM.py:20-28`` derives it."""
    k_max, k_min = topmin_max, topmin_min
    m = n_images - 1
    if k_max < 1:
        k_max = int(m * k_max)
    if k_min < 1:
        k_min = int(m * k_min)
    if k_max < k_min:
        k_max, k_min = k_min, k_max
    return int(k_min), int(k_max)


def nearest_minima(Z: np.ndarray, i: int, chunk: int | None = None) -> np.ndarray:
    """``(P, N-1)`` float32 minima of query image ``i`` (``_MSM.py:14-17``).

    ``chunk``: evaluate the reference images in groups of this many (same arithmetic per
    (query, reference) pair; bounds the ``P x chunk*P`` distance block for large pools).
    """
    Z = np.asarray(Z, dtype=np.float32)
    n, p, c = Z.shape
    q = Z[i]
    others = [j for j in range(n) if j != i]
    step = len(others) if chunk is None else max(1, int(chunk))
    qn = np.einsum('ij,ij->i', q, q, dtype=np.float32)
    out = []
    for s in range(0, len(others), step):
        ids = others[s:s + step]
        ref = Z[ids].reshape(-1, c)
        rn = np.einsum('ij,ij->i', ref, ref, dtype=np.float32)
        d2 = qn[:, None] + rn[None, :] - np.float32(2) * (q @ ref.T)
        d = np.sqrt(np.maximum(d2, np.float32(1e-30)))
        out.append(d.reshape(p, len(ids), p).min(axis=2))
    return np.concatenate(out, axis=1)


def interval_average(minima: np.ndarray, k_min: int, k_max: int) -> np.ndarray:
    """Mean of ranks ``[k_min, k_max)`` per row, float32 then float64 (``_MSM.py:27-30, 57``)."""
    vals = np.sort(minima.astype(np.float32), axis=1)[:, k_min:k_max]
    return vals.mean(axis=1, dtype=np.float32).astype(np.float64)


def msm(Z: np.ndarray, topmin_min: float = 0, topmin_max: float = 0.3) -> np.ndarray:
    """``(N, P)`` float64 anomaly scores (``_MSM.py:53-59``)."""
    Z = np.asarray(Z, dtype=np.float32)
    n = Z.shape[0]
    k_min, k_max = trimmed_ranks(n, topmin_min, topmin_max)
    return np.stack([interval_average(nearest_minima(Z, i), k_min, k_max) for i in range(n)])


def nearest_table(Z: np.ndarray) -> np.ndarray:
    """``(N*P, N)`` float32 minima with the self image set to FLT_MAX.

    This is the intermediate table of the reference's GPU backend
    (``models/modules/_MSM_gpu.py:721``, self slot ``:202``), assembled from
    the ``original`` arithmetic above.
    """
    Z = np.asarray(Z, dtype=np.float32)
    n, p, _ = Z.shape
    out = np.full((n * p, n), np.finfo(np.float32).max, dtype=np.float32)
    for i in range(n):
        m = nearest_minima(Z, i)
        cols = [j for j in range(n) if j != i]
        out[i * p:(i + 1) * p][:, cols] = m
    return out
