"""RsCIN oracle (numpy) -- test infrastructure only.

Restates ``models/modules/_RsCIN.py`` of the reference, the image-score
refinement MuSc applies after scoring (``models/musc.py:287-296``):

* ``rscin`` (``_RsCIN.py:22-31``): with no class tokens, or with 0 in
  ``k_list``, the scores come back unchanged; otherwise the scores are
  min-max normalised in float64, the class-token similarity matrix
  ``W = T T^T`` is formed in float32 and handed to ``mmo``;
* ``mmo`` (``_RsCIN.py:5-20``): for each k, every row of W keeps its k largest
  entries (the reference zeroes the N-k smallest, ``:7-11``), is divided by
  its sum (``:13-15``) and averages the normalised scores (``:16-17``); the
  result is the float32 mean over the k values (``:19``).
"""
from __future__ import annotations

from typing import Sequence

import numpy as np


def mmo(w: np.ndarray, score: np.ndarray, k_list: Sequence[int]) -> np.ndarray:
    w = np.asarray(w, dtype=np.float32)
    score = np.asarray(score, dtype=np.float32)
    n = w.shape[0]
    rows = np.arange(n)[:, None]
    out = []
    for k in k_list:
        keep = np.argsort(-w, axis=1, kind='stable')[:, :k]
        mask = np.zeros_like(w)
        mask[rows, keep] = w[rows, keep]
        d = np.float32(1.0) / mask.sum(axis=1, dtype=np.float32)
        p = (d[:, None] * mask).astype(np.float32)
        out.append((p @ score).astype(np.float32))
    return np.stack(out, -1).mean(-1, dtype=np.float32)


def rscin(scores_old: np.ndarray, cls_tokens=None, k_list: Sequence[int] = (0,)) -> np.ndarray:
    if cls_tokens is None or 0 in k_list:
        return scores_old
    t = np.asarray(cls_tokens, dtype=np.float32)
    s = np.asarray(scores_old, dtype=np.float64)
    s = (s - s.min()) / (s.max() - s.min())
    return mmo((t @ t.T).astype(np.float32), s.astype(np.float32), k_list)
