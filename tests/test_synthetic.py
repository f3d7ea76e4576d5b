"""The synthetic pool that stands in for MVTec: the sigma reading of the stand-in.

The spec's generator (unit-norm prototypes + sigma * N(0, I_C), 5 % of patches replaced by
N(0, I_C)) is ambiguous about sigma: per coordinate (literal, noise norm sigma*sqrt(C)) or
per vector (sigma / sqrt(C) per coordinate, noise norm sigma).  The bench uses the literal
reading.  This check scores small pools with the numpy oracle (LNAMD r = 1, L2-normalised
bank, MSM over the 0-30 % interval) and records what each reading gives: with the per-vector
reading the off-manifold patches separate cleanly from the prototype patches; with the
literal reading the noise dominates and the separation is weak but still in the right
direction.  Anomalous patches are recovered from the token norms (~sqrt(C) versus ~1 to
sigma*sqrt(C)), so the generator's random stream is untouched.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from musc_b200.synthetic import prototype_mixture_layer
from oracle import lnamd as olnamd
from oracle import msm as omsm

N, SIDE, C = 6, 10, 64


def _scores(sigma: float):
    tok = prototype_mixture_layer(N, c=C, side=SIDE, sigma=sigma, generator=torch.Generator().manual_seed(3))
    body = tok[:, 1:].numpy()
    norms = np.linalg.norm(body, axis=-1)
    anomalous = norms > 0.5 * math.sqrt(C)
    z = olnamd.bank(tok.numpy(), 1)
    scores = omsm.msm(z, 0.0, 0.3)
    return scores, anomalous


def test_per_vector_sigma_separates_anomalies():
    scores, anomalous = _scores(0.1 / math.sqrt(C))
    assert 0 < anomalous.sum() < anomalous.size
    normal, anom = scores[~anomalous], scores[anomalous]
    assert anom.min() > normal.max()            # every anomaly above every normal patch
    assert anom.mean() > 3 * normal.mean()


def test_literal_sigma_separation_is_weak_but_ordered():
    scores, anomalous = _scores(0.1)
    normal, anom = scores[~anomalous], scores[anomalous]
    assert anom.mean() > normal.mean()
    assert anom.mean() < 2 * normal.mean()      # the per-coordinate noise dominates the prototypes
