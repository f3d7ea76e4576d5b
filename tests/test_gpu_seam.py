"""The ``b200`` seam driven the way the reference's ``MuSc.make_category_data`` drives it.

``models/musc.py:227-296`` is replayed step for step, with the reference's order and
arguments, using only the objects the patched ``make_category_data`` takes from
``musc_b200.backend``:

* ``aggregation = encode_image.new_aggregation()`` (``:148-151``);
* per radius an ``LNAMD``-shaped layer object (``r``, ``patch_maker.stride``,
  ``LNA.output_dim``, ``LNA.preprocessing_modules``; ``models/modules/_LNAMD.py:64-70``)
  and per batch of 4 images ``aggregation(LNAMD_r, patch_tokens, return_cpu=False)``
  under autocast, then ``features /= features.norm(dim=-1, keepdim=True)`` and the
  per-layer split into ``Z_layers`` (``:229-243``);
* per layer ``scoring(Z=Z, device=..., topmin_min=0, topmin_max=0.3)`` (``:248-256``);
* the layer and radius means, ``F.interpolate(..., mode='bilinear', align_corners=True)``
  to 518, ``.cpu()``, the per-image max (``:257-288``), ``aggregation.clear()`` (``:274-275``);
* ``RsCIN(ac_score, class_tokens, k_list=[1, 2, 3])`` (``:287-296``).

Inputs: the config-1 pool (N = 16, 4 layers x r{1,3,5}); the maps and image scores are
checked against the reference's golden outputs (2e-5 relative), RsCIN against the oracle.
"""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import golden
from oracle import rscin as orscin

pytestmark = pytest.mark.gpu
RTOL = 2e-5


def _lnamd_layer(r: int, feature_dim: int, feature_layer: list[int]):
    """The attributes of ``LNAMD(device, r=r, feature_dim=..., feature_layer=...)`` the seam reads."""
    return SimpleNamespace(r=r, patch_maker=SimpleNamespace(patch_size=r, stride=1),
                           LNA=SimpleNamespace(output_dim=feature_dim,
                                               preprocessing_modules=[object() for _ in feature_layer]))


def test_make_category_data_scoring_half_through_the_seam(cuda_device):
    from musc_b200 import backend
    from musc_b200.synthetic import prototype_mixture
    g = golden('pool16')
    n, batch = int(g['n']), 4
    features_list = [6, 12, 18, 24]                 # models/musc.py:61 for layers 5/11/17/23
    r_list, image_size = [1, 3, 5], 518
    layers = prototype_mixture(n, n_layers=4, c=1024, side=37, seed=int(g['seed']))
    # patch_tokens_list: one entry per encoder batch, a list of 4 (B, 1370, 1024) tensors
    patch_tokens_list = [[t[i:i + batch] for t in layers] for i in range(0, n, batch)]

    encoding = backend.encode_image
    scoring = backend.MSM
    aggregation = encoding.new_aggregation()
    encoding.begin_inference()

    feature_dim = patch_tokens_list[0][0].shape[-1]
    anomaly_maps_r = torch.empty(0, dtype=torch.float64, device=cuda_device)
    for r in r_list:
        LNAMD_r = _lnamd_layer(r, feature_dim, features_list)
        Z_layers = {}
        for im in range(len(patch_tokens_list)):
            patch_tokens = [p.to(cuda_device) for p in patch_tokens_list[im]]
            with torch.no_grad(), torch.autocast('cuda'):
                features = aggregation(LNAMD_r, patch_tokens, return_cpu=False)
                features /= features.norm(dim=-1, keepdim=True)
                for l in range(len(features_list)):
                    Z_layers.setdefault(str(l), []).append(features[:, :, l, :])
        anomaly_maps_l = torch.empty(0, dtype=torch.float64, device=cuda_device)
        for l in Z_layers.keys():
            Z = torch.cat(Z_layers[l], dim=0).to(cuda_device)
            anomaly_maps_msm = scoring(Z=Z, device=cuda_device, topmin_min=0, topmin_max=0.3)
            anomaly_maps_l = torch.cat((anomaly_maps_l, anomaly_maps_msm.unsqueeze(0)), dim=0)
        anomaly_maps_l = torch.mean(anomaly_maps_l, 0)
        anomaly_maps_r = torch.cat((anomaly_maps_r, anomaly_maps_l.unsqueeze(0)), dim=0)
    anomaly_maps_iter = torch.mean(anomaly_maps_r, 0).to(cuda_device)
    B, L = anomaly_maps_iter.shape
    H = int(np.sqrt(L))
    maps_small = anomaly_maps_iter.view(B, H, H).cpu().numpy()
    anomaly_maps = F.interpolate(anomaly_maps_iter.view(B, 1, H, H), size=image_size, mode='bilinear',
                                 align_corners=True).cpu()
    aggregation.clear()
    anomaly_maps = anomaly_maps.numpy()
    ac_score = np.array(anomaly_maps).reshape(B, -1).max(-1)

    np.testing.assert_allclose(maps_small, g['maps'], rtol=RTOL, atol=0)
    np.testing.assert_allclose(ac_score, g['image_max'], rtol=RTOL, atol=0)
    stats = backend.research_diagnostics()
    assert stats['msm_calls'] == 12 and stats['aggregation_calls'] == 12

    # RsCIN with the class tokens the encoder loop collects (unit-norm, 768-d)
    gen = torch.Generator().manual_seed(3)
    cls = torch.randn(n, 768, generator=gen)
    class_tokens = list((cls / cls.norm(dim=-1, keepdim=True)).numpy())
    scores_cls = backend.RsCIN(ac_score, class_tokens, k_list=[1, 2, 3], device=cuda_device)
    want = orscin.rscin(ac_score, np.stack(class_tokens), [1, 2, 3])
    assert scores_cls.dtype == np.float32
    np.testing.assert_allclose(scores_cls, want, rtol=2e-6, atol=0)
    assert backend.RsCIN(ac_score, class_tokens, k_list=[0]) is ac_score
