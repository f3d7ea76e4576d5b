"""The ``b200`` inference backend: a drop-in for the reference's plug-in seam.

``MuSc.make_category_data`` picks its operators by backend
(``models/musc.py:135-153``):

* ``scoring(Z=Z, device=..., topmin_min=0, topmin_max=0.3)`` -> ``(N, P)``
  float64 -- here :func:`MSM` (replacing ``models/modules/_MSM_gpu.py:701``);
* ``encoding(model, image, out_layers)`` -> ``(pooled, [tokens per layer])``
  with the optional hooks ``aggregate_features``, ``new_aggregation`` and
  ``begin_inference`` (``models/modules/_encoder_gpu.py:45-64``) -- here
  :func:`encode_image`, whose aggregation runs the LNAMD kernel.

Backend selection mirrors ``models/modules/_backend.py:5-33`` with one
difference the north star asks for: ``b200`` never falls back.  On anything
but a CUDA sm_100 device it raises instead of returning ``original``.
"""
from __future__ import annotations

import math
from copy import deepcopy

import numpy as np
import torch

from . import ops

BACKENDS = ('original', 'gpu', 'super_fast', 'b200', 'b200_super_fast')
_STATS = {'aggregation_calls': 0, 'direct_pool_calls': 0, 'msm_calls': 0, 'rscin_calls': 0}


def select_backend(requested: str, device_type: str, platform=None, device=None):
    """``(selected, fallback_reason)`` like ``_backend.select_backend`` (``_backend.py:5-14``).

    ``b200`` / ``b200_super_fast`` are returned only on an sm_100 CUDA device;
    otherwise a ``RuntimeError`` is raised (no fallback).  The reference's own
    names keep the reference's behaviour and are not served by this package.
    """
    if requested not in BACKENDS:
        raise ValueError('inference_backend must be original, gpu, super_fast, b200 or b200_super_fast')
    if requested in ('b200', 'b200_super_fast'):
        if device_type != 'cuda' or not torch.cuda.is_available():
            raise RuntimeError('inference_backend b200 requires a CUDA B200 (sm_100) device; '
                               'it has no CPU fallback')
        cap = torch.cuda.get_device_capability(device)
        if cap != (10, 0):
            raise RuntimeError(f'inference_backend b200 requires sm_100, found sm_{cap[0]}{cap[1]}')
        return requested, None
    if requested == 'original':
        return 'original', None
    if device_type != 'cuda':
        return 'original', 'CUDA is unavailable'
    import os
    if (os.name if platform is None else platform) != 'nt':
        return 'original', 'the accelerated NVRTC runtime currently supports native Windows only'
    return requested, None


def configure_backend(cfg: dict, device_type: str, platform=None) -> dict:
    """Apply the super-fast preset (layer [5], r=[3]) like ``_backend.py:17-33``."""
    requested = cfg['models'].get('inference_backend', 'original')
    if requested != 'b200_super_fast':
        return cfg
    select_backend(requested, device_type, platform)
    models, datasets = cfg['models'], cfg['datasets']
    if (models['backbone_name'] != 'ViT-L-14-336' or models['pretrained'] != 'openai'
            or datasets['img_resize'] != 518 or models['batch_size'] != 4
            or datasets['divide_num'] != 1):
        raise ValueError('super_fast requires ViT-L-14-336/openai, img_resize=518, '
                         'batch_size=4 and divide_num=1; use b200 for other configurations')
    result = deepcopy(cfg)
    result['models']['feature_layers'] = [5]
    result['models']['r_list'] = [3]
    return result


# --------------------------------------------------------------------------- scoring
def MSM(Z: torch.Tensor, device=None, topmin_min: float = 0, topmin_max: float = 0.3) -> torch.Tensor:
    """``scoring`` seam: ``(N, P, C)`` CUDA fp32 -> ``(N, P)`` float64 on ``Z.device``.

    Same contract and errors as ``models/modules/_MSM_gpu.py:701-711``, with one
    limit the reference does not have: ``N <= 1790`` (the interval average stages
    32 rows x N minima in shared memory); larger pools raise ``ValueError``.
    Asynchronous like the reference: if a device-side bounded wait expired, the
    scores are NaN; :func:`musc_b200.ops.check_device_error` reports it.
    """
    _STATS['msm_calls'] += 1
    return ops.msm(Z, topmin_min, topmin_max)


# --------------------------------------------------------------------------- RsCIN
def RsCIN(scores_old, cls_tokens=None, k_list=(0,), device=None):
    """Drop-in for ``RsCIN`` (``models/modules/_RsCIN.py:22-31``) on the GPU.

    Same arguments and passthrough rule: with ``cls_tokens`` None or a 0 in
    ``k_list`` the scores come back unchanged (the same object).  Host inputs
    (the numpy ``ac_score`` and list of class-token arrays that
    ``models/musc.py:287-296`` passes) give a host float32 array, like the
    reference; a CUDA float64 tensor gives a CUDA float64 tensor.
    """
    if cls_tokens is None or 0 in k_list:
        return scores_old
    _STATS['rscin_calls'] += 1
    if isinstance(scores_old, torch.Tensor) and scores_old.is_cuda:
        tokens = cls_tokens if isinstance(cls_tokens, torch.Tensor) else torch.as_tensor(
            np.asarray(cls_tokens, dtype=np.float32))
        return ops.rscin(scores_old.to(torch.float64), tokens.to(scores_old.device), k_list)
    dev = torch.device(device) if device is not None else torch.device('cuda', torch.cuda.current_device())
    scores = torch.as_tensor(np.asarray(scores_old, dtype=np.float64)).to(dev)
    tokens = torch.as_tensor(np.asarray(cls_tokens, dtype=np.float32)).to(dev)
    host = ops.rscin(scores, tokens, k_list).cpu().numpy().astype(np.float32)
    ops.check_device_error(dev, 'RsCIN')      # the copy above synchronised already
    return host


# --------------------------------------------------------------------------- aggregation
def _check_layer(layer, features) -> None:
    first = features[0]
    batch, length, channels = first.shape
    side = math.isqrt(length - 1)
    if side * side != length - 1:
        raise ValueError('b200 aggregation: token count must be 1 + side^2')
    if getattr(layer.patch_maker, 'stride', 1) != 1:
        raise ValueError('b200 aggregation: patch stride must be 1')
    if layer.r not in (1, 3, 5):
        raise ValueError('b200 aggregation: r must be 1, 3 or 5')
    if layer.LNA.output_dim != channels or len(features) != len(layer.LNA.preprocessing_modules):
        raise ValueError('b200 aggregation: feature_dim / feature_layer do not match the tokens')
    if any(t.shape != first.shape or t.dtype != first.dtype or t.device != first.device for t in features):
        raise ValueError('b200 aggregation: all layers must share shape, dtype and device')


def aggregate_features(layer, features, return_cpu: bool = True) -> torch.Tensor:
    """``(B, P, layers, C)`` LayerNorm + r x r mean (``models/modules/_encoder_gpu.py:14-42``).

    Unlike the reference hook there is no fallback to ``layer._embed``: a
    contract violation raises ``ValueError``.
    """
    _check_layer(layer, features)
    result = ops.lnamd_layers(list(features), layer.r, l2_normalize=False)
    _STATS['aggregation_calls'] += 1
    if layer.r != 1:
        _STATS['direct_pool_calls'] += 1
    if not return_cpu:
        return result
    host = result.cpu()
    ops.check_device_error(result.device, 'aggregation')   # the copy above synchronised already
    return host


class Aggregation:
    """Per-inference aggregation object (``_aggregation_cache.RadiusAggregationCache``).

    The LNAMD kernel recomputes the per-image LayerNorm statistics in one
    reduction pass per call, so no cross-radius cache is kept; ``clear()``
    exists for the seam (``models/musc.py:274-275``).
    """

    def __call__(self, layer, features, return_cpu: bool = True) -> torch.Tensor:
        return aggregate_features(layer, features, return_cpu)

    def clear(self) -> None:
        pass


class SuperFastAggregation(Aggregation):
    """One layer, r=3, 37x37 -> 28x28 (``models/modules/_super_fast.py:10-27``)."""

    PATCH_GRID = 28

    def __call__(self, layer, tokens, return_cpu: bool = True) -> torch.Tensor:
        _check_layer(layer, tokens)
        first = tokens[0]
        side = math.isqrt(first.shape[1] - 1)
        if side != 37 or len(tokens) != 1 or layer.r != 3:
            raise ValueError('super_fast requires one layer, r=3 and a37x37 source patch grid')
        out = ops.lnamd_super_fast(first, self.PATCH_GRID, l2_normalize=False).unsqueeze(2)
        if not return_cpu:
            return out
        host = out.cpu()
        ops.check_device_error(out.device, 'aggregation')
        return host


def new_aggregation() -> Aggregation:
    return Aggregation()


def new_super_fast_aggregation() -> SuperFastAggregation:
    return SuperFastAggregation()


def begin_inference() -> None:
    for k in _STATS:
        _STATS[k] = 0


def encode_image(model, image, out_layers):
    """``encoding`` seam: the ViT-L/14 forward with the B200 attention kernel."""
    from .encoder import encode_image as b200_encode
    return b200_encode(model, image, out_layers)


encode_image.aggregate_features = aggregate_features
encode_image.new_aggregation = new_aggregation
encode_image.begin_inference = begin_inference


def encode_image_super_fast(model, image, out_layers):
    return encode_image(model, image, out_layers)


encode_image_super_fast.aggregate_features = aggregate_features
encode_image_super_fast.new_aggregation = new_super_fast_aggregation
encode_image_super_fast.begin_inference = begin_inference


def research_diagnostics() -> dict:
    return dict(_STATS)
