"""Timed CPU baseline: the reference's ``original`` path restated with the same torch
CPU operations -- TEST / BENCHMARK INFRASTRUCTURE ONLY.

``bench.py``'s CPU-baseline leg and ``--impl reference`` time this module on the host
cores.  The numpy oracle (``oracle.lnamd``, ``oracle.msm``) is the parity checker; this
module exists so the *timed* baseline runs the library calls the reference itself runs
(the numpy restatement is 2-2.5x slower than the reference on the same cores, which would
understate it).  Its results are pinned against the same golden fixtures.

* ``lnamd_bank`` -- ``LNAMD._embed`` for one layer (``models/modules/_LNAMD.py:72-129``):
  CLS dropped, ``(B, C, side, side)`` view, LayerNorm over ``(C, side, side)`` with unit
  weight and zero bias (``:78-85``), r x r patches by ``unfold`` with zero padding
  (``PatchMaker.patchify``, ``:16-34``; r = 1 is the plain reshape of ``:93-94``), the
  per-channel window mean by ``adaptive_avg_pool1d`` over the flattened ``(C, r, r)``
  patch (``MeanMapper``, ``:58-61``), then the L2 normalisation of ``models/musc.py:238``.
* ``clip_image_transform`` -- the per-image evaluation transform of the pool images.
* ``msm_rows`` -- ``compute_scores_fast`` (``models/modules/_MSM.py:10-30``) for one
  query image: ``cdist`` against every other image's patches, the per-image minimum, the
  two ``topk`` passes of the interval ``[k_min, k_max)`` and the mean.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def lnamd_bank(tokens: torch.Tensor, r: int, l2_normalize: bool = True) -> torch.Tensor:
    """``(B, 1+P, C)`` fp32 CPU tokens -> ``(B, P, C)`` LNAMD features of radius ``r``."""
    b, length, c = tokens.shape
    side = math.isqrt(length - 1)
    grid = tokens[:, 1:, :].reshape(b, side, side, c).permute(0, 3, 1, 2)
    shape = [c, side, side]
    grid = F.layer_norm(grid, shape, torch.ones(shape), torch.zeros(shape), 1e-5)
    if r == 1:
        patches = grid.reshape(b, c, -1, 1, 1).permute(0, 2, 1, 3, 4)
    else:
        cols = F.unfold(grid, kernel_size=r, padding=(r - 1) // 2, stride=1)     # (B, C*r*r, P)
        patches = cols.reshape(b, c, r, r, -1).permute(0, 4, 1, 2, 3)          # (B, P, C, r, r)
    flat = patches.reshape(-1, 1, c * r * r)
    z = F.adaptive_avg_pool1d(flat, c).squeeze(1).reshape(b, -1, c)
    if l2_normalize:
        z = z / z.norm(dim=-1, keepdim=True)
    return z


def lnamd_super_fast(tokens: torch.Tensor, out_side: int = 28, l2_normalize: bool = True) -> torch.Tensor:
    """Super-fast profile on CPU: ``SuperFastAggregation.__call__`` (``models/modules/_super_fast.py:17-27``).

    The r = 3 direct-pool LNAMD of ``aggregate_features`` (``models/modules/_encoder_gpu.py:14-42``:
    ``layer_norm`` with unit weight and zero bias, ``avg_pool2d(3, 1, 1,
    count_include_pad=True)``), then ``adaptive_avg_pool2d`` to ``out_side`` x ``out_side`` in
    float32, then the L2 normalisation of ``models/musc.py:238``.  ``(B, 1+P, C)`` -> ``(B, out_side^2, C)``.
    """
    b, length, c = tokens.shape
    side = math.isqrt(length - 1)
    shape = (c, side, side)
    spatial = tokens[:, 1:].reshape(b, side, side, c).permute(0, 3, 1, 2)
    spatial = F.layer_norm(spatial, shape, torch.ones(shape), torch.zeros(shape))
    spatial = F.avg_pool2d(spatial, 3, stride=1, padding=1, count_include_pad=True)
    pooled = F.adaptive_avg_pool2d(spatial.float(), (out_side, out_side))
    z = pooled.reshape(b, c, out_side * out_side).permute(0, 2, 1).contiguous()
    if l2_normalize:
        z = z / z.norm(dim=-1, keepdim=True)
    return z


def interval(n_images: int, topmin_min: float = 0.0, topmin_max: float = 0.3) -> tuple[int, int]:
    """``(k_min, k_max)`` over the ``n_images - 1`` other images (``_MSM.py:19-27``)."""
    k_max = int((n_images - 1) * topmin_max) if topmin_max < 1 else int(topmin_max)
    k_min = int((n_images - 1) * topmin_min) if topmin_min < 1 else int(topmin_min)
    return (k_max, k_min) if k_max < k_min else (k_min, k_max)


def msm_rows(z: torch.Tensor, i: int, k_min: int, k_max: int) -> torch.Tensor:
    """Scores ``(P,)`` of query image ``i`` of the bank ``z`` ``(N, P, C)``."""
    n, p, c = z.shape
    others = torch.cat((z[:i], z[i + 1:]), dim=0).reshape(-1, c)
    dist = torch.cdist(z[i:i + 1], others).reshape(p, n - 1, p)
    nearest = dist.min(dim=-1).values                                             # (P, N-1)
    low = torch.topk(nearest.float(), k_max, largest=False, sorted=True).values
    band = torch.topk(low.float(), k_max - k_min, largest=True, sorted=True).values
    return band.mean(dim=1)


def msm(z: torch.Tensor, topmin_min: float = 0.0, topmin_max: float = 0.3) -> torch.Tensor:
    """``(N, P, C)`` -> ``(N, P)`` float64 (``_MSM.py:53-59``)."""
    k_min, k_max = interval(z.shape[0], topmin_min, topmin_max)
    return torch.stack([msm_rows(z, i, k_min, k_max) for i in range(z.shape[0])]).double()


def clip_image_transform(size: int = 518):
    """The reference's CLIP evaluation transform (``models/backbone/open_clip/transform.py:124-133``)
    built from the same torchvision classes: ``Resize((size, size), BICUBIC)``,
    ``CenterCrop((size, size))``, RGB conversion, ``ToTensor()``, ``Normalize`` with the OpenAI
    constants (``constants.py:1-2``).  Applied to a PIL image it gives the ``(3, size, size)``
    fp32 tensor the reference's dataset returns (``datasets/mvtec.py:98-99``)."""
    from torchvision import transforms
    from torchvision.transforms import InterpolationMode
    return transforms.Compose([
        transforms.Resize((size, size), interpolation=InterpolationMode.BICUBIC),
        transforms.CenterCrop((size, size)),
        lambda image: image.convert('RGB'),
        transforms.ToTensor(),
        transforms.Normalize(mean=(0.48145466, 0.4578275, 0.40821073), std=(0.26862954, 0.26130258, 0.27577711)),
    ])
