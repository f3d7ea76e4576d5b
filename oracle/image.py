"""Image-preprocessing oracle (numpy) -- test infrastructure only.

Restates the evaluation transform the reference applies to every pool image
before the encoder:

* ``models/backbone/open_clip/transform.py:124-133``: ``Resize((S, S),
  BICUBIC)``, ``CenterCrop((S, S))`` (the identity after a resize to S x S),
  ``_convert_to_rgb``, ``ToTensor()``, ``Normalize(OPENAI mean, std)``;
* applied per item in ``datasets/mvtec.py:98-99`` and collated by
  ``models/modules/_loader.py:8-43``; ``models/musc.py:197`` then moves the
  fp32 batch to the device.

The resize is Pillow's (12.2.0 in this image; a third-party dependency of the
reference through torchvision, not vendored in the checkout), whose published
separable resampling algorithm is restated here:

1. Per axis, coefficient tables in float64: ``scale = in/out``,
   ``filterscale = max(scale, 1)``, ``support = filter_support * filterscale``,
   ``ksize = 2*ceil(support) + 1``; for output index ``o`` the centre is
   ``(o + 0.5) * scale``, the taps run from ``xmin = int(centre - support +
   0.5)`` (clamped at 0) to ``int(centre + support + 0.5)`` (clamped at the
   input size), each weight ``filter((x + xmin - centre + 0.5) / filterscale)``
   (the reciprocal of ``filterscale`` taken first), normalised by their sum.
2. The weights become fixed point with 22 fractional bits, rounded half away
   from zero (``int(w * 2**22 +- 0.5)``).
3. A horizontal pass over the rows the vertical pass needs, then a vertical
   pass; each accumulates ``2**21 + sum(pixel * weight)`` in int32 and clips
   ``acc >> 22`` to [0, 255], so the intermediate image is 8-bit.  A pass whose
   axis keeps its size is skipped.

Bicubic uses a = -0.5 and support 2; bilinear (the reference's non-CLIP path,
``datasets/mvtec.py:53-60``) the triangle with support 1.  ``ToTensor`` is
``float32(u8) / 255`` and ``Normalize`` is ``(x - mean) / std`` in float32, both
with fp32 constants.  ``tests/golden/make_golden.py`` pins this restatement bit
for bit to the reference's own transform.
"""
from __future__ import annotations

import math

import numpy as np

OPENAI_MEAN = (0.48145466, 0.4578275, 0.40821073)
OPENAI_STD = (0.26862954, 0.26130258, 0.27577711)

PRECISION_BITS = 22

BICUBIC, BILINEAR = 'bicubic', 'bilinear'
_SUPPORT = {BICUBIC: 2.0, BILINEAR: 1.0}


def _filter(kind: str, x: float) -> float:
    x = abs(x)
    if kind == BILINEAR:
        return 1.0 - x if x < 1.0 else 0.0
    a = -0.5
    if x < 1.0:
        return ((a + 2.0) * x - (a + 3.0)) * x * x + 1
    if x < 2.0:
        return (((x - 5) * x + 8) * x - 4) * a
    return 0.0


def coefficients(in_size: int, out_size: int, kind: str = BICUBIC):
    """One axis's tables: ``(bounds (out, 2) int [first tap, tap count],
    weights (out, ksize) int32 fixed point)``."""
    scale = float(in_size) / out_size
    filterscale = max(scale, 1.0)
    support = _SUPPORT[kind] * filterscale
    ksize = int(math.ceil(support)) * 2 + 1
    bounds = np.zeros((out_size, 2), dtype=np.int64)
    weights = np.zeros((out_size, ksize), dtype=np.int32)
    ss = 1.0 / filterscale
    for o in range(out_size):
        centre = (o + 0.5) * scale
        xmin = max(int(centre - support + 0.5), 0)
        xmax = min(int(centre + support + 0.5), in_size) - xmin
        w = [_filter(kind, (x + xmin - centre + 0.5) * ss) for x in range(xmax)]
        ww = 0.0
        for v in w:
            ww += v
        if ww != 0.0:
            w = [v / ww for v in w]
        for x, v in enumerate(w):
            weights[o, x] = int(v * (1 << PRECISION_BITS) + (-0.5 if v < 0 else 0.5))
        bounds[o] = (xmin, xmax)
    return bounds, weights


def _pass(img: np.ndarray, bounds: np.ndarray, weights: np.ndarray, axis: int) -> np.ndarray:
    """One 8-bit pass along ``axis`` (0 = rows / vertical, 1 = columns / horizontal)."""
    src = np.moveaxis(img.astype(np.int64), axis, 0)          # (in, other, ch)
    out = np.empty((bounds.shape[0],) + src.shape[1:], dtype=np.int64)
    for o in range(bounds.shape[0]):
        first, count = int(bounds[o, 0]), int(bounds[o, 1])
        acc = np.full(src.shape[1:], 1 << (PRECISION_BITS - 1), dtype=np.int64)
        for t in range(count):
            acc += src[first + t] * int(weights[o, t])
        out[o] = np.clip(acc >> PRECISION_BITS, 0, 255)
    return np.moveaxis(out, 0, axis).astype(np.uint8)


def resize_u8(img: np.ndarray, out_h: int, out_w: int, kind: str = BICUBIC) -> np.ndarray:
    """``(H, W, 3)`` uint8 -> ``(out_h, out_w, 3)`` uint8, Pillow's antialiased resample."""
    img = np.asarray(img, dtype=np.uint8)
    h, w = img.shape[:2]
    bounds_v, weights_v = coefficients(h, out_h, kind)
    if w != out_w:
        bounds_h, weights_h = coefficients(w, out_w, kind)
        first = int(bounds_v[0, 0])
        last = int(bounds_v[-1, 0] + bounds_v[-1, 1])
        img = _pass(img[first:last], bounds_h, weights_h, axis=1)
        bounds_v = bounds_v.copy()
        bounds_v[:, 0] -= first
    if h != out_h:
        img = _pass(img, bounds_v, weights_v, axis=0)
    return img


def to_tensor_normalize(img: np.ndarray, mean=OPENAI_MEAN, std=OPENAI_STD) -> np.ndarray:
    """``(H, W, 3)`` uint8 -> ``(3, H, W)`` float32: ``(u8 / 255 - mean) / std`` in fp32."""
    x = np.ascontiguousarray(np.asarray(img, dtype=np.uint8).transpose(2, 0, 1)).astype(np.float32)
    x = x / np.float32(255)
    m = np.asarray(mean, dtype=np.float32).reshape(3, 1, 1)
    s = np.asarray(std, dtype=np.float32).reshape(3, 1, 1)
    return ((x - m) / s).astype(np.float32)


def preprocess(img: np.ndarray, size: int = 518, kind: str = BICUBIC, mean=OPENAI_MEAN,
               std=OPENAI_STD) -> np.ndarray:
    """The reference's per-image evaluation transform: ``(H, W, 3)`` uint8 ->
    ``(3, size, size)`` float32."""
    return to_tensor_normalize(resize_u8(img, size, size, kind), mean, std)
