"""Device image preprocessing against the reference's transform and the oracle.

``musc_b200_preprocess_images`` must give the reference's fp32 tensors bit for bit
(``open_clip/transform.py:124-133``: Pillow bicubic resize, ToTensor, Normalize), for
up- and down-sampling, one-axis resizes, the identity, the bilinear dataset transform
(``datasets/mvtec.py:53-60``), the full-size MVTec / VisA shapes (by hash) and batched
calls; the loader must keep the reference loader's order and item contract.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import image as oimage

pytestmark = pytest.mark.gpu

SIZES = {'up': 64, 'down': 112, 'wide': 64, 'tall': 40, 'same': 64}
IMAGENET = ((0.485, 0.456, 0.406), (0.229, 0.224, 0.225))


def _device_pre(img: np.ndarray, size, **kw) -> np.ndarray:
    from musc_b200 import ops
    t = torch.from_numpy(np.ascontiguousarray(img)).cuda()
    out = ops.preprocess_images(t[None] if t.ndim == 3 else t, size, **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and np.array_equal(np.ascontiguousarray(a).view(np.uint32),
                                                 np.ascontiguousarray(b).view(np.uint32))


@pytest.mark.parametrize('case', tuple(SIZES) + ('bilinear',))
def test_preprocess_matches_reference_transform(cuda_device, case):
    g = golden('image_preprocess')
    if case == 'bilinear':
        got = _device_pre(g['bilinear_in'], 64, filter='bilinear', mean=IMAGENET[0], std=IMAGENET[1])[0]
    else:
        got = _device_pre(g[f'{case}_in'], SIZES[case])[0]
    assert _bits_equal(got, g[f'{case}_out'])


def test_preprocess_full_size_images_hash_to_the_reference(cuda_device):
    """900 x 900 (MVTec), 1000 x 1500 (VisA-like) and 200 x 240 (up-sampled) -> 518."""
    g = golden('image_preprocess')
    for name, (h, w, seed) in {'mvtec900': (900, 900, 11), 'visa1000x1500': (1000, 1500, 12),
                               'small_up': (200, 240, 13)}.items():
        img = np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)
        got = _device_pre(img, 518)[0]
        assert np.array_equal(got[:, ::37, ::41], g[f'{name}_probe']), name
        assert hashlib.sha256(np.ascontiguousarray(got).tobytes()).hexdigest() == str(g[f'{name}_sha256']), name


@pytest.mark.parametrize('h,w,oh,ow,filt', [(518, 700, 518, 518, 'bicubic'), (700, 518, 518, 518, 'bicubic'),
                                            (33, 17, 5, 61, 'bicubic'), (1, 1, 7, 3, 'bicubic'),
                                            (4000, 600, 300, 64, 'bicubic'), (255, 1024, 64, 96, 'bilinear'),
                                            (9, 700, 40, 23, 'bilinear')])
def test_preprocess_matches_oracle_on_odd_shapes(cuda_device, h, w, oh, ow, filt):
    """One-axis resizes (a pass skipped), extreme ratios, 1-pixel inputs, non-square outputs."""
    rng = np.random.default_rng(h * 7919 + w)
    img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
    want = oimage.to_tensor_normalize(oimage.resize_u8(img, oh, ow, filt))
    got = _device_pre(img, (oh, ow), filter=filt)[0]
    assert _bits_equal(got, want)


def test_preprocess_batches_strides_and_half_outputs(cuda_device):
    """A batch of distinct images in one call, a strided batch view (images inside a larger
    staging buffer), and fp16 / bf16 outputs equal to the fp32 result rounded to nearest."""
    from musc_b200 import ops
    rng = np.random.default_rng(99)
    imgs = rng.integers(0, 256, (5, 120, 90, 3), dtype=np.uint8)
    want = np.stack([oimage.preprocess(im, 72) for im in imgs])
    dev = torch.from_numpy(imgs).cuda()
    got = ops.preprocess_images(dev, 72)
    torch.cuda.synchronize()
    assert _bits_equal(got.cpu().numpy(), want)
    big = torch.zeros((5, 120 * 90 * 3 + 77), dtype=torch.uint8, device='cuda')
    big[:, :120 * 90 * 3] = dev.reshape(5, -1)
    view = big[:, :120 * 90 * 3].view(5, 120, 90, 3)
    got2 = ops.preprocess_images(view, 72)
    assert _bits_equal(got2.cpu().numpy(), want)
    for dt in (torch.float16, torch.bfloat16):
        half = ops.preprocess_images(dev, 72, out_dtype=dt)
        assert torch.equal(half, got.to(dt))


def test_preprocess_rejects_bad_arguments(cuda_device):
    from musc_b200 import _lib, ops
    img = torch.zeros((1, 10, 10, 3), dtype=torch.uint8, device='cuda')
    with pytest.raises(ValueError):
        ops.preprocess_images(img.float(), 8)
    with pytest.raises(ValueError):
        ops.preprocess_images(img[..., :2], 8)
    with pytest.raises(ValueError):
        ops.preprocess_images(img, 8, std=(1.0, 0.0, 1.0))
    with pytest.raises(ValueError):
        ops.preprocess_images(torch.zeros((1, 200, 10, 3), dtype=torch.uint8, device='cuda'), 8)  # 25x
    assert _lib.ERR_INVALID != 0


class _PoolImages:
    def __init__(self, shapes, seed=5):
        rng = np.random.default_rng(seed)
        self.items = [rng.integers(0, 256, s, dtype=np.uint8) for s in shapes]

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        return {'image': self.items[i], 'is_anomaly': i % 3 == 0, 'image_path': f'img{i}.png'}


def test_device_loader_keeps_order_and_contract(cuda_device):
    """Batches in dataset order with the reference's item keys; mixed image sizes inside a
    batch (runs of equal size share a launch); every image equals the oracle's transform."""
    from musc_b200.loader import DeviceImageLoader
    shapes = [(80, 60, 3)] * 3 + [(50, 70, 3)] * 2 + [(80, 60, 3)] * 6
    data = _PoolImages(shapes)
    loader = DeviceImageLoader(data, batch_size=4, workers=3, prefetch_batches=2, size=48)
    assert len(loader) == 3
    seen = 0
    for batch in loader:
        b = batch['image'].shape[0]
        assert batch['image'].is_cuda and batch['image'].dtype == torch.float32
        assert list(batch['image_path']) == [f'img{i}.png' for i in range(seen, seen + b)]
        assert batch['is_anomaly'].tolist() == [i % 3 == 0 for i in range(seen, seen + b)]
        got = batch['image'].cpu().numpy()
        for j in range(b):
            assert _bits_equal(got[j], oimage.preprocess(data.items[seen + j], 48))
        seen += b
    assert seen == len(shapes)
