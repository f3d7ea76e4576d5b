"""Generate the golden fixtures by running the reference's own CPU code.

Run from the repository root in a container where the reference checkout is
available (it is read only through ``--reference``)::

    python tests/golden/make_golden.py --reference <path to the MuSc checkout>

The script imports the reference's ``original`` modules --
``models/modules/_MSM.py`` (``MSM``), ``models/modules/_LNAMD.py``
(``LNAMD._embed``), ``models/modules/_encoder_gpu.py``
(``aggregate_features``), ``models/modules/_super_fast.py``
(``SuperFastAggregation``), ``models/modules/_RsCIN.py`` (``RsCIN``) and
the CLIP ``VisionTransformer``
(``models/backbone/open_clip/transformer.py``) and its evaluation image transform
(``models/backbone/open_clip/transform.py``) -- and evaluates the score
reduction of ``models/musc.py:259-288`` with the same torch calls.  Inputs are
either stored in the fixture (small cases) or regenerated with the recorded
seed (the N=16 prototype-mixture pool from ``musc_b200.synthetic``; the
encoder pool's images and random ViT-L/14 weights from
``musc_b200.synthetic.random_images`` and ``musc_b200.encoder.random_vit_state``).  Nothing at test time reads
the reference; the tests read only the ``.npz`` files written here.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / 'musc-gpu_b200'))


def _reference_modules(reference: str):
    sys.path.insert(0, reference)
    from models.modules._MSM import MSM  # noqa: E402
    from models.modules._LNAMD import LNAMD  # noqa: E402
    from models.modules import _encoder_gpu, _super_fast  # noqa: E402
    return MSM, LNAMD, _encoder_gpu, _super_fast


def _unit_rows(x: torch.Tensor) -> torch.Tensor:
    return x / x.norm(dim=-1, keepdim=True)


def make_msm_small(MSM) -> dict:
    """Small MSM cases with stored inputs, including the edge cases."""
    g = torch.Generator().manual_seed(1234)
    out = {}
    # (name, n, p, c, topmin_min, topmin_max)
    cases = [('a', 5, 49, 64, 0, 0.3), ('b', 9, 49, 64, 0, 0.3),
             ('c', 16, 49, 64, 0.1, 0.5), ('d', 12, 64, 32, 0, 0.3),
             ('e', 7, 100, 128, 0, 0.9)]
    for name, n, p, c, lo, hi in cases:
        z = _unit_rows(torch.randn(n, p, c, generator=g))
        if name == 'b':
            # duplicated patches (distance 0) and exact ties across images
            z[3, :10] = z[0, :10]
            z[5, 20:30] = z[0, 20:30]
            z[6] = z[2]
        if name == 'd':
            # constant image: all its patches identical
            z[4] = z[4, :1].expand(p, c)
        s = MSM(z, 'cpu', topmin_min=lo, topmin_max=hi)
        out[f'{name}_z'] = z.numpy()
        out[f'{name}_scores'] = s.numpy()
        out[f'{name}_ranks'] = np.array([lo, hi], dtype=np.float64)
    return out


def make_lnamd_small(LNAMD, encoder_gpu, super_fast) -> dict:
    """LNAMD (r=1/3/5), the direct-pool form and the super-fast pooling on small C."""
    g = torch.Generator().manual_seed(99)
    b, c = 3, 32
    layers = [torch.randn(b, 1370, c, generator=g) * 2.0 + 0.5 for _ in range(2)]
    out = {'tokens': torch.stack(layers).numpy()}
    for r in (1, 3, 5):
        lnamd = LNAMD(device='cpu', r=r, feature_dim=c, feature_layer=[1, 2])
        emb = lnamd._embed(layers, return_cpu=True)
        direct = encoder_gpu.aggregate_features(lnamd, layers, return_cpu=True)
        out[f'embed_r{r}'] = emb.numpy()
        out[f'direct_r{r}'] = direct.numpy()
    # super-fast profile: one layer, r = 3, 37x37 -> 28x28
    lnamd3 = LNAMD(device='cpu', r=3, feature_dim=c, feature_layer=[1])
    agg = super_fast.SuperFastAggregation()
    sf = agg(lnamd3, [layers[0]], return_cpu=True)
    out['superfast'] = sf.numpy()
    return out


def _reduce_like_musc(scores: torch.Tensor, image_size: int):
    """``models/musc.py:259-288`` on a ``(R, L, N, P)`` float64 tensor."""
    per_r = torch.stack([torch.mean(scores[r], 0) for r in range(scores.shape[0])])
    maps = torch.mean(per_r, 0)
    n, p = maps.shape
    h = int(np.sqrt(p))
    up = F.interpolate(maps.view(n, 1, h, h), size=image_size, mode='bilinear', align_corners=True)
    up = up.cpu().numpy()
    return maps.view(n, h, h).numpy(), up.reshape(n, -1).max(-1), up


def make_reduce_small() -> dict:
    g = torch.Generator().manual_seed(7)
    scores = torch.rand(3, 4, 5, 1369, generator=g, dtype=torch.float64) + 1.0
    maps, image_max, up = _reduce_like_musc(scores, 518)
    return {'scores': scores.numpy(), 'maps': maps, 'image_max': image_max,
            'up_rows_0_7_517': up[:, 0, [0, 7, 517], :]}


def make_pool16(MSM, LNAMD, encoder_gpu) -> dict:
    """Config 1: N=16 prototype-mixture pool, 4 layers x r{1,3,5}, full reference pipeline."""
    from musc_b200.synthetic import prototype_mixture
    n, seed = 16, 0
    tokens = prototype_mixture(n, n_layers=4, c=1024, side=37, seed=seed)
    radii = (1, 3, 5)
    scores = torch.empty(len(radii), 4, n, 1369, dtype=torch.float64)
    probe_rows = np.arange(0, n * 1369, 977)
    bank_probe = np.empty((len(radii), 4, len(probe_rows), 1024), dtype=np.float32)
    torch.set_num_threads(os.cpu_count() or 1)
    for ri, r in enumerate(radii):
        lnamd = LNAMD(device='cpu', r=r, feature_dim=1024, feature_layer=[1, 2, 3, 4])
        feats = lnamd._embed(tokens, return_cpu=True)
        feats /= feats.norm(dim=-1, keepdim=True)
        for li in range(4):
            z = feats[:, :, li, :].contiguous()
            bank_probe[ri, li] = z.reshape(-1, 1024)[probe_rows].numpy()
            scores[ri, li] = MSM(z, 'cpu', topmin_min=0, topmin_max=0.3)
    maps, image_max, _ = _reduce_like_musc(scores, 518)
    return {'seed': np.array(seed), 'n': np.array(n), 'scores': scores.numpy(),
            'maps': maps, 'image_max': image_max, 'probe_rows': probe_rows,
            'bank_probe': bank_probe}


def make_rscin_small(reference: str) -> dict:
    """RsCIN (``models/modules/_RsCIN.py``) on stored class tokens and image scores, for the
    k lists MuSc uses (``models/musc.py:290-295``: [1, 2, 3] for MVTec and the default,
    [1, 8, 9] for VisA), plus the passthrough cases (k = 0, no class tokens)."""
    sys.path.insert(0, reference)
    from models.modules._RsCIN import RsCIN  # noqa: E402
    g = torch.Generator().manual_seed(4321)
    out = {}
    for name, n, dim in (('a', 24, 768), ('b', 60, 768), ('c', 9, 64)):
        tok = _unit_rows(torch.randn(n, dim, generator=g)).numpy().astype(np.float32)
        score = (torch.rand(n, generator=g, dtype=torch.float64) * 0.5 + 1.0).numpy()
        out[f'{name}_tokens'] = tok
        out[f'{name}_scores'] = score
        for kname, ks in (('k123', [1, 2, 3]), ('k189', [1, 8, 9])):
            out[f'{name}_{kname}'] = np.asarray(RsCIN(score, list(tok), k_list=ks))
        out[f'{name}_k0'] = np.asarray(RsCIN(score, list(tok), k_list=[0]))
        out[f'{name}_none'] = np.asarray(RsCIN(score, None, k_list=[1, 2, 3]))
    return out


def _reference_vit_class(reference: str):
    """The reference's ``VisionTransformer`` (``models/backbone/open_clip/transformer.py``),
    imported under a stub package so ``open_clip/__init__.py`` (tokenizer, ftfy) is skipped."""
    import importlib
    import types
    name = 'reference_open_clip'
    if name not in sys.modules:
        pkg = types.ModuleType(name)
        pkg.__path__ = [os.path.join(reference, 'models', 'backbone', 'open_clip')]
        sys.modules[name] = pkg
    return importlib.import_module(name + '.transformer').VisionTransformer


def make_encoder_pool(MSM, LNAMD, reference: str) -> dict:
    """Config 5 in miniature: the reference ViT-L/14 (fp32, CPU) on 6 seeded images with
    seeded random weights, hooks after blocks 6/12/18/24, then LNAMD r{1,3,5} + MSM +
    the score reduction -- the whole reference pipeline from pixels to image scores."""
    from musc_b200.encoder import random_vit_state
    from musc_b200.synthetic import random_images
    VisionTransformer = _reference_vit_class(reference)
    torch.set_num_threads(os.cpu_count() or 1)
    n, seed = 6, 5
    vit = VisionTransformer(image_size=518, patch_size=14, width=1024, layers=24, heads=16, mlp_ratio=4.0,
                            output_dim=768)
    vit.load_state_dict(random_vit_state(seed), strict=True)
    vit.eval()
    images = random_images(n, 518, seed=seed)
    out_layers = [6, 12, 18, 24]
    tokens = [[] for _ in out_layers]
    pooled = []
    with torch.no_grad():
        for i in range(n):
            pl, toks = vit(images[i:i + 1], out_layers)
            pooled.append(pl)
            for li, t in enumerate(toks):
                tokens[li].append(t)
    tokens = [torch.cat(t) for t in tokens]
    probe = np.arange(0, 1370, 17)
    radii = (1, 3, 5)
    scores = torch.empty(len(radii), 4, n, 1369, dtype=torch.float64)
    for ri, r in enumerate(radii):
        lnamd = LNAMD(device='cpu', r=r, feature_dim=1024, feature_layer=[1, 2, 3, 4])
        feats = lnamd._embed(tokens, return_cpu=True)
        feats /= feats.norm(dim=-1, keepdim=True)
        for li in range(4):
            scores[ri, li] = MSM(feats[:, :, li, :].contiguous(), 'cpu', topmin_min=0, topmin_max=0.3)
    maps, image_max, _ = _reduce_like_musc(scores, 518)
    return {'seed': np.array(seed), 'n': np.array(n), 'out_layers': np.array(out_layers),
            'pooled': torch.cat(pooled).numpy(), 'token_probe_rows': probe,
            'tokens_probe': np.stack([t[:, probe].numpy() for t in tokens]),
            'token_rms': np.array([float(t.pow(2).mean().sqrt()) for t in tokens]),
            'scores': scores.numpy(), 'maps': maps, 'image_max': image_max}


def _reference_image_transform(reference: str):
    """``image_transform`` of the reference's open_clip (``models/backbone/open_clip/transform.py``),
    under the same stub package as the ViT."""
    import importlib
    _reference_vit_class(reference)
    return importlib.import_module('reference_open_clip.transform').image_transform


IMAGE_HASHED = {'mvtec900': (900, 900, 518, 11), 'visa1000x1500': (1000, 1500, 518, 12),
                'small_up': (200, 240, 518, 13)}


def make_image_preprocess(reference: str) -> dict:
    """The reference's evaluation transform (``transform.py:124-133``: Resize BICUBIC, CenterCrop,
    ToTensor, Normalize with the OpenAI constants) on seeded 8-bit RGB images: small cases with
    inputs and outputs stored, full-size cases (MVTec's 900 x 900, a VisA-like 1000 x 1500, an
    up-sampled 200 x 240) regenerated from their seeds and pinned by the SHA-256 of the fp32
    output bytes.  ``bilinear`` is the non-CLIP dataset transform (``datasets/mvtec.py:53-60``,
    ``Resize((resize, resize))`` + ``CenterCrop(imagesize)`` with resize == imagesize, ImageNet
    constants), built from the same torchvision classes."""
    import hashlib
    from PIL import Image
    from torchvision import transforms
    image_transform = _reference_image_transform(reference)
    rng = np.random.default_rng(4242)
    out = {}
    for name, (h, w, size) in {'up': (37, 53, 64), 'down': (300, 260, 112), 'wide': (64, 200, 64),
                               'tall': (181, 47, 40), 'same': (64, 64, 64)}.items():
        arr = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        out[f'{name}_in'] = arr
        out[f'{name}_out'] = image_transform(size, is_train=False)(Image.fromarray(arr)).numpy()
    arr = rng.integers(0, 256, (90, 77, 3), dtype=np.uint8)
    mean, std = [0.485, 0.456, 0.406], [0.229, 0.224, 0.225]
    bilinear = transforms.Compose([transforms.Resize((64, 64)), transforms.CenterCrop(64), transforms.ToTensor(),
                                   transforms.Normalize(mean=mean, std=std)])
    out['bilinear_in'] = arr
    out['bilinear_out'] = bilinear(Image.fromarray(arr)).numpy()
    for name, (h, w, size, seed) in IMAGE_HASHED.items():
        arr = np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)
        res = image_transform(size, is_train=False)(Image.fromarray(arr)).numpy()
        out[f'{name}_sha256'] = np.array(hashlib.sha256(np.ascontiguousarray(res).tobytes()).hexdigest())
        out[f'{name}_probe'] = res[:, ::37, ::41].copy()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    ap.add_argument('--only', default='')
    args = ap.parse_args()
    MSM, LNAMD, encoder_gpu, super_fast = _reference_modules(args.reference)
    torch.manual_seed(0)
    jobs = {'msm_small': lambda: make_msm_small(MSM),
            'lnamd_small': lambda: make_lnamd_small(LNAMD, encoder_gpu, super_fast),
            'reduce_small': make_reduce_small,
            'pool16': lambda: make_pool16(MSM, LNAMD, encoder_gpu),
            'encoder_pool6': lambda: make_encoder_pool(MSM, LNAMD, args.reference),
            'rscin_small': lambda: make_rscin_small(args.reference),
            'image_preprocess': lambda: make_image_preprocess(args.reference)}
    for name, job in jobs.items():
        if args.only and name not in args.only.split(','):
            continue
        data = job()
        np.savez_compressed(HERE / f'{name}.npz', **data)
        print(name, {k: v.shape for k, v in data.items()})


if __name__ == '__main__':
    main()
