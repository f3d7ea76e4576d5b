"""Pin the numpy oracle against golden vectors produced by the reference itself.

The fixtures under tests/golden were written by tests/golden/make_golden.py,
which runs the reference's ``original`` modules (``_MSM.MSM``,
``LNAMD._embed``, ``aggregate_features``, ``SuperFastAggregation``) and the
score reduction of ``models/musc.py:259-288``.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import lnamd as olnamd
from oracle import msm as omsm
from oracle import reduce as oreduce


@pytest.mark.parametrize('case', ['a', 'b', 'c', 'd', 'e'])
def test_msm_small_cases(case):
    g = golden('msm_small')
    z, want = g[f'{case}_z'], g[f'{case}_scores']
    lo, hi = g[f'{case}_ranks']
    got = omsm.msm(z, lo, hi)
    assert got.dtype == np.float64 and got.shape == want.shape
    # Exact duplicates put sqrt(fp32 rounding noise) into both sides, so d ~ 0
    # pairs differ at ~1e-3 absolute; everything else agrees to fp32 rounding.
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-3 if case in ('b', 'd') else 1e-6)


def test_trimmed_ranks_follow_reference():
    # _MSM.py:20-28 for the configs' pool sizes
    assert omsm.trimmed_ranks(16) == (0, 4)
    assert omsm.trimmed_ranks(100) == (0, 29)
    assert omsm.trimmed_ranks(200) == (0, 59)
    assert omsm.trimmed_ranks(1024) == (0, 306)
    assert omsm.trimmed_ranks(16, 0.1, 0.5) == (1, 7)


@pytest.mark.parametrize('r', [1, 3, 5])
def test_lnamd_matches_embed_and_direct_pool(r):
    g = golden('lnamd_small')
    tokens = g['tokens']                      # (layers, B, 1370, C)
    embed, direct = g[f'embed_r{r}'], g[f'direct_r{r}']   # (B, P, layers, C)
    np.testing.assert_allclose(embed, direct, rtol=0, atol=2e-5)
    for li in range(tokens.shape[0]):
        got = olnamd.lnamd(tokens[li], r)
        np.testing.assert_allclose(got, embed[:, :, li, :], rtol=1e-5, atol=2e-5)


def test_super_fast_pooling():
    g = golden('lnamd_small')
    got = olnamd.lnamd_super_fast(g['tokens'][0], 28)
    np.testing.assert_allclose(got, g['superfast'][:, :, 0, :], rtol=1e-5, atol=2e-5)


def test_score_reduction():
    g = golden('reduce_small')
    maps, image_max = oreduce.image_scores(g['scores'], 518)
    np.testing.assert_allclose(maps, g['maps'], rtol=0, atol=1e-14)
    np.testing.assert_allclose(image_max, g['image_max'], rtol=0, atol=1e-14)
    up = oreduce.bilinear_align_corners(maps, 518)
    np.testing.assert_allclose(up[:, [0, 7, 517], :], g['up_rows_0_7_517'], rtol=0, atol=1e-14)


def test_pool16_banks_and_one_bank_scores():
    """Config 1: the regenerated tokens reproduce the reference's banks and scores."""
    import torch
    from musc_b200.synthetic import prototype_mixture
    g = golden('pool16')
    n = int(g['n'])
    tokens = prototype_mixture(n, n_layers=4, c=1024, side=37, seed=int(g['seed']))
    rows = g['probe_rows']
    for ri, r in enumerate((1, 3, 5)):
        for li in (0, 3):
            z = olnamd.bank(tokens[li].numpy(), r)
            np.testing.assert_allclose(z.reshape(-1, 1024)[rows], g['bank_probe'][ri, li],
                                       rtol=1e-4, atol=2e-6)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    z = olnamd.bank(tokens[2].numpy(), 3)
    got = omsm.msm(z)
    np.testing.assert_allclose(got, g['scores'][1, 2], rtol=2e-5, atol=0)
    maps, image_max = oreduce.image_scores(g['scores'], 518)
    np.testing.assert_allclose(maps, g['maps'], rtol=0, atol=1e-14)
    np.testing.assert_allclose(image_max, g['image_max'], rtol=0, atol=1e-14)


def test_rscin_oracle_matches_reference():
    """oracle.rscin against RsCIN run by the reference (models/modules/_RsCIN.py): the k lists
    MuSc uses, the k = 0 and no-class-token passthroughs."""
    from oracle import rscin as orscin
    g = golden('rscin_small')
    for c in 'abc':
        tok, s = g[f'{c}_tokens'], g[f'{c}_scores']
        for name, ks in (('k123', [1, 2, 3]), ('k189', [1, 8, 9])):
            np.testing.assert_allclose(orscin.rscin(s, list(tok), ks), g[f'{c}_{name}'], rtol=1e-6, atol=0)
        np.testing.assert_array_equal(orscin.rscin(s, list(tok), [0]), g[f'{c}_k0'])
        np.testing.assert_array_equal(orscin.rscin(s, None, [1, 2, 3]), g[f'{c}_none'])


def test_timed_cpu_port_matches_reference_exactly():
    """oracle.torch_cpu (the timed CPU baseline: the reference's original path with the same
    torch CPU operations) reproduces the reference's LNAMD._embed and MSM outputs bit for bit."""
    import torch
    from oracle import torch_cpu
    g = golden('lnamd_small')
    tokens = torch.from_numpy(g['tokens'])                          # (layers, B, 1+P, C)
    for r in (1, 3, 5):
        for layer in range(tokens.shape[0]):
            got = torch_cpu.lnamd_bank(tokens[layer], r, l2_normalize=False).numpy()
            np.testing.assert_array_equal(got, g[f'embed_r{r}'][:, :, layer, :])
    # super-fast: SuperFastAggregation's r = 3 direct pool + adaptive pooling (unnormalised)
    got = torch_cpu.lnamd_super_fast(tokens[0], 28, l2_normalize=False).numpy()
    np.testing.assert_allclose(got, g['superfast'][:, :, 0, :], rtol=1e-5, atol=2e-6)
    g = golden('msm_small')
    for c in 'abcde':
        lo, hi = (float(v) for v in g[f'{c}_ranks'])
        got = torch_cpu.msm(torch.from_numpy(g[f'{c}_z']), lo, hi).numpy()
        np.testing.assert_array_equal(got, g[f'{c}_scores'])


IMAGE_CASES = ('up', 'down', 'wide', 'tall', 'same')
IMAGE_SIZES = {'up': 64, 'down': 112, 'wide': 64, 'tall': 40, 'same': 64}


@pytest.mark.parametrize('case', IMAGE_CASES + ('bilinear',))
def test_image_oracle_matches_reference_transform(case):
    """The numpy restatement of Pillow's resample + ToTensor + Normalize equals the
    reference's own transform bit for bit (``open_clip/transform.py:124-133``; the bilinear
    case is ``datasets/mvtec.py:53-60``)."""
    from oracle import image as oimage
    g = golden('image_preprocess')
    img = g[f'{case}_in']
    if case == 'bilinear':
        got = oimage.preprocess(img, 64, oimage.BILINEAR, (0.485, 0.456, 0.406), (0.229, 0.224, 0.225))
    else:
        got = oimage.preprocess(img, IMAGE_SIZES[case])
    want = g[f'{case}_out']
    assert got.dtype == np.float32 and got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_image_oracle_full_size_hashes():
    """MVTec-sized (900 x 900), VisA-like (1000 x 1500) and up-sampled (200 x 240) images,
    regenerated from their seeds: the oracle's fp32 bytes hash to the reference's."""
    import hashlib
    from oracle import image as oimage
    g = golden('image_preprocess')
    for name, (h, w, size, seed) in {'mvtec900': (900, 900, 518, 11), 'visa1000x1500': (1000, 1500, 518, 12),
                                     'small_up': (200, 240, 518, 13)}.items():
        img = np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)
        got = oimage.preprocess(img, size)
        assert np.array_equal(got[:, ::37, ::41], g[f'{name}_probe']), name
        assert hashlib.sha256(got.tobytes()).hexdigest() == str(g[f'{name}_sha256']), name


def test_timed_image_transform_matches_reference():
    """The CPU baseline's image transform (``oracle.torch_cpu.clip_image_transform``) gives the
    reference transform's tensors bit for bit."""
    from PIL import Image
    from oracle import torch_cpu
    g = golden('image_preprocess')
    for case in IMAGE_CASES:
        got = torch_cpu.clip_image_transform(IMAGE_SIZES[case])(Image.fromarray(g[f'{case}_in'])).numpy()
        assert np.array_equal(got.view(np.uint32), g[f'{case}_out'].view(np.uint32)), case
