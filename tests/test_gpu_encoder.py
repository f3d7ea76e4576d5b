"""The b200 ViT-L/14 encoder (16-bit GEMMs + the fused attention kernel) against the
reference's own fp32 VisionTransformer, and config 5 in miniature from pixels to scores.

The golden fixture ``encoder_pool6`` holds the reference's tokens after blocks 6/12/18/24
(sampled rows), its pooled output and the full reference pipeline's scores for 6 seeded
images under seeded random weights (``musc_b200.encoder.random_vit_state``).  The encoder
runs fp16 (the reference GPU path's autocast type); the bf16 variant is checked on image
scores.  Tolerances: tokens within 5e-3 RMS / 5e-2 max of the layer's RMS; per-patch maps
and per-image scores within 1e-3 relative -- the north star's bound for the 16-bit encoder
path.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _encode(cuda_device, compute_dtype):
    from musc_b200.encoder import VisionEncoder, random_vit_state
    from musc_b200.synthetic import random_images
    g = golden('encoder_pool6')
    enc = VisionEncoder(random_vit_state(int(g['seed'])), device=cuda_device, compute_dtype=compute_dtype)
    images = random_images(int(g['n']), 518, seed=int(g['seed'])).to(cuda_device)
    pooled, tokens = [], [[] for _ in g['out_layers']]
    for i in range(0, images.shape[0], 4):   # the reference's batch size
        pl, toks = enc.forward(images[i:i + 4], [int(l) for l in g['out_layers']])
        pooled.append(pl)
        for li, t in enumerate(toks):
            tokens[li].append(t)
    return g, torch.cat(pooled), [torch.cat(t) for t in tokens]


@pytest.fixture(scope='module')
def encoded(cuda_device):
    return _encode(cuda_device, torch.float16)


def test_bf16_encoder_image_scores(cuda_device):
    from musc_b200.pipeline import score_pool
    g, _, tokens = _encode(cuda_device, torch.bfloat16)
    res = score_pool(tokens)
    np.testing.assert_allclose(res.image_max.cpu().numpy(), g['image_max'], rtol=1e-3, atol=0)


def test_encoder_tokens_match_reference(encoded):
    g, pooled, tokens = encoded
    rows = torch.from_numpy(g['token_probe_rows']).to(tokens[0].device)
    for li, t in enumerate(tokens):
        diff = t[:, rows].cpu().numpy() - g['tokens_probe'][li]
        rms_err = np.sqrt((diff ** 2).mean()) / g['token_rms'][li]
        max_err = np.abs(diff).max() / g['token_rms'][li]
        print(f'layer {int(g["out_layers"][li])}: rms error {rms_err:.3g}, max error {max_err:.3g} x RMS')
        assert rms_err < 5e-3 and max_err < 5e-2
    perr = np.abs(pooled.cpu().numpy() - g['pooled']).max() / np.sqrt((g['pooled'] ** 2).mean())
    print(f'pooled: max error {perr:.3g} x RMS')
    assert perr < 5e-2


def test_pixels_to_scores_match_reference(encoded):
    """Config 5 in miniature: b200 encoder -> LNAMD -> MSM -> maps / image scores."""
    from musc_b200.pipeline import score_pool
    g, _, tokens = encoded
    res = score_pool(tokens)
    rel = np.abs(res.image_max.cpu().numpy() / g['image_max'] - 1).max()
    rel_maps = np.abs(res.maps.cpu().numpy() / g['maps'] - 1).max()
    print(f'image max rel error {rel:.3g}, maps rel error {rel_maps:.3g}')
    np.testing.assert_allclose(res.maps.cpu().numpy(), g['maps'], rtol=1e-3, atol=0)
    np.testing.assert_allclose(res.image_max.cpu().numpy(), g['image_max'], rtol=1e-3, atol=0)
    # The 12 per-(layer, radius) components the maps average are intermediate; their small
    # values (deep layers, r = 5) carry up to ~2e-3 relative error from the 16-bit encoder.
    np.testing.assert_allclose(res.scores.cpu().numpy(), g['scores'], rtol=5e-3, atol=0)


def test_backend_encode_image_seam(cuda_device):
    """``encoding(model, image, out_layers)`` accepts a reference-style model with ``.visual``."""
    from musc_b200 import backend
    from musc_b200.encoder import VisionEncoder, random_vit_state
    enc = VisionEncoder(random_vit_state(1, layers=2), layers=2, device=cuda_device)
    img = torch.rand(2, 3, 518, 518, device=cuda_device)
    pooled, toks = backend.encode_image(enc, img, [1, 2])
    assert pooled.shape == (2, 768) and [t.shape for t in toks] == [(2, 1370, 1024)] * 2
    assert callable(backend.encode_image.new_aggregation) and callable(backend.encode_image.aggregate_features)


@pytest.mark.parametrize('dt', [torch.float16, torch.bfloat16])
@pytest.mark.parametrize('with_delta', [True, False])
def test_add_layernorm_matches_torch(cuda_device, dt, with_delta):
    """The fused residual add + LayerNorm of the encoder's blocks against torch's add and
    layer_norm: the fp32 residual bit for bit, the 16-bit output within one unit in its
    last place (fp32 statistics summed in a different order)."""
    import torch.nn.functional as F
    from musc_b200 import ops
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 1370, 1024, generator=g).to(cuda_device)
    delta = (0.5 * torch.randn(3, 1370, 1024, generator=g)).to(dt).to(cuda_device) if with_delta else None
    w = (1 + 0.1 * torch.randn(1024, generator=g)).to(cuda_device)
    b = (0.1 * torch.randn(1024, generator=g)).to(cuda_device)
    want_x = x + delta.float() if with_delta else x.clone()
    ref = F.layer_norm(want_x, (1024,), w, b, 1e-5)
    got = ops.add_layernorm(x, delta, w, b, out_dtype=dt)
    assert torch.equal(x, want_x)
    ulp = 2.0 ** -10 if dt == torch.float16 else 2.0 ** -7
    err = (got.float() - ref).abs()
    assert bool((err <= ulp * ref.abs().clamp_min(2.0 ** -6) + 1e-6).all())
