"""Seeded synthetic inputs standing in for MVTec category pools.

MVTec AD is not available offline, so every benchmark and parity case draws its
patch tokens from a prototype mixture:

* ``n_proto`` prototypes drawn from N(0, I_C) and scaled to unit norm;
* each patch token is ``prototype[randint(n_proto)] + sigma * eps`` with
  ``eps ~ N(0, I_C)``;
* a Bernoulli(``anomaly_frac``) subset of patches is replaced by N(0, I_C)
  vectors (the off-manifold "anomalies");
* token 0 (the CLS slot that LNAMD drops, ``models/modules/_LNAMD.py:78``) is
  all zeros.

The layout is the encoder's token layout ``(N, 1 + side*side, C)`` fp32, one
tensor per hooked layer, layers drawn independently.  Generation runs on the
CPU with ``torch.Generator`` so the same seed gives the same tensors on every
machine with the same torch build.
"""
from __future__ import annotations

import torch


def prototype_mixture_layer(n_images: int, c: int = 1024, side: int = 37,
                            n_proto: int = 64, sigma: float = 0.1,
                            anomaly_frac: float = 0.05,
                            generator: torch.Generator | None = None) -> torch.Tensor:
    """One layer of tokens, shape ``(n_images, 1 + side*side, c)`` fp32 (CPU)."""
    g = generator if generator is not None else torch.Generator().manual_seed(0)
    p = side * side
    protos = torch.randn(n_proto, c, generator=g)
    protos = protos / protos.norm(dim=1, keepdim=True)
    idx = torch.randint(0, n_proto, (n_images, p), generator=g)
    tokens = torch.empty(n_images, p + 1, c)
    tokens[:, 0].zero_()
    body = tokens[:, 1:]
    # Chunked over images so peak host memory stays at the output size.
    for i in range(n_images):
        noise = torch.randn(p, c, generator=g)
        body[i] = protos[idx[i]] + sigma * noise
        mask = torch.rand(p, generator=g) < anomaly_frac
        k = int(mask.sum())
        if k:
            body[i, mask] = torch.randn(k, c, generator=g)
    return tokens


def prototype_mixture(n_images: int, n_layers: int = 4, c: int = 1024, side: int = 37,
                      n_proto: int = 64, sigma: float = 0.1, anomaly_frac: float = 0.05,
                      seed: int = 0) -> list[torch.Tensor]:
    """``n_layers`` independent token tensors for one pool (seeded)."""
    g = torch.Generator().manual_seed(seed)
    return [prototype_mixture_layer(n_images, c, side, n_proto, sigma, anomaly_frac, g)
            for _ in range(n_layers)]


def random_images(n_images: int, size: int = 518, seed: int = 0) -> torch.Tensor:
    """Images in [0, 1], shape ``(n_images, 3, size, size)`` fp32 (CPU)."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(n_images, 3, size, size, generator=g)
