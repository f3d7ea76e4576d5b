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


def prototype_mixture_images(image_ids, n_layers: int = 4, c: int = 1024, side: int = 37,
                             n_proto: int = 64, sigma: float = 0.1, anomaly_frac: float = 0.05,
                             seed: int = 0, device='cpu') -> list[torch.Tensor]:
    """The same mixture, drawn image by image: any subset of a pool (one rank's shard)
    is generated without the rest.  Prototypes are seeded by (seed, layer) and each
    image by (seed, layer, image id), so a pool is identical however it is sharded.
    (Not the same stream as :func:`prototype_mixture`, which draws a pool sequentially.)
    """
    ids = list(image_ids)
    p = side * side
    dev = torch.device(device)
    layers = []
    for layer in range(n_layers):
        g = torch.Generator(device=dev).manual_seed((seed * 1_000_003 + layer) * 7919 + 17)
        protos = torch.randn(n_proto, c, generator=g, device=dev)
        protos = protos / protos.norm(dim=1, keepdim=True)
        tokens = torch.zeros(len(ids), p + 1, c, device=dev)
        for k, img in enumerate(ids):
            gi = torch.Generator(device=dev).manual_seed(((seed * 1_000_003 + layer) * 1_000_033 + img) * 31 + 5)
            idx = torch.randint(0, n_proto, (p,), generator=gi, device=dev)
            body = protos[idx] + sigma * torch.randn(p, c, generator=gi, device=dev)
            mask = torch.rand(p, generator=gi, device=dev) < anomaly_frac
            body[mask] = torch.randn(int(mask.sum()), c, generator=gi, device=dev)
            tokens[k, 1:] = body
        layers.append(tokens)
    return layers


def random_images(n_images: int, size: int = 518, seed: int = 0) -> torch.Tensor:
    """Images in [0, 1], shape ``(n_images, 3, size, size)`` fp32 (CPU)."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(n_images, 3, size, size, generator=g)
