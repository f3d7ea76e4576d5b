"""ViT-L/14 image encoder for the ``b200`` backend (the ``encoding`` seam).

Runs the reference CLIP vision tower's forward
(``models/backbone/open_clip/transformer.py:554-614``, blocks ``:190-249``) with
its own block loop so the attention of every block goes through the fused
tcgen05 kernel (``musc_b200.ops.attention``) and no attention probabilities are
materialised.  The reference asks ``nn.MultiheadAttention`` for the weights
(``need_weights=True``, ``:232-234``) but only block 12's are kept, and those
only for an ``out_attn`` map that ``VisionTransformer.forward`` computes and
discards (``:587-591``), so they are not produced here.

Numerics: the linear layers (QKV in-projection, out-projection, MLP) are
16-bit cuBLAS GEMMs with fp32 accumulation (reduced-precision fp16 reductions
off, as ``models/modules/_MSM_gpu.py:733-735`` does for its GEMMs); the residual
stream stays fp32, and each residual add runs fused with the LayerNorm after it
(``ops.add_layernorm``: fp32 statistics, 16-bit output for the next GEMM); attention takes 16-bit q/k/v
with fp32 softmax and accumulation.  The 16-bit type defaults to fp16 -- the
type the reference's GPU path runs its encoder in (``torch.cuda.amp.autocast``
at ``models/musc.py:196``) -- and bf16 is available (``compute_dtype``).
Tokens after blocks ``out_layers`` (1-based, ``models/musc.py:61``,
``transformer.py:336-337``) are returned as ``(B, 1+grid^2, width)`` fp32.
Weights use the reference's ``state_dict`` names, so a trained CLIP
``model.visual`` loads directly (``VisionEncoder.from_reference``).
"""
from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.nn.functional as F

from . import ops


class VisionEncoder:
    """Weights + forward of an open_clip ``VisionTransformer`` (no patch dropout/pooler)."""

    def __init__(self, state: dict, image_size: int = 518, patch_size: int = 14, width: int = 1024,
                 layers: int = 24, heads: int = 16, device='cuda', compute_dtype=torch.float16):
        if width // heads != 64:
            raise ValueError('the b200 attention kernel needs head_dim 64')
        if compute_dtype not in (torch.float16, torch.bfloat16):
            raise ValueError('compute_dtype must be torch.float16 or torch.bfloat16')
        self.dtype = compute_dtype
        self.image_size, self.patch_size, self.width = image_size, patch_size, width
        self.layers, self.heads = layers, heads
        self.grid = image_size // patch_size
        dev = torch.device(device)
        f32 = lambda k: state[k].to(dev, torch.float32).contiguous()
        bf = lambda k: state[k].to(dev, compute_dtype).contiguous()
        self.conv_w = bf('conv1.weight').reshape(width, -1)          # (width, 3*p*p)
        self.cls = f32('class_embedding')
        self.pos = f32('positional_embedding')
        self.ln_pre = (f32('ln_pre.weight'), f32('ln_pre.bias'))
        self.blocks = []
        for i in range(layers):
            pre = f'transformer.resblocks.{i}.'
            self.blocks.append(dict(
                ln_1=(f32(pre + 'ln_1.weight'), f32(pre + 'ln_1.bias')),
                in_w=bf(pre + 'attn.in_proj_weight'), in_b=f32(pre + 'attn.in_proj_bias'),
                out_w=bf(pre + 'attn.out_proj.weight'), out_b=f32(pre + 'attn.out_proj.bias'),
                ln_2=(f32(pre + 'ln_2.weight'), f32(pre + 'ln_2.bias')),
                fc_w=bf(pre + 'mlp.c_fc.weight'), fc_b=f32(pre + 'mlp.c_fc.bias'),
                proj_w=bf(pre + 'mlp.c_proj.weight'), proj_b=f32(pre + 'mlp.c_proj.bias')))
        self.ln_post = (f32('ln_post.weight'), f32('ln_post.bias'))
        self.proj = f32('proj')
        self._graphs: dict = {}

    @classmethod
    def from_reference(cls, visual, device='cuda', compute_dtype=torch.float16) -> 'VisionEncoder':
        """Load from an open_clip ``VisionTransformer`` (``model.visual``) of the reference."""
        state = {k: v.detach() for k, v in visual.state_dict().items()}
        width = state['class_embedding'].shape[0]
        patch = state['conv1.weight'].shape[-1]
        grid = math.isqrt(state['positional_embedding'].shape[0] - 1)
        layers = len({k.split('.')[2] for k in state if k.startswith('transformer.resblocks.')})
        return cls(state, image_size=grid * patch, patch_size=patch, width=width, layers=layers,
                   heads=width // 64, device=device, compute_dtype=compute_dtype)

    def _linear(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        return F.linear(x, w, b.to(self.dtype))

    def forward(self, images: torch.Tensor, out_layers: Sequence[int], graph: bool = True):
        """``images`` (B, 3, H, W) -> ``(pooled (B, out_dim) fp32, [tokens (B, 1+g^2, width) fp32])``.

        With ``graph`` (CUDA inputs), the first call for a batch shape runs eagerly and
        captures the whole forward -- GEMMs, LayerNorms and the attention kernel's launches
        -- into a CUDA graph; later calls copy the images in and replay it.  Outputs are
        fresh tensors either way.
        """
        flag = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
        try:
            if not graph or not images.is_cuda:
                return self._forward(images, out_layers)
            key = (tuple(images.shape), images.dtype, images.device, tuple(int(l) for l in out_layers))
            entry = self._graphs.get(key)
            if entry is None:
                dev = images.device
                static_in = images.detach().clone()
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):               # warm-up: sets up every launch
                    out = self._forward(static_in, out_layers)
                torch.cuda.current_stream(dev).wait_stream(side)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    static_out = self._forward(static_in, out_layers)
                self._graphs[key] = (g, static_in, static_out)
                return out
            g, static_in, (pooled, toks) = entry
            static_in.copy_(images)
            g.replay()
            return pooled.clone(), [t.clone() for t in toks]
        finally:
            torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = flag

    def _forward(self, images: torch.Tensor, out_layers: Sequence[int]):
        lp = self.dtype
        b = images.shape[0]
        p, g, w = self.patch_size, self.grid, self.width
        # conv1 with stride = kernel = patch: a GEMM over non-overlapping patches
        patches = images.reshape(b, 3, g, p, g, p).permute(0, 2, 4, 1, 3, 5).reshape(b, g * g, 3 * p * p)
        x = F.linear(patches.to(lp), self.conv_w).float()                       # (B, g^2, width)
        x = torch.cat([self.cls.expand(b, 1, w), x], dim=1) + self.pos
        x = F.layer_norm(x, (w,), *self.ln_pre).contiguous()
        keep = set(int(l) for l in out_layers)
        tokens = {}
        # Each residual add is fused with the LayerNorm that follows it (ops.add_layernorm:
        # x += branch output in fp32, then the 16-bit normalised input of the next GEMM), so
        # the MLP output of block i is added to x at the start of block i + 1.
        pending = None
        for idx, blk in enumerate(self.blocks, start=1):
            h = ops.add_layernorm(x, pending, *blk['ln_1'], out_dtype=lp)
            if idx - 1 in keep:
                tokens[idx - 1] = x.clone()                              # x after block idx - 1
            qkv = self._linear(h, blk['in_w'], blk['in_b'])                      # (B, L, 3w) 16-bit
            a = ops.attention(qkv[..., :w], qkv[..., w:2 * w], qkv[..., 2 * w:], self.heads)
            h = ops.add_layernorm(x, self._linear(a, blk['out_w'], blk['out_b']), *blk['ln_2'], out_dtype=lp)
            h = F.gelu(self._linear(h, blk['fc_w'], blk['fc_b']))       # evaluated in fp32 by torch
            pending = self._linear(h, blk['proj_w'], blk['proj_b'])
        x = x + pending                                                  # the last block's residual
        if len(self.blocks) in keep:
            tokens[len(self.blocks)] = x
        pooled = F.layer_norm(x[:, 0], (w,), *self.ln_post) @ self.proj
        return pooled, [tokens[l] for l in out_layers]


def random_vit_state(seed: int = 0, image_size: int = 518, patch_size: int = 14, width: int = 1024,
                     layers: int = 24, heads: int = 16, mlp_ratio: float = 4.0,
                     output_dim: int = 768) -> dict:
    """Seeded random ViT weights under the reference's ``state_dict`` names (CPU fp32).

    Linear and conv weights/biases ~ U(+-1/sqrt(fan_in)) (torch's default ranges),
    the QKV in-projection ~ U(+-sqrt(6/(fan_in+fan_out))), LayerNorm affines
    ~ 1 + 0.1 N(0,1) / 0.1 N(0,1) (so the affine path is exercised), embeddings and
    the projection ~ width^-0.5 N(0,1) (``transformer.py:385-386, 403``).
    """
    g = torch.Generator().manual_seed(seed)
    grid = image_size // patch_size
    mlp = int(width * mlp_ratio)
    s = width ** -0.5
    st = {}

    def uni(shape, bound):
        return (torch.rand(*shape, generator=g) * 2 - 1) * bound

    def ln(name, n):
        st[name + '.weight'] = 1 + 0.1 * torch.randn(n, generator=g)
        st[name + '.bias'] = 0.1 * torch.randn(n, generator=g)

    st['class_embedding'] = s * torch.randn(width, generator=g)
    st['positional_embedding'] = s * torch.randn(grid * grid + 1, width, generator=g)
    st['proj'] = s * torch.randn(width, output_dim, generator=g)
    st['conv1.weight'] = uni((width, 3, patch_size, patch_size), (3 * patch_size * patch_size) ** -0.5)
    ln('ln_pre', width)
    ln('ln_post', width)
    for i in range(layers):
        pre = f'transformer.resblocks.{i}.'
        ln(pre + 'ln_1', width)
        ln(pre + 'ln_2', width)
        st[pre + 'attn.in_proj_weight'] = uni((3 * width, width), math.sqrt(6 / (4 * width)))
        st[pre + 'attn.in_proj_bias'] = uni((3 * width,), width ** -0.5)
        st[pre + 'attn.out_proj.weight'] = uni((width, width), width ** -0.5)
        st[pre + 'attn.out_proj.bias'] = uni((width,), width ** -0.5)
        st[pre + 'mlp.c_fc.weight'] = uni((mlp, width), width ** -0.5)
        st[pre + 'mlp.c_fc.bias'] = uni((mlp,), width ** -0.5)
        st[pre + 'mlp.c_proj.weight'] = uni((width, mlp), mlp ** -0.5)
        st[pre + 'mlp.c_proj.bias'] = uni((width,), mlp ** -0.5)
    return st


_CACHE: dict = {}


def encode_image(model, image: torch.Tensor, out_layers: Sequence[int]):
    """``encoding`` seam (``models/musc.py:212``): ``model`` is a reference CLIP model
    (``model.visual`` is used) or a :class:`VisionEncoder`."""
    if isinstance(model, VisionEncoder):
        enc = model
    else:
        visual = getattr(model, 'visual', model)
        key = (id(visual), image.device)
        enc = _CACHE.get(key)
        if enc is None:
            enc = VisionEncoder.from_reference(visual, device=image.device)
            _CACHE.clear()
            _CACHE[key] = enc
    with torch.no_grad():
        return enc.forward(image.float(), out_layers)
