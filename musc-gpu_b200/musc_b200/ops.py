"""Torch-facing wrappers of the C-ABI entry points.

Every function takes and returns CUDA tensors, allocates its outputs and
workspaces with torch's caching allocator, and enqueues the kernels on torch's
current stream of the input's device (the reference launches on the same
stream, ``models/modules/_cuda_runtime.py:95-100``).  Nothing here computes on
the CPU: a missing library or a non-sm_100 device raises.
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _aligned_empty(nbytes: int, device: torch.device, align: int = 1024) -> torch.Tensor:
    """A uint8 buffer whose data pointer is ``align``-byte aligned."""
    raw = torch.empty(nbytes + align, dtype=torch.uint8, device=device)
    off = (-raw.data_ptr()) % align
    return raw[off:off + nbytes]


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f'{what}: expected a CUDA tensor (the b200 backend has no CPU path)')


def check_device_error(device=None, what: str = 'musc_b200') -> None:
    """Raise ``RuntimeError`` if a bounded device-side wait expired since the last check.

    The pipelined kernels never hang: a wait that runs out sets the device's
    error word and the kernel returns early, and from then on the selection,
    map and RsCIN kernels write NaN instead of scores until the word is taken.
    This reads and clears the word (it synchronises the device), so callers
    use it where they synchronise anyway -- after copying results to the host.
    """
    dev = torch.device(device) if device is not None else torch.device('cuda', torch.cuda.current_device())
    with torch.cuda.device(dev):
        code = _lib.take_device_error()
    if code != _lib.OK:
        raise RuntimeError(f'{what}: a device-side bounded wait expired (status {code}); '
                           'the outputs since the last check are NaN or incomplete')


# --------------------------------------------------------------------------- LNAMD
def lnamd(tokens: torch.Tensor, radii: Sequence[int] = (1, 3, 5), l2_normalize: bool = True,
          out: Sequence[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """LNAMD of one layer's tokens ``(B, 1+P, C)`` -> one ``(B, P, C)`` fp32 tensor per radius.

    LayerNorm over the whole ``(C, side, side)`` image, zero-padded r x r mean
    (``models/modules/_encoder_gpu.py:33-37``) and, if ``l2_normalize``, the
    per-patch L2 normalisation of ``models/musc.py:238``.
    """
    _require_cuda(tokens, 'lnamd')
    if tokens.ndim != 3 or tokens.dtype not in _DTYPES:
        raise ValueError('lnamd: expected (B, 1+P, C) float32/float16/bfloat16 tokens')
    tokens = tokens.contiguous()
    b, length, c = tokens.shape
    p = length - 1
    radii = [int(r) for r in radii]
    if out is None:
        out = [torch.empty(b, p, c, dtype=torch.float32, device=tokens.device) for _ in radii]
    outs = list(out)
    for o in outs:
        if o.shape != (b, p, c) or o.dtype != torch.float32 or not o.is_contiguous():
            raise ValueError('lnamd: outputs must be contiguous float32 (B, P, C)')
    _launch_lnamd(tokens, radii, outs, p * c, c, l2_normalize)
    return outs


def lnamd_layers(tokens: Sequence[torch.Tensor], r: int, l2_normalize: bool = False) -> torch.Tensor:
    """The reference aggregation layout: ``(B, P, layers, C)`` for one radius.

    Matches ``aggregate_features`` / ``RadiusAggregationCache.__call__``
    (``models/modules/_encoder_gpu.py:14-42``, ``_aggregation_cache.py:15-58``):
    the per-layer results stacked on dim 2 (``_LNAMD.py:126``).
    """
    first = tokens[0]
    _require_cuda(first, 'lnamd_layers')
    b, length, c = first.shape
    p = length - 1
    layers = len(tokens)
    result = torch.empty(b, p, layers, c, dtype=torch.float32, device=first.device)
    for li, t in enumerate(tokens):
        if t.shape != first.shape or t.dtype != first.dtype or t.device != first.device:
            raise ValueError('lnamd_layers: all layers must share shape, dtype and device')
        view = result[:, :, li, :]
        _launch_lnamd(t.contiguous(), [r], [view], p * layers * c, layers * c, l2_normalize)
    return result


def _launch_lnamd(tokens: torch.Tensor, radii: list[int], outs: list[torch.Tensor],
                  image_stride: int, patch_stride: int, l2_normalize: bool) -> None:
    b, length, c = tokens.shape
    dev = tokens.device
    with torch.cuda.device(dev):
        lib = _lib.lib()
        ws_bytes = lib.musc_b200_lnamd_workspace_bytes(b)
        ws = _aligned_empty(ws_bytes, dev, 256)
        radii_arr = (ctypes.c_int * len(radii))(*radii)
        out_arr = (ctypes.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
        st = lib.musc_b200_lnamd(_ptr(tokens), _DTYPES[tokens.dtype], b, length, c, len(radii),
                                 radii_arr, out_arr, image_stride, patch_stride, int(l2_normalize),
                                 _ptr(ws), ws_bytes, _stream(dev))
        _lib.check(st, 'musc_b200_lnamd')


def lnamd_super_fast(tokens: torch.Tensor, out_side: int = 28, l2_normalize: bool = True,
                     out: torch.Tensor | None = None, image_stride: int | None = None,
                     patch_stride: int | None = None) -> torch.Tensor:
    """r=3 LNAMD then adaptive pooling to ``out_side``^2 patches (``_super_fast.py:17-27``)."""
    _require_cuda(tokens, 'lnamd_super_fast')
    if tokens.ndim != 3 or tokens.dtype not in _DTYPES:
        raise ValueError('lnamd_super_fast: expected (B, 1+P, C) tokens')
    tokens = tokens.contiguous()
    b, length, c = tokens.shape
    q = out_side * out_side
    if out is None:
        out = torch.empty(b, q, c, dtype=torch.float32, device=tokens.device)
        image_stride, patch_stride = q * c, c
    dev = tokens.device
    with torch.cuda.device(dev):
        lib = _lib.lib()
        ws_bytes = lib.musc_b200_lnamd_workspace_bytes(b)
        ws = _aligned_empty(ws_bytes, dev, 256)
        st = lib.musc_b200_lnamd_super_fast(_ptr(tokens), _DTYPES[tokens.dtype], b, length, c, out_side,
                                            _ptr(out), image_stride, patch_stride, int(l2_normalize),
                                            _ptr(ws), ws_bytes, _stream(dev))
        _lib.check(st, 'musc_b200_lnamd_super_fast')
    return out


# --------------------------------------------------------------------------- MSM
def trimmed_ranks(n_images: int, topmin_min: float = 0, topmin_max: float = 0.3) -> tuple[int, int]:
    """``[a, b)`` as the reference derives them (``_MSM_gpu.py:706-709``; ``_MSM.py:20-28``)."""
    a = int((n_images - 1) * topmin_min) if topmin_min < 1 else int(topmin_min)
    b = int((n_images - 1) * topmin_max) if topmin_max < 1 else int(topmin_max)
    a, b = sorted((a, b))
    if not 0 <= a < b <= n_images - 1:
        raise ValueError('Require valid nonempty trimmed ranks 0<=a<b<=N-1.')
    return a, b


def center_stats(z: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Centring statistics of ``z`` ``(rows, C)`` fp32: fp64 ``(C + 1,)`` = the column sums
    and the smallest squared row norm, in a fixed order (the input of :func:`prep_bank`; a
    rank of a multi-GPU pool takes them over its own rows)."""
    _require_cuda(z, 'center_stats')
    if z.ndim != 2 or z.dtype != torch.float32:
        raise ValueError('center_stats: expected (rows, C) float32')
    z = z.contiguous()
    rows, c = z.shape
    dev = z.device
    if out is None:
        out = torch.empty(c + 1, dtype=torch.float64, device=dev)
    if out.dtype != torch.float64 or out.numel() != c + 1 or not out.is_contiguous():
        raise ValueError('center_stats: out must be a contiguous float64 tensor of C + 1 elements')
    with torch.cuda.device(dev):
        lib = _lib.lib()
        nbytes = lib.musc_b200_center_stats_bytes(c)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _lib.check(lib.musc_b200_center_stats(_ptr(z) if rows else None, rows, c, _ptr(out), _ptr(ws), nbytes,
                                              _stream(dev)), 'musc_b200_center_stats')
    return out


def prep_bank(z: torch.Tensor, out: torch.Tensor | None = None, stats: torch.Tensor | None = None,
              count: int | None = None) -> torch.Tensor:
    """Split-fp16 tensor-core operand bank of ``z`` ``(rows, C)`` fp32.

    With ``stats`` (fp64 ``(C + 1,)`` or ``(parts, C + 1)`` from :func:`center_stats`, one
    row per block of the pool) the bank holds the centred rows ``z - mu``,
    ``mu = column sums / count`` (``count`` defaults to ``rows``), when
    ``|mu| <= 2 min |z|`` over the pool; every bank scored against this one must be
    prepared from the same statistics."""
    _require_cuda(z, 'prep_bank')
    if z.ndim != 2 or z.dtype != torch.float32:
        raise ValueError('prep_bank: expected (rows, C) float32')
    z = z.contiguous()
    rows, c = z.shape
    dev = z.device
    with torch.cuda.device(dev):
        lib = _lib.lib()
        nbytes = lib.musc_b200_bank_bytes(rows, c)
        bank = _aligned_empty(nbytes, dev) if out is None else out
        if stats is None:
            _lib.check(lib.musc_b200_prep_bank(_ptr(z), rows, c, _ptr(bank), nbytes, _stream(dev)),
                       'musc_b200_prep_bank')
        else:
            if (stats.dtype != torch.float64 or stats.shape[-1] != c + 1 or not stats.is_contiguous()
                    or stats.device != dev):
                raise ValueError('prep_bank: stats must be contiguous float64 (C + 1,) or (parts, C + 1) '
                                 'on the device')
            parts = 1 if stats.ndim == 1 else stats.shape[0]
            _lib.check(lib.musc_b200_prep_bank_centered(_ptr(z), rows, c, _ptr(stats), parts,
                                                        rows if count is None else int(count), _ptr(bank),
                                                        nbytes, _stream(dev)), 'musc_b200_prep_bank_centered')
    return bank


def nearest(query_bank: torch.Tensor, query_rows: int, query_first_row: int, ref_bank: torch.Tensor,
            ref_rows: int, channels: int, patches: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Squared nearest-patch minima ``(n_images, query_rows)`` fp32 (self image = FLT_MAX)."""
    dev = query_bank.device
    n_images = ref_rows // patches
    if out is None:
        out = torch.empty(n_images, query_rows, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_nearest(_ptr(query_bank), query_rows, query_first_row, _ptr(ref_bank),
                                          ref_rows, channels, patches, _ptr(out), _stream(dev))
        _lib.check(st, 'musc_b200_nearest')
    return out


def nearest_pool_table(rows: int, patches: int, rows_per_block: int | None = None,
                       device=None, min_blocks: int = 1) -> torch.Tensor:
    """An uninitialised ``(blocks, n_images, rows_per_block)`` float32 table for
    :func:`nearest_pool`, backed by ``musc_b200_nearest_pool_bytes`` (the table plus the
    kernel's scheduler word).  ``min_blocks`` pads the block count (a reduce-scatter
    over more ranks than blocks; the padding blocks are never filled)."""
    rpb = rows if rows_per_block is None else rows_per_block
    n_images = rows // patches
    blocks = max(-(-rows // rpb), min_blocks)
    nbytes = max(_lib.lib().musc_b200_nearest_pool_bytes(rows, patches, rpb), blocks * n_images * rpb * 4)
    flat = torch.empty(-(-nbytes // 4), dtype=torch.float32, device=device)
    return flat[:blocks * n_images * rpb].view(blocks, n_images, rpb)


def empty_bank(rows: int, channels: int, device) -> torch.Tensor:
    """An uninitialised, 1024-byte aligned bank buffer for ``rows`` rows."""
    return _aligned_empty(_lib.lib().musc_b200_bank_bytes(rows, channels), torch.device(device))


def bank_planes(bank: torch.Tensor, rows: int, channels: int, layout_rows: int | None = None):
    """uint8 views of the first ``rows`` rows of each plane (hi, lo, |z|^2, 2^-k, residual
    norm) of a bank laid out for ``layout_rows`` rows -- the pieces a rank contributes to a
    gathered bank."""
    layout_rows = rows if layout_rows is None else layout_rows
    offs = (ctypes.c_size_t * 5)()
    _lib.check(_lib.lib().musc_b200_bank_layout(layout_rows, channels, offs), 'musc_b200_bank_layout')
    sizes = (rows * channels * 2, rows * channels * 2, rows * 4, rows * 4, rows * 4)
    return [bank[o:o + n] for o, n in zip(offs, sizes)]


def screen_table(rows: int, patches: int, rows_per_block: int | None = None, device=None,
                 min_blocks: int = 1) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Uninitialised screen tables for :func:`screen_pool`: ``(k1, m2, word)`` with
    ``k1`` ``(blocks, n_images, rpb)`` int64 and ``m2`` the same shape int32 (the signed
    types hold the unsigned keys bit for bit) and ``word`` the scheduler's int64.
    ``min_blocks`` pads the block count (an all-to-all over more ranks than blocks; the
    padding is never filled)."""
    rpb = rows if rows_per_block is None else rows_per_block
    n_images = rows // patches
    blocks = max(-(-rows // rpb), min_blocks)
    dev = torch.device(device) if device is not None else None
    k1 = torch.empty(blocks, n_images, rpb, dtype=torch.int64, device=dev)
    m2 = torch.empty(blocks, n_images, rpb, dtype=torch.int32, device=dev)
    word = torch.empty(1, dtype=torch.int64, device=dev)
    return k1, m2, word


def screen_pool(bank: torch.Tensor, rows: int, channels: int, patches: int, part: int = 0, parts: int = 1,
                rows_per_block: int | None = None, out=None, bank_rows: int | None = None,
                max_ctas: int = 0):
    """Screened symmetric pool pass (one fp16 MMA pass): ``(k1, m2, word)`` of :func:`screen_table`."""
    dev = bank.device
    rpb = rows if rows_per_block is None else rows_per_block
    if out is None:
        out = screen_table(rows, patches, rpb, dev)
    k1, m2, word = out
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_screen_pool(_ptr(bank), rows if bank_rows is None else bank_rows, rows,
                                              channels, patches, part, parts, rpb, int(max_ctas), _ptr(k1),
                                              _ptr(m2), _ptr(word), _stream(dev))
        _lib.check(st, 'musc_b200_screen_pool')
    return out


def refine_launches(n_images: int, query_rows: int, channels: int, workspace_bytes: int | None = None) -> int:
    """Kernels one :func:`refine` call enqueues (with the default workspace)."""
    lib = _lib.lib()
    ws = lib.musc_b200_refine_bytes(n_images, query_rows, channels) if workspace_bytes is None else workspace_bytes
    return lib.musc_b200_refine_launches(n_images, query_rows, channels, ws)


def refine(bank: torch.Tensor, rows: int, channels: int, patches: int, first_row: int, query_rows: int,
           rank_hi: int, k1: torch.Tensor, m2: torch.Tensor, out: torch.Tensor | None = None,
           bank_rows: int | None = None, workspace_bytes: int | None = None) -> torch.Tensor:
    """Exact squared minima ``(n_images, query_rows)`` float32 from screen tables.

    ``k1`` / ``m2``: ``(parts, n_images, table_rows)`` partial screen tables covering the
    query rows (local row = row - first_row), one per part of the pool's tile list.
    Images that cannot reach the trimmed ranks ``[.., rank_hi)`` hold FLT_MAX.
    ``workspace_bytes``: the refinement's scratch (default ``musc_b200_refine_bytes``); any
    size from ``musc_b200_refine_min_bytes`` up gives the same table in more fallback rounds.
    """
    dev = bank.device
    n_images = rows // patches
    if k1.ndim == 2:
        k1, m2 = k1.unsqueeze(0), m2.unsqueeze(0)
    parts, _, table_rows = k1.shape
    if not (k1.is_contiguous() and m2.is_contiguous()):
        raise ValueError('refine: screen tables must be contiguous')
    if out is None:
        out = torch.empty(n_images, query_rows, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        lib = _lib.lib()
        ws_bytes = (lib.musc_b200_refine_bytes(n_images, query_rows, channels) if workspace_bytes is None
                    else int(workspace_bytes))
        ws = _aligned_empty(ws_bytes, dev)
        st = lib.musc_b200_refine(_ptr(bank), rows if bank_rows is None else bank_rows, rows, channels, patches,
                                  first_row, query_rows, rank_hi, _ptr(k1), _ptr(m2), parts, n_images * table_rows,
                                  table_rows, _ptr(out), _ptr(ws), ws_bytes, _stream(dev))
        _lib.check(st, 'musc_b200_refine')
    return out


def nearest_pool(bank: torch.Tensor, rows: int, channels: int, patches: int, part: int = 0,
                 parts: int = 1, rows_per_block: int | None = None,
                 out: torch.Tensor | None = None, bank_rows: int | None = None,
                 max_ctas: int = 0) -> torch.Tensor:
    """Symmetric pool minima: ``(blocks, n_images, rows_per_block)`` squared, FLT_MAX where unset.

    Evaluates part ``part`` of ``parts`` of the pool's symmetric tile list;
    with one part the single block is the full ``(n_images, rows)`` table.
    ``out`` must come from :func:`nearest_pool_table` (it carries the scheduler word).
    ``bank_rows``: the row count the bank is laid out for (a padded gathered bank).
    ``max_ctas``: cap on the persistent grid (0 = one CTA per SM; the default CTA-pair
    kernel rounds it down to an even count).
    """
    dev = bank.device
    rpb = rows if rows_per_block is None else rows_per_block
    if out is None:
        out = nearest_pool_table(rows, patches, rpb, dev)
    need = _lib.lib().musc_b200_nearest_pool_bytes(rows, patches, rpb)
    have = out.untyped_storage().nbytes() - out.storage_offset() * out.element_size()
    if not out.is_contiguous() or have < need:
        raise ValueError('nearest_pool: out must be a contiguous table from nearest_pool_table()')
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_nearest_pool(_ptr(bank), rows if bank_rows is None else bank_rows, rows,
                                               channels, patches, part, parts, rpb, int(max_ctas), _ptr(out),
                                               _stream(dev))
        _lib.check(st, 'musc_b200_nearest_pool')
    return out


def trimmed_mean(nearest_sq: torch.Tensor, rank_lo: int, rank_hi: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Interval average of ``sqrt(nearest_sq)`` over images -> ``(query_rows,)`` float64."""
    n_images, rows = nearest_sq.shape
    dev = nearest_sq.device
    if out is None:
        out = torch.empty(rows, dtype=torch.float64, device=dev)
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_trimmed_mean(_ptr(nearest_sq), rows, n_images, rank_lo, rank_hi,
                                               _ptr(out), _stream(dev))
        _lib.check(st, 'musc_b200_trimmed_mean')
    return out


def msm(Z: torch.Tensor, topmin_min: float = 0, topmin_max: float = 0.3) -> torch.Tensor:
    """Mutual scoring of one bank ``(N, P, C)`` fp32 -> ``(N, P)`` float64 (``_MSM.py:53-59``)."""
    if Z.ndim != 3 or not Z.is_cuda or Z.dtype != torch.float32:
        raise ValueError('Expected CUDA FP32 features with shape (N,P,C).')
    n, p, c = Z.shape
    if not (n >= 2 and p > 0 and c > 0):
        raise ValueError('Requires N>=2, P>0, C>0.')
    a, b = trimmed_ranks(n, topmin_min, topmin_max)
    dev = Z.device
    z = Z.contiguous()
    with torch.cuda.device(dev):
        lib = _lib.lib()
        ws_bytes = lib.musc_b200_msm_workspace_bytes(n, p, c)
        ws = _aligned_empty(ws_bytes, dev)
        scores = torch.empty(n, p, dtype=torch.float64, device=dev)
        st = lib.musc_b200_msm(_ptr(z), n, p, c, a, b, _ptr(scores), _ptr(ws), ws_bytes, _stream(dev))
        _lib.check(st, 'musc_b200_msm')
    return scores


# --------------------------------------------------------------------------- reduction
def score_maps(scores: torch.Tensor, image_size: int = 518, upsampled: bool = False):
    """``(R, L, N, P)`` float64 scores -> ``(maps (N, s, s), image_max (N,), up or None)``.

    ``models/musc.py:259-288``: layer mean, radius mean, bilinear
    align_corners=True up-sampling to ``image_size`` and the per-image max.
    """
    _require_cuda(scores, 'score_maps')
    if scores.ndim != 4 or scores.dtype != torch.float64:
        raise ValueError('score_maps: expected (R, L, N, P) float64')
    scores = scores.contiguous()
    r, l, n, p = scores.shape
    side = math.isqrt(p)
    if side * side != p:
        raise ValueError('score_maps: P must be a square')
    dev = scores.device
    maps = torch.empty(n, side, side, dtype=torch.float64, device=dev)
    image_max = torch.empty(n, dtype=torch.float64, device=dev)
    up = torch.empty(n, image_size, image_size, dtype=torch.float64, device=dev) if upsampled else None
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_score_maps(_ptr(scores), r, l, n, side, image_size, _ptr(maps),
                                             _ptr(image_max), _ptr(up), _stream(dev))
        _lib.check(st, 'musc_b200_score_maps')
    return maps, image_max, up


def rscin(image_scores: torch.Tensor, cls_tokens: torch.Tensor | None,
          k_list: Sequence[int] = (1, 2, 3)) -> torch.Tensor:
    """RsCIN refinement of the per-image scores -> a new ``(N,)`` float64 tensor.

    ``models/modules/_RsCIN.py:5-31``: the min-max normalised scores averaged over
    each image's k most similar images (class-token similarity ``T T^T``, k in
    ``k_list``), then the mean over ``k_list``; ``cls_tokens`` None or a 0 in
    ``k_list`` return a copy of the scores, as in the reference.
    """
    _require_cuda(image_scores, 'rscin')
    if image_scores.ndim != 1 or image_scores.dtype != torch.float64:
        raise ValueError('rscin: expected (N,) float64 image scores')
    n = image_scores.shape[0]
    dev = image_scores.device
    scores = image_scores.contiguous()
    if cls_tokens is not None:
        _require_cuda(cls_tokens, 'rscin')
        if cls_tokens.ndim != 2 or cls_tokens.shape[0] != n or cls_tokens.device != dev:
            raise ValueError('rscin: expected (N, dim) class tokens on the scores\' device')
        cls_tokens = cls_tokens.to(torch.float32).contiguous()
    ks = [int(k) for k in k_list]
    arr = (ctypes.c_int * max(len(ks), 1))(*ks)
    out = torch.empty(n, dtype=torch.float64, device=dev)
    dim = cls_tokens.shape[1] if cls_tokens is not None else 0
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_rscin(_ptr(cls_tokens), n, dim, _ptr(scores), len(ks), arr, _ptr(out), _stream(dev))
        _lib.check(st, 'musc_b200_rscin')
    return out


# --------------------------------------------------------------------------- attention
def add_layernorm(x: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, bias: torch.Tensor,
                  eps: float = 1e-5, out_dtype: torch.dtype = torch.float16,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """``x += delta`` (in place, fp32; skipped when ``delta`` is None) then
    ``layer_norm(x) * weight + bias`` in ``out_dtype`` (fp16 / bf16): the residual add and
    LayerNorm of a ViT block in one pass.  ``x`` ``(..., C)`` contiguous fp32 CUDA."""
    _require_cuda(x, 'add_layernorm')
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError('add_layernorm: x must be contiguous float32')
    c = x.shape[-1]
    rows = x.numel() // c
    if delta is not None:
        if delta.shape != x.shape or delta.dtype not in (torch.float16, torch.bfloat16) or not delta.is_contiguous():
            raise ValueError('add_layernorm: delta must be a contiguous fp16/bf16 tensor of x\'s shape')
    if out_dtype not in (torch.float16, torch.bfloat16):
        raise ValueError('add_layernorm: out_dtype must be float16 or bfloat16')
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    w, b = weight.contiguous(), bias.contiguous()
    dev = x.device
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_add_layernorm(_ptr(x), _ptr(delta), _DTYPES[delta.dtype] if delta is not None else 0,
                                                _ptr(w), _ptr(b), float(eps), _ptr(out), _DTYPES[out_dtype], rows, c,
                                                _stream(dev))
        _lib.check(st, 'musc_b200_add_layernorm')
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """``softmax(q k^T * scale) v`` per head for token-major ``(B, L, heads*64)`` views.

    ``q``, ``k``, ``v`` (fp16 or bf16, one type) may be column slices of one packed QKV
    projection (same row stride); the result is ``(B, L, heads*64)`` in that type.
    """
    _require_cuda(q, 'attention')
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError('attention: q, k, v must all be float16 or all bfloat16')
    if q.ndim != 3 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError('attention: q, k, v must share shape (B, L, heads*head_dim)')
    b, length, width = q.shape
    head_dim = width // heads
    if head_dim * heads != width:
        raise ValueError('attention: width must be heads * head_dim')
    for t in (q, k, v):
        if t.stride(2) != 1 or t.stride(0) != length * t.stride(1) or t.stride(1) != q.stride(1):
            raise ValueError('attention: q, k, v must be token-major with one common row stride')
    if out is None:
        out = torch.empty(b, length, width, dtype=q.dtype, device=q.device)
    scale = head_dim ** -0.5 if scale is None else scale
    dev = q.device
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_attention_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _DTYPES[q.dtype], b,
                                                length, heads,
                                                head_dim, q.stride(1), out.stride(1), float(scale),
                                                _stream(dev))
        _lib.check(st, 'musc_b200_attention_fwd')
    return out


OPENAI_MEAN = (0.48145466, 0.4578275, 0.40821073)
OPENAI_STD = (0.26862954, 0.26130258, 0.27577711)
_FILTERS = {'bicubic': _lib.BICUBIC, 'bilinear': _lib.BILINEAR}


def preprocess_workspace_bytes(in_h: int, in_w: int, out_h: int, out_w: int, filter: str = 'bicubic') -> int:
    if filter not in _FILTERS:
        raise ValueError("preprocess_images: filter must be 'bicubic' or 'bilinear'")
    n = _lib.lib().musc_b200_preprocess_workspace_bytes(in_h, in_w, out_h, out_w, _FILTERS[filter])
    if n == 0:
        raise ValueError(f'preprocess_images: unsupported sizes {in_h}x{in_w} -> {out_h}x{out_w}')
    return n


def preprocess_images(images: torch.Tensor, size: int | tuple[int, int] = 518, filter: str = 'bicubic',
                      mean: Sequence[float] = OPENAI_MEAN, std: Sequence[float] = OPENAI_STD,
                      out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None,
                      workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's evaluation transform on the device: ``(B, H, W, 3)`` uint8 RGB ->
    ``(B, 3, size, size)`` -- Pillow's antialiased resize (bicubic, or bilinear), ToTensor,
    Normalize -- bit for bit with ``open_clip/transform.py:124-133`` for fp32 output.

    ``images`` may be a batch view whose images are evenly spaced in memory with contiguous
    rows (e.g. a slice of a larger staging buffer)."""
    _require_cuda(images, 'preprocess_images')
    if images.dtype != torch.uint8 or images.ndim != 4 or images.shape[-1] != 3:
        raise ValueError('preprocess_images: images must be a (B, H, W, 3) uint8 tensor')
    b, h, w, _ = images.shape
    if images.stride()[1:] != (3 * w, 3, 1):
        raise ValueError('preprocess_images: each image must be H x W x 3 with contiguous rows')
    out_h, out_w = (size, size) if isinstance(size, int) else (int(size[0]), int(size[1]))
    if out_dtype not in _DTYPES:
        raise ValueError('preprocess_images: out_dtype must be float32, float16 or bfloat16')
    if len(mean) != 3 or len(std) != 3:
        raise ValueError('preprocess_images: mean and std need 3 values')
    dev = images.device
    if out is None:
        out = torch.empty((b, 3, out_h, out_w), dtype=out_dtype, device=dev)
    elif out.shape != (b, 3, out_h, out_w) or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError('preprocess_images: out must be a contiguous (B, 3, out_h, out_w) tensor of out_dtype')
    ws_bytes = preprocess_workspace_bytes(h, w, out_h, out_w, filter)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    m = (ctypes.c_float * 3)(*[float(v) for v in mean])
    s = (ctypes.c_float * 3)(*[float(v) for v in std])
    stride = images.stride(0) if b > 1 else 3 * h * w
    with torch.cuda.device(dev):
        st = _lib.lib().musc_b200_preprocess_images(_ptr(images), b, h, w, stride, out_h, out_w, _FILTERS[filter],
                                                    m, s, _DTYPES[out_dtype], _ptr(out), _ptr(workspace),
                                                    workspace.numel(), _stream(dev))
        _lib.check(st, 'musc_b200_preprocess_images')
    return out
