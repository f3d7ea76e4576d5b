"""Device-resident pool scoring: LNAMD -> MSM -> score reduction, 1..G GPUs.

This is the scoring half of ``MuSc.make_category_data``
(``models/musc.py:224-288``) with every stage on the B200:

* per layer, one LNAMD launch produces the L2-normalised banks of all radii
  (``models/musc.py:227-245``; the bank assembly ``Z = cat(Z_layers[l])`` of
  ``:252`` is the output layout itself);
* per (radius, layer) bank, MSM (``:248-262``) = the bank prep (centred on the
  pool's column mean: same distances, tighter split-fp16 bounds), the fused
  distance/min GEMM and the interval average;
* layer and radius means, up-sampling and image maxima (``:259-288``).

Each bank's MSM is the screened symmetric pass (one fp16 MMA pass over every
unordered pair of patches from different images) followed by the refinement
to exact minima of the pairs that can reach the trimmed ranks (the reference
GPU driver's rank-deferred scheme, ``models/modules/_MSM_gpu.py:739-786``);
``MUSC_B200_MSM_EXACT=1`` selects the 3-pass exact kernel for every pair.

Multi-GPU (one process per GPU): rank r owns the query images
``[r*ceil(N/G), ...)`` and aggregates only those; each bank is all-gathered
over NCCL (overlapped with the previous bank's work), every rank screens a
balanced share of the pool's symmetric distance tiles into tables blocked by
the rows' owners, and an all-to-all hands each rank the partial tables of its
own query rows, which it refines.  The reference is single-device; the
sharding is this library's addition.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import torch

from . import ops


def shard_range(n_images: int, world: int, rank: int) -> tuple[int, int, int]:
    """``(first, end, per)``: rank's query images ``[first, end)``, ``per = ceil(N/G)``.

    Ranks take ``per`` images each in order, so the gathered, per-padded banks
    hold the pool contiguously in their first ``N`` images.
    """
    if n_images <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError('shard_range: requires N > 0, world > 0, 0 <= rank < world')
    per = -(-n_images // world)
    first = min(n_images, rank * per)
    end = min(n_images, first + per)
    return first, end, per


@dataclass
class PoolScores:
    scores: torch.Tensor      # (R, L, n_local, P) float64, this rank's query images
    maps: torch.Tensor        # (n_local, side, side) float64
    image_max: torch.Tensor   # (n_local,) float64
    first_image: int
    n_images: int
    verified: dict | None = None   # sharded-vs-whole check of the last bank (``verify=True``)


def score_pool(tokens: Sequence[torch.Tensor], n_images: int | None = None,
               radii: Sequence[int] = (1, 3, 5), topmin_min: float = 0, topmin_max: float = 0.3,
               image_size: int = 518, super_fast_side: int | None = None,
               group=None, kernels=ops, ready: Sequence | None = None,
               collective_sms: int = 0, verify: bool = False, exchange=None) -> PoolScores:
    """Score one pool from device-resident tokens.

    ``tokens``: per hooked layer, this rank's ``(n_local, 1+P, C)`` tokens
    (all ``N`` images when running on one GPU).  ``super_fast_side``: if set,
    the super-fast profile (r=3 LNAMD, adaptive pooling to that side).
    ``group``: a ``torch.distributed`` process group (None = single GPU).
    ``kernels``: the operator set (``musc_b200.ops``, the CUDA library); the
    CPU tests of the sharding logic substitute the numpy oracle here.
    ``ready``: optional per-layer CUDA events (e.g. the end of each layer's
    host-to-device copy on another stream); the current stream waits on layer
    l's event just before that layer's LNAMD, so later layers' copies overlap
    the scoring of earlier ones.  Banks are processed layer by layer.
    ``collective_sms``: with a process group, SMs left free during each bank's
    GEMM so the neighbouring banks' gather and exchange run alongside it
    (0 = none, the default: the GEMM's dynamic tile scheduler already lets a
    collective that starts first keep its SMs).
    ``exchange``: with a process group, a :class:`musc_b200.exchange.PeerExchange` of this
    pool's shape: the banks and the screen tables then move between the GPUs by peer
    copies on copy engines (no SMs, overlapping the GEMMs) instead of NCCL collectives.
    ``verify``: with a process group, re-score the last bank on every rank as one
    whole-pool part from the gathered bank and compare the rows each rank owns
    with the sharded result, bit for bit; the outcome (summed over ranks) is in
    ``PoolScores.verified``.  Off the timed path: it costs one more bank.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group) if group is not None else 1
    rank = dist.get_rank(group) if group is not None else 0
    first_tok = tokens[0]
    dev = first_tok.device
    n_local, length, c = first_tok.shape
    if n_images is None:
        n_images = n_local * world if world == 1 else None
        if n_images is None:
            raise ValueError('score_pool: n_images is required with a process group')
    first, end, per = shard_range(n_images, world, rank)
    if end - first != n_local:
        raise ValueError(f'score_pool: rank {rank} holds {n_local} images, expected {end - first}')
    a, b = kernels.trimmed_ranks(n_images, topmin_min, topmin_max)
    if super_fast_side is not None:
        radii = (3,)
        p = super_fast_side * super_fast_side
    else:
        p = length - 1
    side = math.isqrt(p)
    n_r, n_l = len(radii), len(tokens)

    # 1. LNAMD of the local images into the R radii banks of one layer, padded to `per`
    #    images (only the padding is zeroed: it is gathered but never scored).  Layer l+1's
    #    LNAMD overwrites them; every bank of layer l is prepared (stream-ordered) before it.
    local = torch.empty(n_r, per, p, c, dtype=torch.float32, device=dev)   # one layer's radii at a time
    if per > n_local:
        local[:, n_local:].zero_()
    done = [False] * n_l

    def aggregate(li: int) -> None:
        if done[li]:
            return
        done[li] = True
        if ready is not None and ready[li] is not None and dev.type == 'cuda':
            torch.cuda.current_stream(dev).wait_event(ready[li])
        if n_local == 0:
            return
        t = tokens[li]
        if super_fast_side is not None:
            kernels.lnamd_super_fast(t, super_fast_side, True, out=local[0, :n_local],
                                     image_stride=p * c, patch_stride=c)
        else:
            kernels.lnamd(t, radii, True, out=[local[ri, :n_local] for ri in range(n_r)])

    # 2. Per bank: prep, (gather), symmetric nearest minima, interval average.
    #    One GPU: prep the whole bank, one symmetric launch, select.
    #    G GPUs: each rank preps the bank of its own rows; the five bank planes are
    #    all-gathered into a padded pool bank (the next bank's gather overlaps this
    #    bank's GEMM); rank r screens part r of the symmetric tile list into tables
    #    whose blocks are the ranks' query rows; an all-to-all (overlapping the next
    #    bank's GEMM) hands each rank the partial tables of its own rows to refine.
    banks = [(li, ri) for li in range(n_l) for ri in range(n_r)]
    verified = None
    scores = torch.empty(n_r, n_l, n_local, p, dtype=torch.float64, device=dev)
    rows = n_images * p
    q_rows = n_local * p
    rpb = per * p if world > 1 else rows

    def select(near: torch.Tensor, li: int, ri: int) -> None:
        # near: (N, width) table whose first q_rows columns are this rank's rows
        if q_rows == 0:
            return
        if near.shape[1] == q_rows:
            kernels.trimmed_mean(near, a, b, out=scores[ri, li].view(-1))
        else:
            tmp = torch.empty(near.shape[1], dtype=torch.float64, device=dev)
            kernels.trimmed_mean(near, a, b, out=tmp)
            scores[ri, li].view(-1).copy_(tmp[:q_rows])

    exact_path = exact_pool_path()
    if world == 1:
        bank = kernels.empty_bank(rows, c, dev)
        stats = torch.empty(c + 1, dtype=torch.float64, device=dev)
        if exact_path:
            table = kernels.nearest_pool_table(rows, p, rows, dev)
        else:
            screen = kernels.screen_table(rows, p, rows, dev)
            table = torch.empty(1, n_images, rows, dtype=torch.float32, device=dev)
        for li, ri in banks:
            aggregate(li)
            z = local[ri, :n_images].reshape(rows, c)
            kernels.prep_bank(z, out=bank, stats=kernels.center_stats(z, out=stats), count=rows)
            if exact_path:
                kernels.nearest_pool(bank, rows, c, p, 0, 1, rows, out=table)
            else:
                kernels.screen_pool(bank, rows, c, p, 0, 1, rows, out=screen)
                kernels.refine(bank, rows, c, p, 0, rows, b, screen[0], screen[1], out=table[0])
            select(table[0], li, ri)
    elif exchange is not None and not exact_path:
        if not exchange.matches(n_images, p, c, world):
            raise ValueError('score_pool: the exchange was created for another pool shape')
        verified = _score_with_exchange(kernels, exchange, banks, aggregate, local, select, rows, c, p, rank,
                                        world, first, q_rows, a, b, scores, verify, group, n_images)
    else:
        local_rows, bank_rows = per * p, world * per * p
        sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == 'cuda' else 0
        max_ctas = max(1, sms - collective_sms) if (sms and collective_sms) else 0
        # The gathers run on their own communicator (own NCCL stream), so bank k+1's gather
        # is never queued behind bank k-1's exchange, which must wait for GEMM k-1.
        gather_group = _side_group(group)
        local_bank = [kernels.empty_bank(local_rows, c, dev) for _ in range(2)]
        full_bank = [kernels.empty_bank(bank_rows, c, dev) for _ in range(3)]
        stats_local = [torch.empty(c + 1, dtype=torch.float64, device=dev) for _ in range(2)]
        stats_all = [torch.empty(world, c + 1, dtype=torch.float64, device=dev) for _ in range(2)]

        def start_gather(k):
            li, ri = banks[k]
            aggregate(li)
            # every rank centres on the same mean: the ranks' statistics (over their real
            # rows, not the padding), gathered
            kernels.center_stats(local[ri, :n_local].reshape(-1, c), out=stats_local[k % 2])
            dist.all_gather_into_tensor(stats_all[k % 2].view(-1), stats_local[k % 2], group=gather_group)
            kernels.prep_bank(local[ri].reshape(local_rows, c), out=local_bank[k % 2], stats=stats_all[k % 2],
                              count=rows)
            pieces = zip(kernels.bank_planes(full_bank[k % 3], bank_rows, c),
                         kernels.bank_planes(local_bank[k % 2], local_rows, c))
            return [dist.all_gather_into_tensor(f, l, group=gather_group, async_op=True) for f, l in pieces]

        if exact_path:
            tables = [kernels.nearest_pool_table(rows, p, rpb, dev, min_blocks=world) for _ in range(3)]
            mine = [torch.empty(n_images, rpb, dtype=torch.float32, device=dev) for _ in range(3)]
        else:
            # Each rank screens part r of the symmetric tiles into tables blocked by the
            # rows' owners; an all-to-all hands every rank the partial tables of its own
            # rows, which the refinement combines (not a plain minimum: the second minimum
            # also takes the partial minima that lose).
            screens = [kernels.screen_table(rows, p, rpb, dev, min_blocks=world) for _ in range(2)]
            recv = [(torch.empty(world, n_images, rpb, dtype=torch.int64, device=dev),
                     torch.empty(world, n_images, rpb, dtype=torch.int32, device=dev)) for _ in range(2)]
            exact_t = torch.empty(n_images, max(q_rows, 1), dtype=torch.float32, device=dev)

            def start_exchange(k):
                k1, m2, _ = screens[k % 2]
                rk, rm = recv[k % 2]
                return [dist.all_to_all_single(rk, k1[:world], group=group, async_op=True),
                        dist.all_to_all_single(rm, m2[:world], group=group, async_op=True)]

            def finish_bank(k, works):
                for w in works:
                    w.wait()
                if q_rows:
                    rk, rm = recv[k % 2]
                    kernels.refine(full_bank[k % 3], rows, c, p, first * p, q_rows, b, rk, rm, out=exact_t,
                                   bank_rows=bank_rows)
                    select(exact_t, *banks[k])

        gathers = {0: start_gather(0)}
        pending = []   # (finish, k): reduce-scatter or exchange in flight
        for k, (li, ri) in enumerate(banks):
            if k + 1 < len(banks):
                gathers[k + 1] = start_gather(k + 1)
            for w in gathers.pop(k):
                w.wait()
            if exact_path:
                kernels.nearest_pool(full_bank[k % 3], rows, c, p, rank, world, rpb, out=tables[k % 3],
                                     bank_rows=bank_rows, max_ctas=max_ctas)
                pending.append((_min_reduce_scatter(tables[k % 3], mine[k % 3], rank, group), k))
                if len(pending) > 2:
                    finish, kk = pending.pop(0)
                    finish()
                    select(mine[kk % 3], *banks[kk])
            else:
                kernels.screen_pool(full_bank[k % 3], rows, c, p, rank, world, rpb, out=screens[k % 2],
                                    bank_rows=bank_rows, max_ctas=max_ctas)
                pending.append((start_exchange(k), k))
                if len(pending) > 1:
                    works, kk = pending.pop(0)
                    finish_bank(kk, works)
        for item, kk in pending:
            if exact_path:
                item()
                select(mine[kk % 3], *banks[kk])
            else:
                finish_bank(kk, item)
        if verify:
            verified = _verify_last_bank(kernels, full_bank[(len(banks) - 1) % 3], bank_rows, rows, c, p,
                                         n_images, first, q_rows, a, b, scores[banks[-1][1], banks[-1][0]],
                                         banks[-1], group, exact_path)

    # 3. Layer/radius means, up-sampling, image maxima for the local images.
    if n_local:
        maps, image_max, _ = kernels.score_maps(scores, image_size)
    else:
        maps = torch.empty(0, side, side, dtype=torch.float64, device=dev)
        image_max = torch.empty(0, dtype=torch.float64, device=dev)
    return PoolScores(scores, maps, image_max, first, n_images, verified)


def _score_with_exchange(kernels, ex, banks, aggregate, local, select, rows, c, p, rank, world, first, q_rows,
                         a, b, scores, verify, group, n_images):
    """The multi-GPU bank loop over peer copies.  Compute-stream order per bank k:
    prep k+1 (its copies then run under GEMM k), wait for bank k's copies, screen k, the
    refinement of bank k-1 (its table copies ran under GEMM k), and so on."""
    dev = scores.device
    compute = torch.cuda.current_stream(dev)
    exact_t = torch.empty(n_images, max(q_rows, 1), dtype=torch.float32, device=dev)

    def start(k):
        li, ri = banks[k]
        aggregate(li)
        v = ex.begin_bank()
        stats = ex.center(v, compute, local[ri].reshape(ex.local_rows, c)[:q_rows], kernels)
        lb = ex.local_bank_for(v, compute)
        kernels.prep_bank(local[ri].reshape(ex.local_rows, c), out=lb, stats=stats, count=rows)
        full, events = ex.gather(v, compute)
        return v, k, full, events

    def finish(item):
        v, k, full, k1, m2, events = item
        for e in events:
            compute.wait_event(e)
        if q_rows:
            kernels.refine(full, rows, c, p, first * p, q_rows, b, k1, m2, out=exact_t, bank_rows=ex.bank_rows)
            select(exact_t, *banks[k])
        ex.release(v, compute)

    cur = start(0)
    pending = None
    for k in range(len(banks)):
        nxt = start(k + 1) if k + 1 < len(banks) else None
        v, _, full, events = cur
        for e in events:
            compute.wait_event(e)
        scr = ex.screen_for(v, compute)
        kernels.screen_pool(full, rows, c, p, rank, world, ex.rpb, out=scr, bank_rows=ex.bank_rows)
        k1, m2, xevents = ex.exchange(v, compute)
        if pending is not None:
            finish(pending)
        pending = (v, k, full, k1, m2, xevents)
        cur = nxt
    finish(pending)
    if not verify:
        return None
    # the last bank's pool bank stays intact until the next call's third bank
    return _verify_last_bank(kernels, ex.full_bank[pending[0] % 3], ex.bank_rows, rows, c, p, n_images, first,
                             q_rows, a, b, scores[banks[-1][1], banks[-1][0]], banks[-1], group, False)


def _verify_last_bank(kernels, bank, bank_rows, rows, c, p, n_images, first, q_rows, a, b, got, bank_id, group,
                      exact_path):
    """Every rank scores the gathered bank as one part (the single-GPU computation) and
    compares its own query rows with the sharded scores ``got``; counts summed over ranks."""
    import torch.distributed as dist
    dev = got.device
    mism = torch.zeros(3, dtype=torch.float64, device=dev)
    if q_rows:
        if exact_path:
            whole = kernels.nearest_pool(bank, rows, c, p, 0, 1, rows, bank_rows=bank_rows)[0]   # (N, rows)
            mine = whole[:, first * p:first * p + q_rows].contiguous()
        else:
            k1, m2, _ = kernels.screen_pool(bank, rows, c, p, 0, 1, rows, bank_rows=bank_rows)
            k1 = k1[:, :, first * p:first * p + q_rows].contiguous()
            m2 = m2[:, :, first * p:first * p + q_rows].contiguous()
            mine = kernels.refine(bank, rows, c, p, first * p, q_rows, b, k1, m2, bank_rows=bank_rows)
        ref = kernels.trimmed_mean(mine, a, b)
        sharded = got.reshape(-1)
        diff = (ref - sharded).abs()
        mism[0] = (ref != sharded).sum()
        mism[1] = diff.max()
        mism[2] = q_rows
    dist.all_reduce(mism[0:1], group=group)
    dist.all_reduce(mism[1:2], op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(mism[2:3], group=group)
    bad, worst, checked = mism.tolist()
    return {'bank': {'layer': bank_id[0], 'radius_index': bank_id[1]}, 'rows_checked': int(checked),
            'rows_differing': int(bad), 'max_abs_diff': worst, 'bit_exact': bad == 0}


def exact_pool_path() -> bool:
    """``MUSC_B200_MSM_EXACT=1``: score every bank with the 3-pass exact kernel instead of the
    screen + refinement (the same switch as the C library's ``musc_b200_msm``)."""
    import os
    return os.environ.get('MUSC_B200_MSM_EXACT', '0') == '1'


_SIDE_GROUPS: dict = {}


def _side_group(group):
    """A second communicator over the same ranks (created once per group, collectively)."""
    import torch.distributed as dist
    key = id(group)
    if key not in _SIDE_GROUPS:
        ranks = dist.get_process_group_ranks(group)
        _SIDE_GROUPS[key] = dist.new_group(ranks=ranks, backend=dist.get_backend(group))
    return _SIDE_GROUPS[key]


def _min_reduce_scatter(table: torch.Tensor, out: torch.Tensor, rank: int, group):
    """Start an element-wise MIN over ranks of ``table`` (G, N, rpb) of which rank r keeps
    block r in ``out``; returns a callable that completes it (the stream then waits)."""
    import torch.distributed as dist
    if dist.get_backend(group) == 'nccl':
        work = dist.reduce_scatter_tensor(out, table[:dist.get_world_size(group)], op=dist.ReduceOp.MIN,
                                          group=group, async_op=True)
        return work.wait
    # gloo (CPU tests of the sharding logic) has no reduce-scatter
    work = dist.all_reduce(table, op=dist.ReduceOp.MIN, group=group, async_op=True)

    def finish():
        work.wait()
        out.copy_(table[rank])
    return finish


def gather_pool(result: PoolScores, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All ranks' ``maps`` and ``image_max`` concatenated in image order (every rank gets them)."""
    import torch.distributed as dist

    if group is None:
        return result.maps, result.image_max
    world = dist.get_world_size(group)
    _, _, per = shard_range(result.n_images, world, 0)
    side = result.maps.shape[-1] if result.maps.ndim == 3 else 0
    dev = result.image_max.device
    n_local = result.image_max.shape[0]
    maps = torch.zeros(per, side, side, dtype=torch.float64, device=dev)
    mx = torch.zeros(per, dtype=torch.float64, device=dev)
    maps[:n_local] = result.maps
    mx[:n_local] = result.image_max
    all_maps = torch.empty(world * per, side, side, dtype=torch.float64, device=dev)
    all_mx = torch.empty(world * per, dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(all_maps, maps, group=group)
    dist.all_gather_into_tensor(all_mx, mx, group=group)
    return all_maps[:result.n_images], all_mx[:result.n_images]
