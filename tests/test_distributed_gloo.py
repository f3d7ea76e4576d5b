"""Multi-rank sharding logic on CPU: world_size 2 (and 3) gloo ranks.

``musc_b200.pipeline.score_pool`` is run with the numpy oracle substituted for
the CUDA operator set, so the test exercises exactly the host logic of the
multi-GPU path -- the query-image partition, the per-rank LNAMD, the bank
all-gather, the split of the symmetric distance work into per-rank parts, the
MIN reduction of the nearest tables and the score assembly -- and checks the
gathered maps and image maxima against the single-process result bit for bit.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from musc_b200 import ops
from musc_b200.pipeline import gather_pool, score_pool, shard_range
from oracle import lnamd as olnamd
from oracle import reduce as oreduce

N_IMAGES, SIDE, C, LAYERS, RADII = 5, 7, 32, 2, (1, 3)


class OracleKernels:
    """The pipeline's operator set, evaluated by the numpy oracle on CPU tensors."""

    trimmed_ranks = staticmethod(ops.trimmed_ranks)

    @staticmethod
    def lnamd(tokens, radii, l2_normalize, out):
        for r, o in zip(radii, out):
            z = olnamd.bank(tokens.numpy(), r) if l2_normalize else olnamd.lnamd(tokens.numpy(), r)
            o.copy_(torch.from_numpy(z))

    @staticmethod
    def lnamd_super_fast(tokens, side, l2_normalize, out, image_stride, patch_stride):
        z = olnamd.lnamd_super_fast(tokens.numpy(), side)
        out.copy_(torch.from_numpy(olnamd.l2_normalize(z) if l2_normalize else z))

    @staticmethod
    def nearest_pool_table(rows, patches, rpb, device, min_blocks=1):
        return torch.empty(max(-(-rows // rpb), min_blocks), rows // patches, rpb)

    @staticmethod
    def empty_bank(rows, c, device):
        return torch.empty(rows, c)

    @staticmethod
    def bank_planes(bank, rows, c, layout_rows=None):
        return [bank[:rows].reshape(-1)]

    @staticmethod
    def center_stats(z, out=None):
        x = z.numpy().astype(np.float64)
        norms = (z.numpy() ** 2).sum(1)
        s = np.concatenate([x.sum(0), [norms.min() * (1 - 2 ** -20) if len(norms) else np.inf]])
        if out is None:
            return torch.from_numpy(s)
        out.copy_(torch.from_numpy(s))
        return out

    @staticmethod
    def prep_bank(z, out=None, stats=None, count=None):
        # the library's centring: fp32 mu from the fp64 sums of every part, applied when
        # |mu|^2 <= 4 x the smallest squared row norm of every part
        if stats is not None:
            st = stats.reshape(-1, z.shape[1] + 1)
            mu = (st[:, :-1].sum(0) / (z.shape[0] if count is None else count)).float()
            if float((mu.double() ** 2).sum()) <= 4 * float(st[:, -1].min()):
                z = z - mu
        if out is None:
            return z.clone()
        out[:z.shape[0]].copy_(z)
        return out

    @staticmethod
    def nearest_pool(bank, rows, c, p, part, parts, rpb, out=None, bank_rows=None, max_ctas=0):
        """Squared minima for the image pairs {i, j} with min(i, j) % parts == part."""
        n = rows // p
        if out is None:
            out = torch.empty(-(-rows // rpb), n, rpb)
        z = bank[:rows].numpy().reshape(n, p, c).astype(np.float64)
        out.fill_(float(np.finfo(np.float32).max))
        for i in range(n):
            for j in range(n):
                if i == j or min(i, j) % parts != part:
                    continue
                d2 = ((z[i][:, None, :] - z[j][None, :, :]) ** 2).sum(-1).min(1)  # rows of i vs image j
                for q in range(p):
                    row = i * p + q
                    out[row // rpb, j, row % rpb] = float(np.float32(d2[q]))
        return out

    @staticmethod
    def screen_table(rows, patches, rpb, device, min_blocks=1):
        blocks = max(-(-rows // rpb), min_blocks)
        n = rows // patches
        return (torch.empty(blocks, n, rpb, dtype=torch.int64), torch.empty(blocks, n, rpb, dtype=torch.int32),
                torch.empty(1, dtype=torch.int64))

    @staticmethod
    def screen_pool(bank, rows, c, p, part, parts, rpb, out=None, bank_rows=None, max_ctas=0):
        """The screen tables' contract for the pairs {i, j} with min(i, j) % parts == part:
        k1 = (bits of the smallest squared distance with the low 8 bits cleared) << 32 | patch,
        m2 = bits of the second smallest (low 8 bits cleared); -1 (all ones) where unset."""
        n = rows // p
        if out is None:
            out = OracleKernels.screen_table(rows, p, rpb, None)
        k1, m2, _ = out
        k1.fill_(-1)
        m2.fill_(-1)
        z = bank[:rows].numpy().reshape(n, p, c).astype(np.float64)
        for i in range(n):
            for j in range(n):
                if i == j or min(i, j) % parts != part:
                    continue
                d2 = ((z[i][:, None, :] - z[j][None, :, :]) ** 2).sum(-1).astype(np.float32)  # rows of i vs j
                bits = (d2.view(np.uint32) & np.uint32(0xFFFFFF00)).astype(np.int64)
                order = np.argsort(bits, axis=1, kind='stable')
                for q in range(p):
                    row = i * p + q
                    best, second = order[q, 0], order[q, 1] if p > 1 else None
                    key = (int(bits[q, best]) << 32) | int(best)
                    k1[row // rpb, j, row % rpb] = key - (1 << 64) if key >= (1 << 63) else key
                    if second is not None:
                        m2[row // rpb, j, row % rpb] = int(np.int64(bits[q, second]).astype(np.uint32).view(np.int32))
        return out

    @staticmethod
    def refine(bank, rows, c, p, first_row, q_rows, rank_hi, k1, m2, out=None, bank_rows=None):
        """Exact minima of the query rows (float32 identity as the oracle's nearest table),
        after checking that the partial screen tables combine to the exact argmin."""
        n = rows // p
        z = bank[:rows].numpy().reshape(n * p, c).astype(np.float64)
        if out is None:
            out = torch.empty(n, q_rows, dtype=torch.float32)
        k1u = k1.numpy().view(np.uint64)
        for q in range(q_rows):
            g = first_row + q
            img = g // p
            for j in range(n):
                if j == img:
                    out[j, q] = float(np.finfo(np.float32).max)
                    continue
                d2 = ((z[j * p:(j + 1) * p] - z[g]) ** 2).sum(-1)
                best = int(k1u[:, j, q].min() & np.uint64(0xFFFFFFFF))
                assert abs(d2[best] - d2.min()) <= 1e-6 * max(d2.min(), 1e-12) + 1e-12, 'combined argmin'
                out[j, q] = float(np.float32(d2.min()))
        return out

    @staticmethod
    def trimmed_mean(near, a, b, out=None):
        if out is None:
            out = torch.empty(near.shape[1], dtype=torch.float64)
        d = np.sort(np.sqrt(near.numpy().astype(np.float64)), axis=0)[a:b]
        out.copy_(torch.from_numpy(d.mean(axis=0).astype(np.float32).astype(np.float64)))
        return out

    @staticmethod
    def score_maps(scores, image_size):
        maps, mx = oreduce.image_scores(scores.numpy(), image_size)
        return torch.from_numpy(maps), torch.from_numpy(mx), None


def _tokens():
    g = torch.Generator().manual_seed(21)
    return [torch.randn(N_IMAGES, 1 + SIDE * SIDE, C, generator=g) for _ in range(LAYERS)]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, queue):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        first, end, _ = shard_range(N_IMAGES, world, rank)
        local = [t[first:end].contiguous() for t in _tokens()]
        res = score_pool(local, n_images=N_IMAGES, radii=RADII, image_size=40, group=dist.group.WORLD,
                         kernels=OracleKernels(), verify=True)
        maps, mx = gather_pool(res, dist.group.WORLD)
        if rank == 0:
            queue.put((maps.numpy(), mx.numpy(), res.scores.numpy(), res.verified))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 3])
def test_sharded_pool_equals_single_process(world):
    single = score_pool(_tokens(), radii=RADII, image_size=40, kernels=OracleKernels())
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    maps, mx, scores0, verified = queue.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    np.testing.assert_array_equal(maps, single.maps.numpy())
    np.testing.assert_array_equal(mx, single.image_max.numpy())
    first, end, _ = shard_range(N_IMAGES, world, 0)
    np.testing.assert_array_equal(scores0, single.scores.numpy()[:, :, first:end])
    # the in-run check the bench reports: every rank's rows of the last bank, re-scored as
    # one whole-pool part, equal the sharded scores bit for bit
    assert verified['bit_exact'] and verified['rows_differing'] == 0
    assert verified['rows_checked'] == N_IMAGES * SIDE * SIDE
