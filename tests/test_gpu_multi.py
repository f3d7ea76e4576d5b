"""Multi-GPU parity: the sharded pipeline on 2 GPUs against the reference's golden pool.

Each rank aggregates its query images, the banks are gathered, every rank screens its
part of the symmetric tiles, the partial screen tables of each rank's rows are exchanged
and refined.  Both transports are checked -- NCCL collectives, and peer copies on copy
engines ordered by device-memory flags (``musc_b200.exchange``), over two pool steps so
the flags' counters carry across calls.  The gathered maps and image maxima must match
the reference (config 1, N=16) within 2e-5 relative, and the two transports must agree
bit for bit.  Skipped when fewer than 2 GPUs are visible.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
RTOL = 2e-5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank(rank, world, port, queue):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / 'musc-gpu_b200'), str(repo / 'tests')]
    import torch.distributed as dist
    from conftest import golden
    from musc_b200.pipeline import gather_pool, score_pool, shard_range
    from musc_b200.synthetic import prototype_mixture
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
    dev = torch.device('cuda', rank)
    torch.cuda.set_device(dev)
    dist.init_process_group('nccl', rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = golden('pool16')
        n = int(g['n'])
        tokens = prototype_mixture(n, n_layers=4, c=1024, side=37, seed=int(g['seed']))
        from musc_b200.exchange import PeerExchange
        first, end, _ = shard_range(n, world, rank)
        mine = [t[first:end].to(dev) for t in tokens]
        res = score_pool(mine, n_images=n, group=dist.group.WORLD)
        maps, mx = gather_pool(res, dist.group.WORLD)
        ex = PeerExchange(dist.group.WORLD, dev, n, 1369, 1024)
        copies = []
        for _ in range(2):                       # two steps: counters carry across calls
            r2 = score_pool(mine, n_images=n, group=dist.group.WORLD, exchange=ex, verify=True)
            m2, x2 = gather_pool(r2, dist.group.WORLD)
            copies.append((m2.cpu().numpy(), x2.cpu().numpy(), r2.verified))
        ex.close()
        if rank == 0:
            queue.put((maps.cpu().numpy(), mx.cpu().numpy(), copies))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2])
def test_sharded_pool16_matches_reference(cuda_device, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')
    import torch.multiprocessing as mp
    from conftest import golden
    g = golden('pool16')
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    maps, mx, copies = queue.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    np.testing.assert_allclose(maps, g['maps'], rtol=RTOL, atol=0)
    np.testing.assert_allclose(mx, g['image_max'], rtol=RTOL, atol=0)
    for m2, x2, verified in copies:
        np.testing.assert_array_equal(m2, maps)
        np.testing.assert_array_equal(x2, mx)
        assert verified['bit_exact']
