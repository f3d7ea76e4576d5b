"""Host logic of the device image loader (no GPU): ordering, bounded prefetch, worker
errors and argument checks, as ``models/modules/_loader.py:8-43`` defines them."""
from __future__ import annotations

import threading

import numpy as np
import pytest


class _Items:
    def __init__(self, n, fail_at=None):
        self.n, self.fail_at = n, fail_at
        self.lock = threading.Lock()
        self.started = []

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        with self.lock:
            self.started.append(i)
        if i == self.fail_at:
            raise KeyError(f'item {i}')
        return {'image': np.full((2, 3, 3), i, dtype=np.uint8), 'is_anomaly': i % 2}


@pytest.mark.parametrize('n,batch,workers,prefetch', [(0, 4, 4, 2), (1, 4, 4, 2), (10, 4, 3, 2), (9, 3, 1, 1),
                                                      (7, 8, 2, 3)])
def test_ordered_batches_keep_dataset_order(n, batch, workers, prefetch):
    from musc_b200.loader import ordered_batches
    items = _Items(n)
    batches = list(ordered_batches(items, batch, workers, prefetch))
    assert [len(b) for b in batches] == [min(batch, n - i) for i in range(0, n, batch)]
    flat = [int(s['image'][0, 0, 0]) for b in batches for s in b]
    assert flat == list(range(n))


def test_ordered_batches_bound_items_in_flight():
    from musc_b200.loader import ordered_batches
    items = _Items(40)
    seen = 0
    for b in ordered_batches(items, 4, 4, 2):
        seen += len(b)
        # never more than batch_size * prefetch_batches submitted beyond what was consumed
        assert len(items.started) <= seen + 4 * 2


def test_ordered_batches_raise_worker_errors():
    from musc_b200.loader import ordered_batches
    with pytest.raises(KeyError, match='item 5'):
        for _ in ordered_batches(_Items(12, fail_at=5), 4, 2, 2):
            pass


def test_loader_checks_arguments_like_the_reference():
    from musc_b200.loader import DeviceImageLoader
    for kw in ({'batch_size': 0}, {'workers': 0}, {'prefetch_batches': 0}):
        with pytest.raises(ValueError, match='Loader sizes must be positive'):
            DeviceImageLoader(_Items(3), device='cpu', **kw)
    with pytest.raises(ValueError, match='filter'):
        DeviceImageLoader(_Items(3), device='cpu', filter='lanczos')
    loader = DeviceImageLoader(_Items(10), batch_size=4, device='cpu')
    assert len(loader) == 3
    loader.close()   # nothing started: no-op


def test_raw_rgb_converts_modes():
    from PIL import Image
    from musc_b200.loader import RawRGB
    gray = Image.fromarray(np.arange(12, dtype=np.uint8).reshape(3, 4))
    arr = RawRGB()(gray)
    assert arr.shape == (3, 4, 3) and arr.dtype == np.uint8
    assert np.array_equal(arr[..., 0], np.arange(12, dtype=np.uint8).reshape(3, 4))


def test_preprocess_query_rejects_unsupported_sizes():
    from musc_b200 import ops
    assert ops.preprocess_workspace_bytes(900, 900, 518, 518) > 518 * 9 * 4 * 2
    with pytest.raises(ValueError):
        ops.preprocess_workspace_bytes(10000, 900, 518, 518)   # more than 15.75x on one side
    with pytest.raises(ValueError):
        ops.preprocess_workspace_bytes(0, 900, 518, 518)
    with pytest.raises(ValueError):
        ops.preprocess_workspace_bytes(900, 900, 518, 518, 'lanczos')
