"""Host-side logic of the b200 backend that runs without a GPU."""
from __future__ import annotations

from copy import deepcopy
from types import SimpleNamespace

import pytest
import torch

from musc_b200 import backend, ops
from musc_b200.pipeline import shard_range
from oracle import msm as omsm


@pytest.mark.parametrize('n', [2, 5, 16, 100, 200, 1024])
@pytest.mark.parametrize('lo,hi', [(0, 0.3), (0.1, 0.5), (0, 0.9), (0.3, 0)])
def test_trimmed_ranks_match_oracle(n, lo, hi):
    try:
        want = omsm.trimmed_ranks(n, lo, hi)
    except Exception:  # pragma: no cover
        want = None
    if want is None or not (0 <= want[0] < want[1] <= n - 1):
        with pytest.raises(ValueError, match='trimmed ranks'):
            ops.trimmed_ranks(n, lo, hi)
    else:
        assert ops.trimmed_ranks(n, lo, hi) == want


@pytest.mark.parametrize('n', [1, 7, 100, 1024])
@pytest.mark.parametrize('world', [1, 2, 3, 8])
def test_shard_range_partitions_contiguously(n, world):
    seen = []
    for rank in range(world):
        first, end, per = shard_range(n, world, rank)
        assert per == -(-n // world) and first == min(n, rank * per) and end - first <= per
        seen.extend(range(first, end))
    assert seen == list(range(n))


def test_b200_backend_never_falls_back():
    with pytest.raises(RuntimeError, match='no CPU fallback'):
        backend.select_backend('b200', 'cpu')
    with pytest.raises(ValueError, match='inference_backend must be'):
        backend.select_backend('fastest', 'cuda')
    # the reference's own names keep the reference's fallback behaviour
    assert backend.select_backend('original', 'cpu') == ('original', None)
    assert backend.select_backend('gpu', 'cuda', 'posix')[0] == 'original'


def test_super_fast_preset_requires_cuda_and_is_isolated():
    cfg = {'models': dict(inference_backend='b200_super_fast', backbone_name='ViT-L-14-336',
                          pretrained='openai', batch_size=4, feature_layers=[5, 11, 17, 23],
                          r_list=[1, 3, 5]),
           'datasets': dict(img_resize=518, divide_num=1)}
    with pytest.raises(RuntimeError):
        backend.configure_backend(cfg, 'cpu')
    plain = deepcopy(cfg)
    plain['models']['inference_backend'] = 'b200'
    assert backend.configure_backend(plain, 'cpu') is plain


def test_msm_contract_errors_match_reference():
    """Same messages as models/modules/_MSM_gpu.py:702-711."""
    with pytest.raises(ValueError, match='Expected CUDA FP32 features'):
        backend.MSM(torch.zeros(4, 9, 8))
    with pytest.raises(ValueError, match='Expected CUDA FP32 features'):
        backend.MSM(torch.zeros(4, 9))


def test_aggregation_rejects_bad_layers():
    layer = SimpleNamespace(r=2, patch_maker=SimpleNamespace(stride=1),
                            LNA=SimpleNamespace(output_dim=8, preprocessing_modules=[0]))
    with pytest.raises(ValueError, match='r must be'):
        backend.aggregate_features(layer, [torch.zeros(1, 10, 8)])
    layer.r = 3
    with pytest.raises(ValueError, match='1 \\+ side'):
        backend.aggregate_features(layer, [torch.zeros(1, 11, 8)])
