"""GPU parity: the sm_100a kernels against the reference's golden vectors and the oracle.

Tolerance (the north star's): per-patch and per-image scores within 2e-5
relative of the reference's ``original`` backend; identical ordering of the
per-image scores.  Where exact duplicate patches make a distance 0, both the
reference (``torch.cdist`` = sqrt(max(fp32 rounding noise, 1e-30))) and this
library produce sqrt of rounding noise, so those cases use 2e-3 absolute.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import lnamd as olnamd
from oracle import msm as omsm
from oracle import reduce as oreduce

pytestmark = pytest.mark.gpu
RTOL = 2e-5


def _cuda(x, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t.to(dtype) if dtype is not None else t


# --------------------------------------------------------------------------- LNAMD
@pytest.mark.parametrize('r', [1, 3, 5])
def test_lnamd_layers_match_reference(cuda_device, r):
    from musc_b200 import ops
    g = golden('lnamd_small')
    tokens = [_cuda(t, cuda_device) for t in g['tokens']]
    got = ops.lnamd_layers(tokens, r, l2_normalize=False).cpu().numpy()
    np.testing.assert_allclose(got, g[f'embed_r{r}'], rtol=1e-5, atol=2e-5)


@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16])
def test_lnamd_low_precision_tokens(cuda_device, dtype):
    from musc_b200 import ops
    g = golden('lnamd_small')
    t = _cuda(g['tokens'][1], cuda_device, dtype)
    outs = ops.lnamd(t, (1, 3, 5), l2_normalize=True)
    ref_tokens = t.float().cpu().numpy()
    for r, o in zip((1, 3, 5), outs):
        np.testing.assert_allclose(o.cpu().numpy(), olnamd.bank(ref_tokens, r), rtol=1e-4, atol=1e-5)


def test_lnamd_banks_pool16(cuda_device):
    """C = 1024, the regenerated config-1 tokens: normalised banks vs the reference's."""
    from musc_b200 import ops
    from musc_b200.synthetic import prototype_mixture
    g = golden('pool16')
    tokens = prototype_mixture(int(g['n']), n_layers=4, c=1024, side=37, seed=int(g['seed']))
    rows = torch.from_numpy(g['probe_rows'])
    for li in range(4):
        outs = ops.lnamd(tokens[li].to(cuda_device), (1, 3, 5), l2_normalize=True)
        for ri, o in enumerate(outs):
            got = o.reshape(-1, 1024)[rows.to(cuda_device)].cpu().numpy()
            np.testing.assert_allclose(got, g['bank_probe'][ri, li], rtol=1e-4, atol=2e-6)


def test_super_fast_matches_reference(cuda_device):
    from musc_b200 import ops
    g = golden('lnamd_small')
    t = _cuda(g['tokens'][0], cuda_device)
    got = ops.lnamd_super_fast(t, 28, l2_normalize=False).cpu().numpy()
    np.testing.assert_allclose(got, g['superfast'][:, :, 0, :], rtol=1e-5, atol=2e-5)


# --------------------------------------------------------------------------- MSM
@pytest.mark.parametrize('case', ['a', 'b', 'c', 'd', 'e'])
def test_msm_small_cases_match_reference(cuda_device, case):
    from musc_b200 import backend
    g = golden('msm_small')
    lo, hi = g[f'{case}_ranks']
    got = backend.MSM(_cuda(g[f'{case}_z'], cuda_device), cuda_device, lo, hi)
    assert got.dtype == torch.float64 and got.device == cuda_device
    want = g[f'{case}_scores']
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=RTOL,
                               atol=2e-3 if case in ('b', 'd') else 0)


@pytest.mark.parametrize('n,p,c', [(5, 49, 64), (9, 100, 32), (3, 300, 1024), (12, 1369, 64)])
def test_nearest_table_matches_oracle(cuda_device, n, p, c):
    from musc_b200 import ops
    gen = torch.Generator().manual_seed(n * 1000 + p)
    z = torch.randn(n, p, c, generator=gen)
    z = z / z.norm(dim=-1, keepdim=True)
    zd = z.to(cuda_device)
    bank = ops.prep_bank(zd.reshape(n * p, c))
    near = ops.nearest(bank, n * p, 0, bank, n * p, c, p)          # (n, n*p) squared
    got = near.t().sqrt().cpu().numpy()                            # (n*p, n)
    want = omsm.nearest_table(z.numpy())
    self_mask = np.zeros_like(want, dtype=bool)
    for i in range(n):
        self_mask[i * p:(i + 1) * p, i] = True
    assert np.all(near.t().cpu().numpy()[self_mask] == np.finfo(np.float32).max)
    np.testing.assert_allclose(got[~self_mask], want[~self_mask], rtol=1e-5, atol=1e-6)


def test_nearest_query_slices_are_bit_identical(cuda_device):
    """Sharded query rows (global self exclusion) reproduce the full table exactly."""
    from musc_b200 import ops
    n, p, c = 10, 100, 64
    z = torch.randn(n * p, c, generator=torch.Generator().manual_seed(3)).to(cuda_device)
    bank = ops.prep_bank(z)
    full = ops.nearest(bank, n * p, 0, bank, n * p, c, p)
    for first_img, count in [(0, 3), (3, 4), (7, 3)]:
        qb = ops.prep_bank(z[first_img * p:(first_img + count) * p])
        part = ops.nearest(qb, count * p, first_img * p, bank, n * p, c, p)
        assert torch.equal(part, full[:, first_img * p:(first_img + count) * p])


@pytest.mark.parametrize('n,p,c', [(6, 49, 64), (11, 1369, 64), (4, 300, 1024)])
def test_symmetric_pool_table_matches_directed(cuda_device, n, p, c):
    """Each unordered pair evaluated once gives the same minima as the directed kernel."""
    from musc_b200 import ops
    z = torch.randn(n * p, c, generator=torch.Generator().manual_seed(n + p)).to(cuda_device)
    bank = ops.prep_bank(z)
    directed = ops.nearest(bank, n * p, 0, bank, n * p, c, p)
    sym = ops.nearest_pool(bank, n * p, c, p)[0]
    assert torch.equal(sym == torch.finfo(torch.float32).max, directed == torch.finfo(torch.float32).max)
    torch.testing.assert_close(sym, directed, rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize('parts', [2, 3, 8])
def test_symmetric_parts_combine_exactly(cuda_device, parts):
    """Per-rank parts of the tile list, MIN-combined, equal the one-part table bit for bit,
    including the rank-blocked layout used by the reduce-scatter."""
    from musc_b200 import ops
    from musc_b200.pipeline import shard_range
    n, p, c = 13, 1369, 64
    z = torch.randn(n * p, c, generator=torch.Generator().manual_seed(parts)).to(cuda_device)
    bank = ops.prep_bank(z)
    whole = ops.nearest_pool(bank, n * p, c, p)[0]
    _, _, per = shard_range(n, parts, 0)
    rpb = per * p
    combined = None
    for k in range(parts):
        t = ops.nearest_pool(bank, n * p, c, p, k, parts, rpb)          # (parts, n, rpb)
        combined = t if combined is None else torch.minimum(combined, t)
    # un-block: row = blk * rpb + r
    blocks = combined.shape[0]                                          # ceil(rows / rpb)
    flat = combined.permute(1, 0, 2).reshape(n, blocks * rpb)[:, :n * p]
    assert torch.equal(flat, whole)


@pytest.mark.parametrize('n,p,c,parts,max_ctas', [(2, 196, 64, 1, 0), (13, 1369, 64, 1, 0),
                                                    (13, 1369, 64, 3, 0), (9, 1369, 1024, 2, 0),
                                                    (7, 1369, 256, 1, 5)])
def test_cta_pair_kernel_equals_single_cta(cuda_device, monkeypatch, n, p, c, parts, max_ctas):
    """The CTA-pair pool kernel (cta_group::2, 256 x 256 tiles over two SMs) and the single-CTA
    kernel (128 x 256 tiles) give the same MIN-combined table bit for bit: row counts that are
    not a multiple of 256, N = 2, per-rank parts in the blocked layout, an odd CTA cap."""
    from musc_b200 import ops
    from musc_b200.pipeline import shard_range
    z = torch.randn(n * p, c, generator=torch.Generator().manual_seed(n * 7 + parts)).to(cuda_device)
    bank = ops.prep_bank(z)
    rpb = shard_range(n, parts, 0)[2] * p
    tables = {}
    for pair in ('0', '1'):
        monkeypatch.setenv('MUSC_B200_NEAREST_PAIR', pair)
        combined = None
        for k in range(parts):
            t = ops.nearest_pool(bank, n * p, c, p, k, parts, rpb, max_ctas=max_ctas).clone()
            combined = t if combined is None else torch.minimum(combined, t)
        tables[pair] = combined
    assert torch.equal(tables['0'], tables['1'])
    assert _lib_device_error_clear()


def _lib_device_error_clear() -> bool:
    from musc_b200 import _lib
    return _lib.take_device_error() == _lib.OK


@pytest.mark.parametrize('b,side,c,dtype,normalize,radii', [
    (3, 7, 64, torch.float32, True, (1, 3, 5)), (2, 37, 1024, torch.float32, True, (1, 3, 5)),
    (2, 37, 1024, torch.float16, False, (3,)), (2, 16, 256, torch.bfloat16, True, (5, 1)),
    (2, 2, 32, torch.float32, True, (1, 3, 5)), (2, 9, 1028, torch.float16, True, (1, 3, 5))])
def test_lnamd_staged_stencil_equals_register_stencil(cuda_device, monkeypatch, b, side, c, dtype, normalize,
                                                      radii):
    """The bulk-copy staged LNAMD stencil and the register-pipelined one give identical
    outputs: every dtype, with and without the L2 normalisation, side 2 (fewer columns than
    the copy ring), and a channel count whose fp16 rows are not 16-byte multiples (which
    takes the register kernel either way)."""
    from musc_b200 import ops
    g = torch.Generator().manual_seed(side * 31 + c)
    tokens = (torch.randn(b, 1 + side * side, c, generator=g) * 2 + 0.5).to(dtype).to(cuda_device)
    res = {}
    for bulk in ('0', '1'):
        monkeypatch.setenv('MUSC_B200_LNAMD_BULK', bulk)
        res[bulk] = ops.lnamd(tokens, radii, l2_normalize=normalize)
    for a, bb in zip(res['0'], res['1']):
        assert torch.equal(a, bb)
    assert _lib_device_error_clear()


def test_trimmed_mean_ties_and_offsets(cuda_device):
    from musc_b200 import ops
    gen = torch.Generator().manual_seed(5)
    n, rows = 37, 5000
    vals = (torch.randint(0, 6, (n, rows), generator=gen).float() * 0.25 + 1.0) ** 2  # many exact ties
    vals[torch.randint(0, n, (rows,), generator=gen), torch.arange(rows)] = float(np.finfo(np.float32).max)
    for lo, hi in [(0, 10), (3, 11), (0, 36), (35, 36)]:
        got = ops.trimmed_mean(vals.to(cuda_device), lo, hi).cpu().numpy()
        d = np.sort(np.sqrt(vals.numpy().astype(np.float64)), axis=0)[lo:hi]
        want = d.mean(axis=0).astype(np.float32).astype(np.float64)
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=0)


def test_pool16_full_pipeline_matches_reference(cuda_device):
    """Config 1 end to end on the GPU: 4 layers x r{1,3,5}, maps and image maxima."""
    from musc_b200.pipeline import score_pool
    from musc_b200.synthetic import prototype_mixture
    g = golden('pool16')
    tokens = prototype_mixture(int(g['n']), n_layers=4, c=1024, side=37, seed=int(g['seed']))
    res = score_pool([t.to(cuda_device) for t in tokens])
    got = res.scores.cpu().numpy()
    np.testing.assert_allclose(got, g['scores'], rtol=RTOL, atol=0)
    np.testing.assert_allclose(res.maps.cpu().numpy(), g['maps'], rtol=RTOL, atol=0)
    mx = res.image_max.cpu().numpy()
    np.testing.assert_allclose(mx, g['image_max'], rtol=RTOL, atol=0)
    want_order = np.argsort(g['image_max'], kind='stable')
    gaps = np.diff(g['image_max'][want_order])
    # identical ordering wherever the reference's gap exceeds the tolerance
    got_order = np.argsort(mx, kind='stable')
    resolved = np.concatenate([[True], gaps > RTOL * g['image_max'][want_order][1:]])
    assert np.array_equal(got_order[resolved], want_order[resolved])


def test_score_maps_match_reference(cuda_device):
    from musc_b200 import ops
    g = golden('reduce_small')
    maps, mx, up = ops.score_maps(_cuda(g['scores'], cuda_device), 518, upsampled=True)
    np.testing.assert_allclose(maps.cpu().numpy(), g['maps'], rtol=0, atol=1e-14)
    np.testing.assert_allclose(mx.cpu().numpy(), g['image_max'], rtol=0, atol=1e-14)
    np.testing.assert_allclose(up.cpu().numpy()[:, [0, 7, 517], :], g['up_rows_0_7_517'], rtol=0, atol=1e-14)


def test_config2_bank_against_oracle_rows(cuda_device):
    """N = 100 (config 2 size): one bank's GPU scores for sampled query images vs the oracle."""
    from musc_b200 import ops
    from musc_b200.synthetic import prototype_mixture_layer
    n = 100
    tokens = prototype_mixture_layer(n, generator=torch.Generator().manual_seed(11))
    z = ops.lnamd(tokens.to(cuda_device), (3,), l2_normalize=True)[0]
    scores = ops.msm(z).cpu().numpy()
    zc = z.cpu().numpy()
    a, b = omsm.trimmed_ranks(n)
    for i in (0, 57, 99):
        want = omsm.interval_average(omsm.nearest_minima(zc, i), a, b)
        np.testing.assert_allclose(scores[i], want, rtol=RTOL, atol=0)


def test_msm_is_invariant_to_row_scale_split(cuda_device):
    """Unnormalised features: the per-row power-of-two scaling keeps fp32-class accuracy."""
    from musc_b200 import ops
    gen = torch.Generator().manual_seed(8)
    z = torch.randn(6, 64, 96, generator=gen) * torch.logspace(-3, 3, 6).view(6, 1, 1)
    got = ops.msm(z.to(cuda_device)).cpu().numpy()
    want = omsm.msm(z.numpy())
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=0)


def test_no_device_timeout_recorded(cuda_device):
    from musc_b200 import _lib
    assert _lib.take_device_error() == _lib.OK


def test_trimmed_mean_large_pool(cuda_device):
    """N = 1024 (config 4): the selection kernel's large-pool shared-memory tile."""
    from musc_b200 import ops
    gen = torch.Generator().manual_seed(9)
    n, rows = 1024, 3000
    vals = torch.rand(n, rows, generator=gen) + 0.5
    a, b = ops.trimmed_ranks(n)
    got = ops.trimmed_mean(vals.to(cuda_device), a, b).cpu().numpy()
    d = np.sort(np.sqrt(vals.numpy().astype(np.float64)), axis=0)[a:b]
    np.testing.assert_allclose(got, d.mean(axis=0).astype(np.float32).astype(np.float64), rtol=1e-6, atol=0)


def test_super_fast_pipeline_matches_oracle(cuda_device):
    """Config 3 shape: the super-fast profile through score_pool equals the oracle on the
    super-fast banks (r = 3, 37x37 -> 28x28, L2-normalised)."""
    from musc_b200.pipeline import score_pool
    from musc_b200.synthetic import prototype_mixture_layer
    n = 12
    tokens = prototype_mixture_layer(n, generator=torch.Generator().manual_seed(4))
    res = score_pool([tokens.to(cuda_device)], super_fast_side=28, image_size=64)
    z = olnamd.l2_normalize(olnamd.lnamd_super_fast(tokens.numpy(), 28))
    want = omsm.msm(z)
    np.testing.assert_allclose(res.scores[0, 0].cpu().numpy(), want, rtol=RTOL, atol=0)
    maps, mx = oreduce.image_scores(want[None, None], 64)
    np.testing.assert_allclose(res.image_max.cpu().numpy(), mx, rtol=RTOL, atol=0)


def test_c_abi_score_pool_matches_pipeline_and_reference(cuda_device):
    """musc_b200_score_pool (the one-call C ABI path for non-Python hosts) on config 1:
    identical to the Python pipeline and within 2e-5 of the reference."""
    import ctypes
    from musc_b200 import _lib, ops
    from musc_b200.pipeline import score_pool
    from musc_b200.synthetic import prototype_mixture
    g = golden('pool16')
    n = int(g['n'])
    tokens = [t.to(cuda_device) for t in prototype_mixture(n, n_layers=4, c=1024, side=37, seed=int(g['seed']))]
    lib = _lib.lib()
    nbytes = lib.musc_b200_score_pool_bytes(n, 1370, 1024, 3)
    ws = ops._aligned_empty(nbytes, cuda_device)
    scores = torch.empty(3, 4, n, 1369, dtype=torch.float64, device=cuda_device)
    maps = torch.empty(n, 1369, dtype=torch.float64, device=cuda_device)
    mx = torch.empty(n, dtype=torch.float64, device=cuda_device)
    tok_ptrs = (ctypes.c_void_p * 4)(*[t.data_ptr() for t in tokens])
    radii = (ctypes.c_int * 3)(1, 3, 5)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    st = lib.musc_b200_score_pool(tok_ptrs, _lib.F32, n, 1370, 1024, 4, 3, radii, 0.0, 0.3, 518,
                                  ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(maps.data_ptr()),
                                  ctypes.c_void_p(mx.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nbytes, stream)
    _lib.check(st, 'musc_b200_score_pool')
    res = score_pool(tokens)
    assert torch.equal(scores, res.scores)
    assert torch.equal(mx, res.image_max)
    np.testing.assert_allclose(maps.view(n, 37, 37).cpu().numpy(), g['maps'], rtol=RTOL, atol=0)
    np.testing.assert_allclose(mx.cpu().numpy(), g['image_max'], rtol=RTOL, atol=0)


def test_rscin_matches_reference(cuda_device):
    """RsCIN on the GPU (musc_b200_rscin) against the reference's own RsCIN: the MVTec and
    VisA k lists, N = 9 / 24 / 60, 64- and 768-dimensional class tokens; passthroughs."""
    from musc_b200 import backend, ops
    g = golden('rscin_small')
    for c in 'abc':
        tok, s = g[f'{c}_tokens'], g[f'{c}_scores']
        for name, ks in (('k123', [1, 2, 3]), ('k189', [1, 8, 9])):
            got = ops.rscin(torch.from_numpy(s).to(cuda_device), torch.from_numpy(tok).to(cuda_device), ks)
            np.testing.assert_allclose(got.cpu().numpy(), g[f'{c}_{name}'], rtol=2e-6, atol=0)
            host = backend.RsCIN(s, list(tok), k_list=ks, device=cuda_device)     # the musc.py call form
            assert host.dtype == np.float32
            np.testing.assert_allclose(host, g[f'{c}_{name}'], rtol=2e-6, atol=0)
        assert backend.RsCIN(s, list(tok), k_list=[0]) is s
        same = ops.rscin(torch.from_numpy(s).to(cuda_device), None, [1, 2, 3]).cpu().numpy()
        np.testing.assert_array_equal(same, g[f'{c}_none'])
    with pytest.raises(ValueError):
        ops.rscin(torch.zeros(5, dtype=torch.float64, device=cuda_device),
                  torch.zeros(5, 8, device=cuda_device), [6])              # k > N


def test_config4_pool_sampled_images_against_oracle(cuda_device):
    """Config 4 size: N = 1024 images of 1369 patches (C = 64 to keep the oracle short).
    LNAMD r = 3 on the GPU, then the MSM of the whole 1.4 M-row bank (symmetric tiles,
    blocked table, interval over the 306 smallest of 1023 minima); the first, a middle and
    the last query image against the oracle's minima and interval average."""
    from musc_b200 import ops
    from musc_b200.synthetic import prototype_mixture_layer
    n, c = 1024, 64
    tokens = prototype_mixture_layer(n, c=c, generator=torch.Generator().manual_seed(44))
    z = ops.lnamd(tokens.to(cuda_device), (3,), l2_normalize=True)[0]
    del tokens
    scores = ops.msm(z).cpu().numpy()
    zc = z.cpu().numpy()
    del z
    a, b = omsm.trimmed_ranks(n)
    assert (a, b) == (0, 306)
    for i in (0, 511, 1023):
        want = omsm.interval_average(omsm.nearest_minima(zc, i, chunk=64), a, b)
        np.testing.assert_allclose(scores[i], want, rtol=RTOL, atol=0)
    assert _lib_device_error_clear()


def test_config3_super_fast_pool100_against_oracle(cuda_device):
    """Config 3 size: N = 100, one layer, r = 3 then 37x37 -> 28x28 (784 patches), C = 1024,
    through score_pool's super-fast profile; sampled query images against the oracle's
    super-fast banks, minima and interval average, and the image maxima of those images."""
    from musc_b200.pipeline import score_pool
    from musc_b200.synthetic import prototype_mixture_layer
    n = 100
    tokens = prototype_mixture_layer(n, generator=torch.Generator().manual_seed(33))
    res = score_pool([tokens.to(cuda_device)], super_fast_side=28)
    got = res.scores[0, 0].cpu().numpy()
    mx = res.image_max.cpu().numpy()
    z = olnamd.l2_normalize(olnamd.lnamd_super_fast(tokens.numpy(), 28))
    a, b = omsm.trimmed_ranks(n)
    for i in (0, 57, 99):
        want = omsm.interval_average(omsm.nearest_minima(z, i), a, b)
        np.testing.assert_allclose(got[i], want, rtol=RTOL, atol=0)
        _, want_mx = oreduce.image_scores(want[None, None, None], 518)
        np.testing.assert_allclose(mx[i], want_mx[0], rtol=RTOL, atol=0)
    assert _lib_device_error_clear()


# --------------------------------------------------------------------------- screen + refinement
def _exact_tables(z: np.ndarray):
    """float64 squared distances per (row, image): min, argmin and second min (self image skipped)."""
    n, p, c = z.shape
    flat = z.reshape(n * p, c).astype(np.float64)
    d2 = ((flat[:, None, :] - flat[None, :, :]) ** 2).sum(-1).reshape(n * p, n, p)
    order = np.argsort(d2, axis=2, kind='stable')
    mins = np.take_along_axis(d2, order[:, :, :1], 2)[..., 0]
    second = np.take_along_axis(d2, order[:, :, 1:2], 2)[..., 0] if p > 1 else np.full_like(mins, np.inf)
    return mins, order[:, :, 0], second, d2


@pytest.mark.parametrize('n,p,c', [(5, 49, 64), (7, 300, 128), (4, 1369, 64)])
def test_screen_tables_bound_the_exact_minima(cuda_device, n, p, c):
    """nearest_kernel<SCREEN>: the key's patch attains a distance within the screen's error
    of the exact minimum, its value is that screened distance, and the second-smallest value
    is a screened second minimum (within the bound of the exact second smallest)."""
    from musc_b200 import ops
    z = torch.randn(n, p, c, generator=torch.Generator().manual_seed(n * 31 + p))
    z = z / z.norm(dim=-1, keepdim=True)
    bank = ops.prep_bank(z.reshape(n * p, c).to(cuda_device))
    k1, m2, _ = ops.screen_pool(bank, n * p, c, p)
    k1 = k1[0].cpu().numpy().view(np.uint64).T            # (rows, n)
    m2 = m2[0].cpu().numpy().view(np.uint32).T
    mins, _, second, d2 = _exact_tables(z.numpy())
    tol = 2.5e-3                                          # the screen's certified bound is ~1.1e-3 here
    for row in range(n * p):
        for j in range(n):
            if j == row // p:
                assert k1[row, j] == np.uint64(0xFFFFFFFFFFFFFFFF)
                continue
            patch = int(k1[row, j] & np.uint64(0xFFFFFFFF))
            val = np.uint32(k1[row, j] >> np.uint64(32)).view(np.float32)
            assert 0 <= patch < p
            assert d2[row, j, patch] <= mins[row, j] + tol
            assert abs(float(val) - d2[row, j, patch]) <= tol
            assert float(np.uint32(m2[row, j]).view(np.float32)) >= second[row, j] - tol


@pytest.mark.parametrize('n,p,c,dup', [(6, 49, 64, False), (9, 100, 32, True), (5, 300, 1024, False),
                                       (11, 1369, 64, False), (8, 196, 64, True)])
def test_refine_equals_exact_path(cuda_device, n, p, c, dup):
    """screen + refinement vs the 3-pass exact table: every entry the refinement keeps is the
    exact minimum, entries it drops lie above the rank threshold, and the interval averages
    agree; with duplicated patches (exact ties, zero distances) most pairs go through the
    gathered 3-pass fallback."""
    from musc_b200 import ops
    g = torch.Generator().manual_seed(n * 7 + c)
    z = torch.randn(n, p, c, generator=g)
    if dup:
        z[:, 1::2] = z[:, 0::2][:, :z[:, 1::2].shape[1]]          # every other patch repeated
        z[1] = z[0]                                              # and a duplicated image
    z = z / z.norm(dim=-1, keepdim=True)
    rows = n * p
    bank = ops.prep_bank(z.reshape(rows, c).to(cuda_device))
    exact = ops.nearest_pool(bank, rows, c, p)[0]
    for lo, hi in [(0, max(1, int((n - 1) * 0.3))), (1, n - 1)]:
        if hi <= lo:
            continue
        k1, m2, _ = ops.screen_pool(bank, rows, c, p)
        ref = ops.refine(bank, rows, c, p, 0, rows, hi, k1, m2)
        kept = ref != torch.finfo(torch.float32).max
        torch.testing.assert_close(ref[kept], exact[kept], rtol=2e-5, atol=2e-6)
        s_ref = ops.trimmed_mean(ref, lo, hi)
        s_exact = ops.trimmed_mean(exact, lo, hi)
        # zero distances: the 3-pass identity leaves sqrt(fp32 rounding noise), the exact fp32
        # difference gives 0 (the duplicate-patch convention of the golden cases: 2e-3 absolute)
        torch.testing.assert_close(s_ref, s_exact, rtol=2e-6, atol=2e-3 if dup else 2e-6)
    assert _lib_device_error_clear()


@pytest.mark.parametrize('parts', [2, 3])
def test_refine_combines_partial_screens_exactly(cuda_device, parts):
    """Per-rank screen parts, handed to the refinement as partial tables of the rows each
    rank owns, give the single-part refinement bit for bit (the all-to-all path)."""
    from musc_b200 import ops
    from musc_b200.pipeline import shard_range
    n, p, c = 10, 1369, 64
    z = torch.randn(n * p, c, generator=torch.Generator().manual_seed(parts + 40)).to(cuda_device)
    bank = ops.prep_bank(z)
    rows = n * p
    _, _, per = shard_range(n, parts, 0)
    rpb = per * p
    k1w, m2w, _ = ops.screen_pool(bank, rows, c, p)
    b = int((n - 1) * 0.3)
    whole = ops.refine(bank, rows, c, p, 0, rows, b, k1w, m2w)
    tabs = [ops.screen_pool(bank, rows, c, p, k, parts, rpb, out=ops.screen_table(rows, p, rpb, cuda_device,
                                                                                 min_blocks=parts))
            for k in range(parts)]
    for r in range(parts):
        first, end, _ = shard_range(n, parts, r)
        q_rows = (end - first) * p
        if q_rows == 0:
            continue
        k1 = torch.stack([t[0][r] for t in tabs]).contiguous()
        m2 = torch.stack([t[1][r] for t in tabs]).contiguous()
        got = ops.refine(bank, rows, c, p, first * p, q_rows, b, k1, m2)
        assert torch.equal(got, whole[:, first * p:first * p + q_rows])


def test_refine_fallback_rounds_with_a_small_workspace(cuda_device):
    """A pool of repeated patches (every pair a near tie, nothing certifiable) with the
    interval reaching every image queues every pair for the exact fallback.  With the
    smallest workspace (a 128-row staging bank) the fallback runs in many rounds and must
    give the default workspace's table bit for bit; the scores match the oracle."""
    from musc_b200 import _lib, ops
    n, p, c = 12, 49, 64
    base = torch.randn(7, c, generator=torch.Generator().manual_seed(12))
    z = base[torch.arange(n * p) % 7].reshape(n, p, c)
    z = z + 1e-4 * torch.randn(n, p, c, generator=torch.Generator().manual_seed(13))
    z = (z / z.norm(dim=-1, keepdim=True)).contiguous()
    rows = n * p
    bank = ops.prep_bank(z.reshape(rows, c).to(cuda_device))
    k1, m2, _ = ops.screen_pool(bank, rows, c, p)
    lib = _lib.lib()
    small = lib.musc_b200_refine_min_bytes(n, rows, c)
    assert small < lib.musc_b200_refine_bytes(n, rows, c)
    assert ops.refine_launches(n, rows, c, small) > ops.refine_launches(n, rows, c)
    whole = ops.refine(bank, rows, c, p, 0, rows, n - 1, k1, m2)
    rounds = ops.refine(bank, rows, c, p, 0, rows, n - 1, k1, m2, workspace_bytes=small)
    assert torch.equal(whole, rounds)
    got = ops.trimmed_mean(rounds, 0, n - 1).view(n, p).cpu().numpy()
    want = omsm.msm(z.numpy(), 0, n - 1)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=2e-3)   # near-zero distances: see above
    with pytest.raises(ValueError):
        ops.refine(bank, rows, c, p, 0, rows, n - 1, k1, m2, workspace_bytes=small - 1024)
    assert _lib_device_error_clear()


def test_msm_screen_path_equals_exact_path_config2_bank(cuda_device, monkeypatch):
    """One config-2 bank (N = 100, C = 1024, LNAMD r = 3): the default screen + refinement
    and the 3-pass exact kernel give the same scores within fp32 rounding."""
    from musc_b200 import ops
    from musc_b200.synthetic import prototype_mixture_layer
    tokens = prototype_mixture_layer(100, generator=torch.Generator().manual_seed(5))
    z = ops.lnamd(tokens.to(cuda_device), (3,), l2_normalize=True)[0]
    deferred = ops.msm(z)
    monkeypatch.setenv('MUSC_B200_MSM_EXACT', '1')
    exact = ops.msm(z)
    torch.testing.assert_close(deferred, exact, rtol=2e-6, atol=0)
    assert _lib_device_error_clear()


@pytest.mark.parametrize('rows,c', [(0, 64), (1, 8), (1000, 1024), (37 * 296 + 5, 2048)])
def test_center_stats_in_a_fixed_order(cuda_device, rows, c):
    """The centring statistics: column sums (fp32 partials added in fp64) and the smallest
    squared row norm, the same bits on every call; zeros and +inf for an empty block."""
    from musc_b200 import ops
    z = torch.randn(rows, c, generator=torch.Generator().manual_seed(rows + c)).to(cuda_device)
    s1 = ops.center_stats(z)
    s2 = ops.center_stats(z)
    assert torch.equal(s1, s2)
    torch.testing.assert_close(s1[:c], z.double().sum(0), rtol=1e-6, atol=1e-6 * max(rows, 1) ** 0.5)
    if rows:
        want = (z.double() ** 2).sum(1).min()
        assert want * (1 - 2e-6) <= s1[c] <= want
    else:
        assert torch.isinf(s1[c])
    assert _lib_device_error_clear()


@pytest.mark.parametrize('n,p,c,shift', [(12, 196, 256, 0.0), (6, 784, 512, 0.0), (9, 196, 256, 3.0)])
def test_centred_msm_on_clustered_features(cuda_device, n, p, c, shift):
    """Features in a narrow cone, |z - mu| ~ 0.1 as for ViT tokens (without centring the
    screen's bound, ~1e-3 for unit rows, exceeds most nearest-neighbour gaps there): the
    screened + refined MSM equals MSM over float64 distances.  A pool shifted by a constant
    vector (|z| ~ 3.2) scores the same: the centring removes the shift, where fp32
    |a|^2 + |b|^2 - 2 a.b over the shifted rows would lose ~1e-3 to cancellation."""
    from musc_b200 import ops
    g = torch.Generator().manual_seed(n * 13 + c)
    d = torch.randn(c, generator=g)
    z = d / d.norm() + (0.1 / c ** 0.5) * torch.randn(n, p, c, generator=g)
    z = z / z.norm(dim=-1, keepdim=True)
    if shift:
        z = z + shift * torch.ones(c) / c ** 0.5
    got = ops.msm(z.to(cuda_device)).cpu().numpy()
    np.testing.assert_allclose(got, _msm_float64(z.numpy()), rtol=RTOL, atol=0)
    assert _lib_device_error_clear()


def _msm_float64(z: np.ndarray, topmin_max: float = 0.3) -> np.ndarray:
    """MSM with float64 distances of the fp32 rows (the reference's fp32 |q|^2 + |p|^2 - 2 q.p
    loses ~1e-7 (|q|^2 + |p|^2) to cancellation, more than the tolerance for rows of norm 3)."""
    n, p, c = z.shape
    flat = z.reshape(n * p, c).astype(np.float64)
    a, b = omsm.trimmed_ranks(n, 0, topmin_max)
    out = []
    for i in range(n):
        q = flat[i * p:(i + 1) * p]
        d2 = (q * q).sum(1)[:, None] + (flat * flat).sum(1)[None, :] - 2.0 * (q @ flat.T)
        minima = np.sqrt(np.maximum(d2.reshape(p, n, p).min(axis=2), 0.0))[:, [j for j in range(n) if j != i]]
        out.append(omsm.interval_average(minima, a, b))
    return np.stack(out)


def test_centred_banks_share_one_mean(cuda_device):
    """A pool split into row blocks (the ranks of a multi-GPU pool), each block prepared
    with the gathered statistics of all blocks, is bit for bit the bank of the whole pool
    prepared with the same statistics (and differs from the uncentred bank); and the screen + refinement of a centred bank equals the 3-pass
    exact table of the uncentred one within fp32 rounding (distances do not move)."""
    from musc_b200 import ops
    n, p, c = 8, 196, 128
    g = torch.Generator().manual_seed(77)
    d = torch.randn(c, generator=g)
    z = (d / d.norm() + (0.1 / c ** 0.5) * torch.randn(n * p, c, generator=g)).to(cuda_device)
    z = z / z.norm(dim=-1, keepdim=True)
    rows = n * p
    blocks = [z[:3 * p], z[3 * p:6 * p], z[6 * p:]]
    stats = torch.stack([ops.center_stats(b) for b in blocks])
    whole = ops.prep_bank(z, stats=stats, count=rows)
    parts = [ops.prep_bank(b, stats=stats, count=rows) for b in blocks]
    wp = ops.bank_planes(whole, rows, c)
    pp = [ops.bank_planes(bk, blk.shape[0], c) for bk, blk in zip(parts, blocks)]
    for i in range(5):
        assert torch.equal(wp[i], torch.cat([q[i] for q in pp]))
    assert not torch.equal(wp[0], ops.bank_planes(ops.prep_bank(z), rows, c)[0])
    k1, m2, _ = ops.screen_pool(whole, rows, c, p)
    b = int((n - 1) * 0.3)
    ref = ops.refine(whole, rows, c, p, 0, rows, b, k1, m2).cpu().numpy()
    flat = z.cpu().numpy().astype(np.float64)
    d2 = (flat * flat).sum(1)[:, None] + (flat * flat).sum(1)[None, :] - 2.0 * (flat @ flat.T)
    want = d2.reshape(rows, n, p).min(axis=2).T                          # (n, rows) float64 squared minima
    kept = ref != np.finfo(np.float32).max
    assert kept.sum() >= rows * b
    np.testing.assert_allclose(ref[kept], want[kept], rtol=2e-5, atol=1e-7)
    assert _lib_device_error_clear()


@pytest.mark.parametrize('n', [600, 1500])
def test_refine_large_pools_share_rows_between_warps(cuda_device, n):
    """Pools where fewer than 32 rows of screen tables fit a refinement CTA: at 600 images
    16 rows with one warp each in 512-thread CTAs, at 1500 images 4 rows shared by groups of
    six warps (the upper bounds of a row filled by the group together).  The refined table
    equals the 3-pass exact table wherever it keeps an entry, and the interval averages agree."""
    from musc_b200 import ops
    p, c = 16, 32
    z = torch.randn(n, p, c, generator=torch.Generator().manual_seed(n))
    z = z / z.norm(dim=-1, keepdim=True)
    rows = n * p
    bank = ops.prep_bank(z.reshape(rows, c).to(cuda_device))
    exact = ops.nearest_pool(bank, rows, c, p)[0]
    b = int((n - 1) * 0.3)
    k1, m2, _ = ops.screen_pool(bank, rows, c, p)
    ref = ops.refine(bank, rows, c, p, 0, rows, b, k1, m2)
    kept = ref != torch.finfo(torch.float32).max
    assert int(kept.sum()) >= rows * b
    torch.testing.assert_close(ref[kept], exact[kept], rtol=2e-5, atol=2e-6)
    torch.testing.assert_close(ops.trimmed_mean(ref, 0, b), ops.trimmed_mean(exact, 0, b), rtol=2e-6, atol=2e-6)
    assert _lib_device_error_clear()
