#!/usr/bin/env python
"""Benchmark of the MuSc scoring hot path on B200: pool images scored per second.

Workload: a pool of N = 100 images, 4 hooked layers x
radii {1, 3, 5}, 1369 patches x 1024 channels fp32 tokens from the seeded
prototype-mixture generator (MVTec is not available; the generator stands in
for it).  One step = the whole scoring path for one pool: LNAMD of 4 layers
(3 radii each), 12 MSM banks (bank prep, fused distance/min GEMM, interval
average) and the score reduction (maps, up-sampled image maxima).

* ``value``  -- N / step time with the tokens already resident in HBM
  (2.24 GB of inputs per step, far above the 126 MB L2, so no flush is needed).
* ``e2e``    -- the same through the public API with host buffers: pinned
  host tokens copied in and maps / image maxima copied out every step (steps
  pipelined: step k+1's inputs are copied while step k computes).
* ``roofline`` -- the dominant kernel (nearest_kernel) timed live with CUDA
  events on its stream: algorithmic flops 2*C*P^2*N*(N-1) per launch.
* ``cpu_baseline`` -- the reference's ``original`` path (restated with the same torch
  CPU operations, ``oracle.torch_cpu``) on the host cores, on a bounded sample, scaled
  to images/s.

``--gpus N`` under torchrun: rank r scores query images [r*ceil(N/G), ...)
against the whole pool: banks are all-gathered over NCCL, each rank evaluates a
balanced share of the symmetric distance tiles and a MIN reduce-scatter hands
each rank its query rows' minima; the time is the max over ranks and ``value``
counts the whole pool (strong scaling).
``--impl reference`` times that CPU port of the reference path instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / 'musc-gpu_b200'))

N_POOL = 100
N_LAYERS = 4
RADII = (1, 3, 5)
SIDE = 37
C = 1024
P = SIDE * SIDE
METRIC = 'pool images scored/sec (1369x1024 patches, 4 layers x 3 radii)'
UNIT = 'images/s'


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=5)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--pool', type=int, default=None, help='pool size (default: the config\'s)')
    ap.add_argument('--config', default='2', choices=['1', '2', '3', '4', '5', 'images'],
                    help='BASELINE.json config: 1 (N=16, the reference arm runs it in full), 2 (default, '
                         'the metric\'s), 3 super-fast, 4 N=1024, 5 encoder end to end; "images" = the '
                         'pool-image preprocessing ahead of the encoder (its own metric)')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--collective-sms', type=int, default=0,
                    help='SMs left free for NCCL during each bank GEMM (multi-GPU; 0 = none)')
    ap.add_argument('--exchange', default='copy', choices=['copy', 'nccl'],
                    help='multi-GPU transport of banks and screen tables: peer copies on copy engines '
                         '(default) or NCCL collectives')
    return ap.parse_args()


def _peaks():
    try:
        return json.loads((REPO / 'MEASURED_PEAKS.json').read_text()), 'measured'
    except Exception:
        return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0, 'bf16_tflops_sustained': 1400.0}, 'fallback'


def _traffic(exact_path: bool):
    """DRAM bytes per launch of the dominant GEMM at config 2, from the committed ncu summary
    (or None when no capture of that kernel variant is committed)."""
    f = REPO / 'profiles' / 'nearest_kernel_traffic.json'
    try:
        d = json.loads(f.read_text())
        return d.get('bytes_per_launch_config2' if exact_path else 'screen_bytes_per_launch_config2')
    except Exception:
        return None


# ----------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--id={self.gpu}', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                 '-lms', '200'], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.file is None:
            return None
        try:
            lines = [l.strip() for l in Path(self.file.name).read_text().splitlines() if l.strip()]
            os.unlink(self.file.name)
        except Exception:
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for l in lines:
            f = [x.strip() for x in l.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == 'active':
                    reasons.add(name)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


# ----------------------------------------------------------------- CPU baseline
class CpuSample:
    """Time the reference's original CPU path on the host cores.

    The timed code is ``oracle.torch_cpu``: the reference's ``LNAMD._embed``,
    ``SuperFastAggregation`` and ``compute_scores_fast`` restated with the same torch CPU
    operations (pinned bit for bit to the reference's golden outputs), with every host
    thread.  ``full`` runs the whole pool (LNAMD of every layer and radius, MSM of every
    bank) -- config 1 (N = 16), about a minute.  Otherwise one call is a bounded sample:
    LNAMD of 2 images of one layer (all radii) and the MSM rows of one query image against
    the whole pool for one bank, extrapolated to a pool image (layers x LNAMD + banks x MSM
    rows).  Setup (the pool's tokens and one bank) is untimed.
    """

    def __init__(self, cfg: dict, pool: int, full: bool, seed: int = 1):
        import torch
        from musc_b200.synthetic import prototype_mixture, prototype_mixture_layer
        from oracle import torch_cpu
        torch.set_num_threads(os.cpu_count() or 1)
        self.torch_cpu = torch_cpu
        self.cfg, self.pool, self.full = cfg, pool, full
        self.layers, self.radii, self.sf = cfg['layers'], cfg['radii'], cfg['super_fast']
        if full:
            self.tokens = prototype_mixture(pool, n_layers=self.layers, seed=seed)
        else:
            self.tokens = [prototype_mixture_layer(pool, generator=torch.Generator().manual_seed(seed))]
            self.z = self._bank(self.tokens[0], self.radii[-1])
        self.k_min, self.k_max = torch_cpu.interval(pool)

    def _bank(self, tokens, r):
        if self.sf:
            return self.torch_cpu.lnamd_super_fast(tokens, self.sf)
        return self.torch_cpu.lnamd_bank(tokens, r)

    def run(self) -> tuple[float, float]:
        """One step: ``(wall seconds, seconds per pool image)``."""
        t_start = time.perf_counter()
        if self.full:
            for layer in self.tokens:
                for r in self.radii:
                    self.torch_cpu.msm(self._bank(layer, r), 0.0, 0.3)
            wall = time.perf_counter() - t_start
            return wall, wall / self.pool
        for r in self.radii:
            self._bank(self.tokens[0][:2], r)
        t_lnamd = (time.perf_counter() - t_start) / 2          # per image, all radii, one layer
        t0 = time.perf_counter()
        self.torch_cpu.msm_rows(self.z, 0, self.k_min, self.k_max)
        t_msm = time.perf_counter() - t0                       # one query image, one bank
        wall = time.perf_counter() - t_start
        return wall, self.layers * t_lnamd + self.layers * len(self.radii) * t_msm

    def describe(self) -> str:
        what = ('LNAMD._embed + compute_scores_fast' if not self.sf else
                'SuperFastAggregation (r=3 LNAMD + adaptive_avg_pool2d) + compute_scores_fast')
        head = f'the reference original path ({what}) restated with the same torch CPU operations'
        if self.full:
            return f'{head}: the whole pool (N={self.pool}, {self.layers} layers x {len(self.radii)} radii) per step'
        tail = (f'; one step = LNAMD of 2 images x 1 layer (all radii) + MSM rows of 1 query image x 1 bank vs '
                f'the whole pool (N={self.pool}), extrapolated to {self.layers} layers x '
                f'{self.layers * len(self.radii)} banks per pool image')
        if self.cfg.get('encoder'):
            tail += '; the ViT encoder\'s CPU time is not included (favours the reference)'
        return head + tail


def cpu_measure(cfg: dict, pool: int, full: bool, steps: int, warmup: int) -> dict:
    """Run ``warmup`` + ``steps`` CPU steps; the numbers of the timed ones."""
    sample = CpuSample(cfg, pool, full)
    for _ in range(max(warmup, 0)):
        sample.run()
    runs = [sample.run() for _ in range(max(steps, 1))]
    walls, per_image = zip(*runs)
    return {'value': 1.0 / statistics.median(per_image), 'ms_per_step': statistics.median(walls) * 1e3,
            'wall_s': sum(walls), 'cores': os.cpu_count() or 1, 'sample': sample.describe(),
            'extrapolated': not full}


def run_reference(args):
    """``--impl reference``: the reference's CPU path (torch-CPU port, ``oracle.torch_cpu``), rank 0 only.

    Every reported step ran: ``ms_per_step`` is the median wall time of one step (the whole
    pool for config 1, one bounded sample otherwise, marked ``extrapolated``), so
    ``steps * ms_per_step`` is the timed region's length.
    """
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    sys.path.insert(0, str(REPO))
    cfg = CONFIGS[args.config]
    pool = args.pool if args.pool is not None else cfg['pool']
    m = cpu_measure(cfg, pool, args.config == '1', args.steps, args.warmup)
    line = {
        'metric': METRIC, 'value': m['value'], 'unit': UNIT, 'n_gpus': args.gpus, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': m['ms_per_step'], 'higher_is_better': True,
        'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'impl': 'reference', 'extrapolated': m['extrapolated'],
        'config': config_of(args, cfg, pool, 1 if args.gpus < 1 else args.gpus),
        'cpu_baseline': {'value': m['value'], 'unit': UNIT, 'cores': m['cores'], 'kind': 'port',
                         'sample': m['sample'], 'extrapolated': m['extrapolated']},
        'e2e': {'value': m['value'], 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def symmetric_tiles(rows: int, patches: int, n_images: int, bm: int = 128, bn: int = 256) -> int:
    """Tiles the symmetric nearest kernel evaluates (tiles holding an img(r) < img(c) element)."""
    num_m, num_n = -(-rows // bm), -(-rows // bn)
    total = 0
    for m in range(num_m):
        img = m * bm // patches
        if img >= n_images - 1:
            continue
        need = (img + 1) * patches - bn + 1
        total += num_n - (0 if need <= 0 else -(-need // bn))
    return total


# ----------------------------------------------------------------- GPU arm
CONFIGS = {
    '1': dict(pool=16, layers=4, radii=(1, 3, 5), super_fast=None, encoder=False,
              desc='config1: pool N={pool}, 4 layers x r{{1,3,5}}, P=1369, C=1024 fp32 prototype-mixture '
                   'tokens resident in HBM'),
    '2': dict(pool=100, layers=4, radii=(1, 3, 5), super_fast=None, encoder=False,
              desc='config2: pool N={pool}, 4 layers x r{{1,3,5}}, P=1369, C=1024 fp32 prototype-mixture '
                   'tokens resident in HBM'),
    '3': dict(pool=100, layers=1, radii=(3,), super_fast=28, encoder=False,
              desc='config3 super-fast: pool N={pool}, 1 layer, r=3 then 37x37->28x28 (784 patches), '
                   'C=1024 fp32 prototype-mixture tokens'),
    '4': dict(pool=1024, layers=4, radii=(1, 3, 5), super_fast=None, encoder=False,
              desc='config4: pool N={pool}, 4 layers x r{{1,3,5}}, P=1369, C=1024 fp32 prototype-mixture tokens'),
    '5': dict(pool=200, layers=4, radii=(1, 3, 5), super_fast=None, encoder=True,
              desc='config5 end to end: random-init ViT-L/14 (24 blocks, d=1024, 16x64 heads, fp16 GEMMs + '
                   'fused attention) on N={pool} seeded 518x518x3 U[0,1] images, batch 4, hooks 6/12/18/24, '
                   'then LNAMD r{{1,3,5}} + MSM + reduction'),
}


def config_of(args, cfg: dict, pool: int, world: int) -> dict:
    """The line's ``config``: the same dict for both arms of one command."""
    p_score = cfg['super_fast'] ** 2 if cfg['super_fast'] else P
    tok_bytes = cfg['layers'] * pool * (P + 1) * C * 4
    return {'workload': cfg['desc'].format(pool=pool), 'global_batch': pool, 'seq_len': p_score,
            'parallelism': f'query-shard{world}',
            'l2': (f'inputs larger than L2 ({tok_bytes / 1e9:.2f} GB of tokens per step); no flush'
                   if not cfg['encoder'] else 'encoder activations and banks larger than L2; no flush')}


def run_b200(args):
    import torch
    import torch.distributed as dist
    from musc_b200 import ops, pipeline
    from musc_b200.synthetic import prototype_mixture_images, random_images

    cfg = CONFIGS[args.config]
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    if world != args.gpus:
        raise SystemExit(f'--gpus {args.gpus} but WORLD_SIZE={world}')
    torch.cuda.set_device(local_rank)
    dev = torch.device('cuda', local_rank)
    group = None
    if world > 1:
        import datetime
        if args.collective_sms > 0:
            # The bank GEMM leaves `collective_sms` SMs free; NCCL's channels (one CTA
            # each) must all fit there to run beside it.
            os.environ.setdefault('NCCL_MAX_CTAS', str(args.collective_sms))
            os.environ.setdefault('NCCL_MAX_NCHANNELS', str(args.collective_sms))
        dist.init_process_group('nccl', device_id=dev, timeout=datetime.timedelta(seconds=300))
        group = dist.group.WORLD

    pool = args.pool if args.pool is not None else cfg['pool']
    radii, n_layers, sf = cfg['radii'], cfg['layers'], cfg['super_fast']
    p_score = sf * sf if sf else P
    first, end, _ = pipeline.shard_range(pool, world, rank)
    n_local = end - first

    # ---- inputs: pinned host copies + resident device copies of this rank's images
    encoder = None
    if cfg['encoder']:
        from musc_b200.encoder import VisionEncoder, random_vit_state
        encoder = VisionEncoder(random_vit_state(0), device=dev)
        host = [random_images(end, 518, seed=0)[first:end].contiguous().pin_memory()]
    else:
        # this rank's images only, generated on its GPU (per-image seeds: shard-independent)
        host = [t.cpu().pin_memory()
                for t in prototype_mixture_images(range(first, end), n_layers, C, SIDE, seed=0, device=dev)]
    resident = [h.to(dev, non_blocking=True) for h in host]
    torch.cuda.synchronize()
    h2d = sum(h.numel() * h.element_size() for h in host)

    # ---- our kernels, instrumented: launch counts and the dominant kernel's event timing
    near_events, launches = [], [0]
    # our kernels per call: lnamd = statistics + stencil; nearest_pool = fill + GEMM; screen_pool = GEMM
    # (its fills are memsets); refine = image bounds + refinement + 3 per fallback round (plan, gather,
    # gathered GEMM), counted by the library
    per_call = {'lnamd': 2, 'lnamd_super_fast': 2, 'center_stats': 2, 'prep_bank': 1, 'nearest_pool': 2,
                'screen_pool': 1,
                'refine': 6, 'trimmed_mean': 1, 'score_maps': 1}
    gemm_ops = ('nearest_pool', 'screen_pool')

    class Kernels:
        trimmed_ranks = staticmethod(ops.trimmed_ranks)
        nearest_pool_table = staticmethod(ops.nearest_pool_table)
        screen_table = staticmethod(ops.screen_table)
        empty_bank = staticmethod(ops.empty_bank)
        bank_planes = staticmethod(ops.bank_planes)
    kern = Kernels()

    op_events = {}

    def counted(name):
        fn = getattr(ops, name)

        def call(*a, **k):
            if name == 'refine':   # 2 kernels + 3 per fallback round (args: bank, rows, c, p, first, q_rows, ...)
                launches[0] += ops.refine_launches(a[1] // a[3], a[5], a[2])
            else:
                launches[0] += per_call[name]
            st = torch.cuda.current_stream(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            out = fn(*a, **k)
            e1.record(st)
            (near_events if name in gemm_ops else op_events.setdefault(name, [])).append((e0, e1))
            return out
        return call
    for name in per_call:
        setattr(kern, name, counted(name))
    orig_attention = ops.attention
    attn_events = []

    def counted_attention(*a, **k):
        launches[0] += 1
        st = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        out = orig_attention(*a, **k)
        e1.record(st)
        attn_events.append((e0, e1, a[0].shape[0], a[0].shape[1], a[3]))
        return out
    ops.attention = counted_attention

    def tokens_of(inputs, graph=True):
        if encoder is None:
            return inputs
        images = inputs[0]
        layers = [[] for _ in range(4)]
        for i in range(0, images.shape[0], 4):           # the reference's batch size
            if graph:
                launches[0] += encoder.layers            # attention launches replayed by the graph
            _, toks = encoder.forward(images[i:i + 4], [6, 12, 18, 24], graph=graph)
            for li, t in enumerate(toks):
                layers[li].append(t)
        return [torch.cat(t) if t else torch.empty(0, 1 + P, C, device=dev) for t in layers]

    exchange = None
    if group is not None and args.exchange == 'copy':
        from musc_b200.exchange import PeerExchange
        exchange = PeerExchange(group, dev, pool, p_score, C)

    def step(inputs, ready=None):
        # NVTX range "pool_step": lets a profiler capture the launches of the pool steps only
        # (ncu --nvtx --nvtx-include "pool_step/"), not the synthetic-input generation
        torch.cuda.nvtx.range_push('pool_step')
        try:
            return pipeline.score_pool(tokens_of(inputs), n_images=pool, radii=radii, group=group, kernels=kern,
                                       super_fast_side=sf, ready=None if encoder is not None else ready,
                                       collective_sms=args.collective_sms, exchange=exchange)
        finally:
            torch.cuda.nvtx.range_pop()

    def barrier():
        if group is not None:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step(resident)
    torch.cuda.synchronize()
    near_events.clear()
    attn_events.clear()
    op_events.clear()
    launches[0] = 0
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        t0.record(stream)
        for _ in range(args.steps):
            step(resident)
        t1.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed_ms = t0.elapsed_time(t1)
    near_ms = [a.elapsed_time(b) for a, b in near_events]
    op_ms = {name: sum(a.elapsed_time(b) for a, b in evs) / args.steps for name, evs in op_events.items()}
    from musc_b200.pipeline import exact_pool_path
    exact_path = exact_pool_path()
    op_ms['nearest_pool' if exact_path else 'screen_pool'] = sum(near_ms) / args.steps
    refine_ms = [a.elapsed_time(b) for a, b in op_events.get('refine', [])]
    launches_timed = launches[0]
    # attention: timed on one eager encoder pass (the timed steps replay CUDA graphs);
    # 4 * L^2 * d flop per (batch item, head), head_dim 64
    attn_ms = attn_flop = 0.0
    if encoder is not None:
        attn_events.clear()
        tokens_of(resident, graph=False)
        torch.cuda.synchronize()
        attn_ms = sum(e0.elapsed_time(e1) for e0, e1, *_ in attn_events)
        attn_flop = sum(4.0 * length * length * 64 * bsz * heads for _, _, bsz, length, heads in attn_events)

    # ---- e2e: every step copies its inputs from pinned host memory (per-layer copies on a
    # side stream; each layer's scoring waits only for its own copy) and reads its maps and
    # image maxima back into pinned host memory.  Steps are pipelined like a serving loop:
    # step k+1's inputs are copied into a second device buffer while step k computes.
    dev_bufs = [[torch.empty_like(t) for t in resident] for _ in range(2)]
    copy_stream = torch.cuda.Stream(dev)
    compute = torch.cuda.current_stream(dev)
    consumed = [None, None]

    def issue_copies(k):
        buf = dev_bufs[k % 2]
        if consumed[k % 2] is not None:
            copy_stream.wait_event(consumed[k % 2])   # the step that last used this buffer is done
        events = []
        with torch.cuda.stream(copy_stream):
            for h, d in zip(host, buf):
                d.copy_(h, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                events.append(ev)
        return events

    host_maps = host_mx = None

    def e2e_run(n_steps):
        nonlocal host_maps, host_mx
        pending = issue_copies(0)
        d2h_bytes = 0
        for k in range(n_steps):
            events = pending
            if k + 1 < n_steps:
                pending = issue_copies(k + 1)
            if encoder is not None:
                compute.wait_event(events[-1])
            res = step(dev_bufs[k % 2], ready=events)
            ev = torch.cuda.Event()
            ev.record(compute)
            consumed[k % 2] = ev
            maps, mx = pipeline.gather_pool(res, group)
            if rank == 0:
                if host_maps is None:
                    host_maps = torch.empty(maps.shape, dtype=maps.dtype).pin_memory()
                    host_mx = torch.empty(mx.shape, dtype=mx.dtype).pin_memory()
                host_maps.copy_(maps, non_blocking=True)
                host_mx.copy_(mx, non_blocking=True)
                d2h_bytes = host_maps.numel() * 8 + host_mx.numel() * 8
        return d2h_bytes

    e2e_run(1)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    d2h = e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    ops.attention = orig_attention
    # Every bounded device-side wait completed in the timed runs (else: RuntimeError, no line).
    ops.check_device_error(dev, 'bench')

    # ---- sharded parity (N > 1): every rank re-scores the last bank of one more pool step
    # as one whole-pool part from the gathered bank and compares its own query rows with
    # the sharded scores bit for bit (untimed).
    parity = None
    if group is not None:
        res = pipeline.score_pool(tokens_of(resident), n_images=pool, radii=radii, group=group, kernels=ops,
                                  super_fast_side=sf, verify=True, exchange=exchange)
        parity = res.verified
        torch.cuda.synchronize()
        ops.check_device_error(dev, 'bench parity')

    stats = torch.tensor([elapsed_ms, e2e_ms, sum(near_ms) / max(len(near_ms), 1),
                          sum(refine_ms) / max(len(refine_ms), 1)], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms, near_avg_ms, refine_avg_ms = stats.tolist()

    if rank == 0:
        peaks, peak_kind = _peaks()
        ms_per_step = elapsed_ms / args.steps
        value = pool / (ms_per_step / 1e3)
        # algorithmic (directed) MSM flops per bank, 2*C*P^2*N*(N-1) (the count the reference's
        # original path computes); each rank's launch covers 1/world of the pool's tiles
        msm_flop_per_bank = 2.0 * C * p_score * p_score * pool * (pool - 1)
        # the MSM contraction's time per bank: the GEMM plus (default path) the refinement to
        # exact minima; effective rate = the directed algorithmic flops over that time
        msm_ms = near_avg_ms + (0.0 if exact_path else refine_avg_ms)
        achieved_tflops = msm_flop_per_bank / world / (msm_ms / 1e3) / 1e12
        # executed tensor-core work of the GEMM alone: MMA passes (3 exact, 1 screened) over the
        # symmetric tiles (whole tiles holding a pair of different images, each pair once; 256 x 256
        # for the CTA-pair kernel, 128 x 256 for the single-CTA one), this rank's share
        tile_m = 256 if os.environ.get('MUSC_B200_NEAREST_PAIR', '1') != '0' else 128
        passes = 3 if exact_path else 1
        mma_tflops = (passes * 2.0 * symmetric_tiles(pool * p_score, p_score, pool, bm=tile_m) * tile_m * 256 * C
                      / world / (near_avg_ms / 1e3) / 1e12)
        peak = peaks.get('bf16_tflops_sustained', peaks.get('bf16_tflops'))
        line = {
            'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms_per_step, 'higher_is_better': True,
            'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'config': dict(config_of(args, cfg, pool, world),
                           **({'exchange': args.exchange} if world > 1 else {})),
            'e2e': {'value': pool / (e2e_ms / args.steps / 1e3), 'unit': UNIT,
                    'h2d_bytes_per_step': h2d * world, 'd2h_bytes_per_step': d2h},
            'roofline': {'kernel': ('nearest_kernel<symmetric>' if exact_path
                                    else 'nearest_kernel<screen> + refinement'),
                         'bound': 'tensor', 'achieved': achieved_tflops,
                         'peak': peak, 'unit': 'TFLOP/s', 'frac': achieved_tflops / peak,
                         'traffic': _traffic(exact_path) if (args.config == '2' and pool == N_POOL) else None,
                         'peak_kind': f'{peak_kind} bf16 sustained (kernel timed inside a long step)',
                         'mma_executed_tflops': mma_tflops, 'mma_frac': mma_tflops / peak,
                         'mma_kind': ('kind::f16 cta_group::%d (fp16 %s, symmetric %dx256 tiles)'
                                      % (2 if tile_m == 256 else 1,
                                         'split hi/lo, 3 passes' if exact_path else 'hi only, 1 screening pass',
                                         tile_m)),
                         'gemm_ms_per_bank': near_avg_ms, 'refine_ms_per_bank': refine_avg_ms,
                         'launch_ms': msm_ms},
            'gpu_launches': launches_timed,
            'clocks': clocks.summary(),
            'op_ms_per_step': {k: round(v, 3) for k, v in sorted(op_ms.items(), key=lambda kv: -kv[1])},
        }
        if args.config == '5':
            line['dtype'] = 'f32 scoring, fp16 encoder'
            if attn_ms > 0:
                at = attn_flop / (attn_ms / 1e3) / 1e12
                line['attention'] = {'kernel': 'attention_kernel', 'bound': 'tensor', 'achieved': at,
                                     'peak': peaks.get('bf16_tflops'), 'unit': 'TFLOP/s',
                                     'frac': at / peaks.get('bf16_tflops'), 'launches': len(attn_events),
                                     'ms_per_pool': attn_ms, 'timed_on': 'one eager encoder pass',
                                     'peak_kind': f'{peak_kind} bf16 burst (short launches)'}
        if parity is not None:
            line['parity'] = parity
        if not args.no_cpu_baseline and world == 1 and args.config != '1':
            # rank 0 at N = 1 only (no other rank is waiting meanwhile); the same sampler as
            # the reference arm, so the two CPU figures agree on the same host
            sys.path.insert(0, str(REPO))
            m = cpu_measure(cfg, pool, False, 3, 1)
            line['cpu_baseline'] = {'value': m['value'], 'unit': UNIT, 'cores': m['cores'], 'kind': 'port',
                                    'sample': m['sample'], 'extrapolated': m['extrapolated'],
                                    'timed_s': round(m['wall_s'], 2)}
        print(json.dumps(line), flush=True)
    if group is not None:
        if exchange is not None:
            exchange.close()
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


# ----------------------------------------------------------------- image preprocessing
IMG_METRIC = 'pool images preprocessed/sec (900x900 RGB -> 3x518x518 fp32, CLIP bicubic transform)'
IMG_H = IMG_W = 900
IMG_OUT = 518


def _img_pool(n: int, seed: int = 3):
    import numpy as np
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (n, IMG_H, IMG_W, 3), dtype=np.uint8)


def images_cpu_measure(n_sample: int, min_seconds: float = 5.0) -> dict:
    """The reference's per-image transform (PIL bicubic resize, ToTensor, Normalize; the
    torchvision classes of ``open_clip/transform.py:124-133``) on ``n_sample`` images, one
    image per host thread as the reference's threaded loader runs them."""
    from concurrent.futures import ThreadPoolExecutor
    import torch
    from PIL import Image
    sys.path.insert(0, str(REPO))
    from oracle import torch_cpu
    cores = os.cpu_count() or 1
    torch.set_num_threads(1)
    tf = torch_cpu.clip_image_transform(IMG_OUT)
    pil = [Image.fromarray(a) for a in _img_pool(min(n_sample, 8), seed=4)]
    done = 0
    with ThreadPoolExecutor(max_workers=cores) as ex:
        list(ex.map(tf, pil[:2]))
        t0 = time.perf_counter()
        while True:   # batches of n_sample images until at least min_seconds have passed
            list(ex.map(tf, [pil[i % len(pil)] for i in range(n_sample)]))
            done += n_sample
            wall = time.perf_counter() - t0
            if wall >= min_seconds:
                break
    return {'value': done / wall, 'cores': cores, 'wall_s': wall,
            'sample': f'{done} images of {IMG_H}x{IMG_W} through the torchvision/PIL transform '
                      f'({wall:.1f} s), {cores} threads, torch intra-op threads 1'}


def run_images_reference(args):
    if int(os.environ.get('RANK', '0')) != 0:
        return
    n_sample = 4 * (os.cpu_count() or 1)
    ms = []
    for i in range(args.warmup + args.steps):
        m = images_cpu_measure(n_sample, min_seconds=1.0)
        if i >= args.warmup:
            ms.append(m)
    value = statistics.median(x['value'] for x in ms)
    line = {'metric': IMG_METRIC, 'value': value, 'unit': UNIT, 'n_gpus': 1, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': statistics.median(x['wall_s'] for x in ms) * 1e3,
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8 -> f32',
            'data': 'synthetic', 'impl': 'reference',
            'config': {'workload': f'at least {n_sample} images and 1 s per step (sample), {IMG_H}x{IMG_W} -> {IMG_OUT}'},
            'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': ms[0]['cores'], 'kind': 'reference',
                             'sample': ms[0]['sample']},
            'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def _img_traffic(n: int):
    """DRAM bytes per launch of the resample kernel for ``n`` images, scaled from the committed
    ncu capture (or None)."""
    try:
        d = json.loads((REPO / 'profiles' / 'resample_kernel_traffic.json').read_text())
        return d['bytes_per_launch_pool200'] * n / 200
    except Exception:
        return None


def run_images(args):
    """``value``: the device transform over a resident batch of ``--pool`` (default 200, the
    config-5 pool) 900 x 900 images (486 MB in, 644 MB out: no L2 flush needed); ``e2e``: the
    loader's path from host arrays (pinned staging, H2D on the copy stream, the kernels), the
    (B, 3, 518, 518) result left on the device for the encoder (no D2H)."""
    import torch
    from musc_b200 import ops
    from musc_b200.loader import DeviceImageLoader
    if int(os.environ.get('WORLD_SIZE', '1')) != 1:
        raise SystemExit('--config images runs on one GPU')
    n = args.pool or 200
    dev = torch.device('cuda', 0)
    host = _img_pool(n)
    images = torch.from_numpy(host).to(dev)
    out = torch.empty((n, 3, IMG_OUT, IMG_OUT), dtype=torch.float32, device=dev)
    ws = torch.empty(ops.preprocess_workspace_bytes(IMG_H, IMG_W, IMG_OUT, IMG_OUT), dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        ops.preprocess_images(images, IMG_OUT, out=out, workspace=ws)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(0) as clocks:
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for k in range(args.steps):
            starts[k].record()
            ops.preprocess_images(images, IMG_OUT, out=out, workspace=ws)
            ends[k].record()
        t1.record()
        torch.cuda.synchronize()
    elapsed_ms = t0.elapsed_time(t1)
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    # parity of the timed output: a sampled image against the oracle restatement
    sys.path.insert(0, str(REPO))
    from oracle import image as oimage
    probe = [0, n // 2, n - 1]
    exact = all(oimage.preprocess(host[i], IMG_OUT).view('uint32').tolist()
                == out[i].cpu().numpy().view('uint32').tolist() for i in probe)
    # e2e through the loader from host arrays
    loader = DeviceImageLoader([], device=dev)
    arrays = [host[i] for i in range(n)]
    for k in range(args.warmup):
        loader.preprocess(arrays, slot=k % 2)
    torch.cuda.synchronize()
    e0 = time.perf_counter()
    for k in range(args.steps):
        loader.preprocess(arrays, slot=k % 2)
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - e0) / args.steps
    peaks, peak_kind = _peaks()
    algo_bytes = n * (IMG_H * IMG_W * 3 + 3 * IMG_OUT * IMG_OUT * 4)
    achieved = algo_bytes / (launch_ms / 1e3) / 1e9
    ms_per_step = elapsed_ms / args.steps
    line = {'metric': IMG_METRIC, 'value': n / (ms_per_step / 1e3), 'unit': UNIT, 'n_gpus': 1,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms_per_step, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8 -> f32 (int32 fixed-point resample)',
            'data': 'synthetic',
            'config': {'workload': f'{n} images {IMG_H}x{IMG_W}x3 u8 -> 3x{IMG_OUT}x{IMG_OUT} f32 per step',
                       'l2': 'inputs + outputs 1.13 GB > L2, no flush'},
            'e2e': {'value': n / e2e_s, 'unit': UNIT, 'h2d_bytes_per_step': int(host.nbytes),
                    'd2h_bytes_per_step': 0, 'note': 'host arrays -> pinned staging -> H2D -> kernels; '
                                                     'the result stays on the device for the encoder'},
            'roofline': {'kernel': 'resample_staged_kernel (+ tables_kernel)', 'bound': 'hbm', 'achieved': achieved,
                         'peak': peaks['hbm_gbs'], 'unit': 'GB/s', 'frac': achieved / peaks['hbm_gbs'],
                         'traffic': _img_traffic(n), 'algorithmic_bytes_per_launch': algo_bytes,
                         'launch_ms': launch_ms, 'peak_kind': f'{peak_kind} HBM copy'},
            'gpu_launches': 2 * args.steps, 'clocks': clocks.summary(),
            'parity': {'images_checked': probe, 'bit_exact_vs_oracle': exact}}
    if not args.no_cpu_baseline:
        m = images_cpu_measure(4 * (os.cpu_count() or 1))
        line['cpu_baseline'] = {'value': m['value'], 'unit': UNIT, 'cores': m['cores'], 'kind': 'reference',
                                'sample': m['sample'], 'timed_s': round(m['wall_s'], 2)}
    print(json.dumps(line), flush=True)


def main():
    args = _args()
    if args.config == 'images':
        (run_images_reference if args.impl == 'reference' else run_images)(args)
        return
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
