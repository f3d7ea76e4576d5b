"""The image workload's reference arm on CPU: one JSON line with the contract's keys.

``bench.py --config images --impl reference`` times the reference's own per-image
transform (PIL bicubic resize, ToTensor, Normalize; ``open_clip/transform.py:124-133``)
on the host cores, so it runs here without a GPU."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def test_images_reference_arm_prints_one_contract_line():
    res = subprocess.run([sys.executable, str(REPO / 'bench.py'), '--config', 'images', '--impl', 'reference',
                          '--steps', '1', '--warmup', '0'], capture_output=True, text=True, timeout=600,
                         cwd=str(REPO))
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith('{')]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better',
                'scaling', 'vs_baseline', 'dtype', 'data', 'config', 'impl', 'cpu_baseline', 'e2e'):
        assert key in line, key
    assert line['impl'] == 'reference' and line['value'] > 0
    assert line['cpu_baseline']['kind'] == 'reference' and line['cpu_baseline']['cores'] >= 1
    assert line['e2e'] == {'value': line['value'], 'unit': line['unit'], 'h2d_bytes_per_step': 0,
                           'd2h_bytes_per_step': 0}
    # the reported step ran: ms_per_step x steps fits the sample's own timing
    assert line['ms_per_step'] >= 1000.0
