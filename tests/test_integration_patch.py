"""The reference-side patch of INTEGRATION.md, applied to copies of the reference's files.

The diff block of INTEGRATION.md section 2 is the whole change a maintainer makes to the
reference (``models/modules/_backend.py`` and ``models/musc.py``).  This test copies the
two files from the reference checkout into a temporary directory, applies the block with
``git apply --ignore-whitespace`` (the reference uses CRLF line endings) and checks that

* it applies cleanly;
* the patched ``select_backend`` keeps the reference's behaviour for its own names and
  raises for ``b200`` / ``b200_super_fast`` where there is no B200 (no fallback), and the
  patched ``configure_backend`` does the same for the super-fast preset;
* the patched ``musc.py`` still compiles and selects the ``b200`` operators and image loader.

The reference checkout is found through ``MUSC_REFERENCE`` (default: the directory
``reference`` beside this repository); where it is absent the test is skipped.
"""
from __future__ import annotations

import ast
import importlib.util
import os
import re
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get('MUSC_REFERENCE', str(REPO.parent / 'reference')))
FILES = ('models/modules/_backend.py', 'models/musc.py')

pytestmark = pytest.mark.skipif(not all((REFERENCE / f).exists() for f in FILES),
                                reason='reference checkout not available')


def _patch_text() -> str:
    text = (REPO / 'INTEGRATION.md').read_text()
    blocks = re.findall(r'```diff\n(.*?)```', text, flags=re.S)
    assert len(blocks) == 1, 'INTEGRATION.md must hold exactly one diff block'
    return blocks[0]


@pytest.fixture()
def patched(tmp_path):
    for f in FILES:
        (tmp_path / f).parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(REFERENCE / f, tmp_path / f)
    patch = tmp_path / 'b200.patch'
    patch.write_text(_patch_text())
    res = subprocess.run(['git', 'apply', '--ignore-whitespace', '--verbose', str(patch)], cwd=tmp_path,
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return tmp_path


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_patch_applies_and_b200_never_falls_back(patched):
    backend = _load(patched / 'models/modules/_backend.py', 'patched_backend')
    # the reference's own names behave as before (this container has no CUDA)
    assert backend.select_backend('original', 'cpu') == ('original', None)
    assert backend.select_backend('gpu', 'cpu') == ('original', 'CUDA is unavailable')
    assert backend.select_backend('super_fast', 'cuda', 'posix')[0] == 'original'
    with pytest.raises(ValueError):
        backend.select_backend('bogus', 'cpu')
    # the new names never fall back
    for name in ('b200', 'b200_super_fast'):
        for device_type in ('cpu', 'cuda'):
            with pytest.raises(RuntimeError):
                backend.select_backend(name, device_type)
    cfg = {'models': {'inference_backend': 'b200_super_fast', 'backbone_name': 'ViT-L-14-336',
                      'pretrained': 'openai', 'batch_size': 4},
           'datasets': {'img_resize': 518, 'divide_num': 1}}
    with pytest.raises(RuntimeError):
        backend.configure_backend(cfg, 'cpu')


def test_patched_musc_selects_the_b200_operators(patched):
    src = (patched / 'models/musc.py').read_text()
    tree = ast.parse(src)                                   # still valid Python
    compile(tree, 'musc.py', 'exec')
    assert "'b200', 'b200_super_fast'" in src
    assert 'gpu_msm = b200.MSM' in src and 'b200.encode_image' in src
    assert 'b200_rscin(ac_score, class_tokens, k_list=k_score, device=self.device)' in src
    # pool images: decoded by the dataset, preprocessed on the device by the b200 loader
    assert 'test_dataset.transform_img = RawRGB()' in src and 'DeviceImageLoader(' in src
    assert 'from models.modules._loader import ThreadedDatasetLoader' in src
    # the reference's own GPU imports are still there for its own backends
    assert 'from models.modules._MSM_gpu import MSM as gpu_msm' in src
