"""The header is a C ABI: a C99 program compiles against include/musc_b200.h, links the
built library and makes host-only calls (no device work), like a non-Python host would."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which('gcc') is None, reason='no C compiler')
def test_c99_host_builds_links_and_runs(tmp_path):
    from musc_b200 import _lib
    lib = Path(_lib.LIB_PATH)
    exe = tmp_path / 'abi_check'
    subprocess.run(['gcc', '-std=c99', '-Wall', '-Wextra', '-Werror', '-I', str(REPO / 'include'),
                    str(REPO / 'tests' / 'c_abi' / 'abi_check.c'), '-o', str(exe), '-L', str(lib.parent),
                    f'-l:{lib.name}', f'-Wl,-rpath,{lib.parent}'], check=True, capture_output=True, text=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stderr
    assert 'c abi ok' in res.stdout
