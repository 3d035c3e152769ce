"""The fused FFN kernel's work order (vflash_b200/csrc/ffn_plan.h), checked on the host.

The kernel hands out work items from one global counter in this order; it is
deadlock-free and correct only if every up and down tile appears exactly once
and every down tile of a row block comes after all of that row block's up
tiles.  tests/ffn_schedule_check.cpp enumerates the order with the kernel's
own decoder (compiled here with the host compiler) and checks both.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    exe = tmp_path_factory.mktemp("plan") / "ffn_schedule_check"
    subprocess.run([cxx, "-std=c++17", "-O1", f"-I{ROOT / 'vflash_b200' / 'csrc'}",
                    str(ROOT / "tests" / "ffn_schedule_check.cpp"), "-o", str(exe)], check=True)
    return exe


BASE = [
    # R, ju, jd, group, band_up, band_down, lead
    (128, 64, 16, 4, 12, 3, 148),    # config 2 GELU: M = 32760, F = 16384, H = 4096
    (128, 128, 16, 4, 12, 3, 148),   # config 2 SwiGLU (128 value + 128 gate columns per up tile)
    (40, 56, 21, 4, 12, 3, 148),     # H3 shape: F = 14336, H = 5376, M = 10000
    (1, 64, 16, 4, 12, 3, 148),      # one row block
    (3, 5, 2, 4, 2, 1, 7),           # one partial group
    (9, 7, 3, 4, 3, 2, 0),           # no lead, last group partial
    (10, 3, 5, 2, 8, 8, 1),          # bands wider than the grid
    (17, 4, 4, 1, 1, 1, 2),          # groups of one row block
]
# every case with the down tiles one, two and three groups behind their up tiles
CASES = [(*c, lag) for c in BASE for lag in (1, 2, 3)]


@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_every_tile_once_and_down_after_up(checker, case):
    out = subprocess.run([str(checker), *map(str, case)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    r, ju, jd = case[:3]
    assert out.stdout.strip() == f"ok {r * (ju + jd)}"
