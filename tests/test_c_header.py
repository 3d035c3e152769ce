"""The C ABI is usable from plain C and from C++: the header compiles, the library links and answers.

A small C99 program (and the same file as C++) includes include/vflash_b200.h,
links against the built library and calls entry points that need no GPU:
the version string, a workspace query, and argument validation that must
fail with VFB_EINVAL and a message before any device work.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "vflash_b200"

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "vflash_b200.h"

int main(void) {
  const char *version = vfb_version();
  if (version == NULL || strlen(version) == 0) return 10;
  if (vfb_fp8_ffn_workspace_bytes(10, 64, 64) != 4096) return 11;
  if (vfb_fp8_ffn_workspace_bytes(10, 48, 64) != -1) return 12;
  vfb_epilogue ep;
  memset(&ep, 0, sizeof ep);
  ep.kind = VFB_EPI_STORE;
  /* N = 48 is not a multiple of 32: refused before anything runs */
  if (vfb_fp8_gemm(NULL, 64, NULL, NULL, 64, NULL, 4, 48, 64, &ep, NULL) != VFB_EINVAL) return 13;
  if (strstr(vfb_last_error(), "vfb_fp8_gemm") == NULL) return 14;
  if (vfb_bf16_gemm(NULL, 64, NULL, 64, 4, 64, 12, &ep, NULL) != VFB_EINVAL) return 15;
  printf("%s|%zu\n", version, sizeof(vfb_epilogue));
  return 0;
}
"""


def build_and_run(tmp_path: Path, compiler: str, std: str, suffix: str) -> str:
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} is not installed")
    if not (LIB_DIR / "libvflash_b200.so").exists():
        pytest.skip("the library is not built")
    source = tmp_path / f"abi{suffix}"
    source.write_text(PROGRAM)
    exe = tmp_path / f"abi_{compiler}"
    cmd = [compiler, f"-std={std}", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(source), "-o", str(exe),
           f"-L{LIB_DIR}", "-lvflash_b200", f"-Wl,-rpath,{LIB_DIR}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    result = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=120)
    assert result.returncode == 0, (result.returncode, result.stdout, result.stderr)
    return result.stdout.strip()


def test_header_compiles_as_c99_and_links(tmp_path):
    version, size = build_and_run(tmp_path, "gcc", "c99", ".c").split("|")
    assert version and int(size) == 192


def test_header_compiles_as_cpp17_and_links(tmp_path):
    version, size = build_and_run(tmp_path, "g++", "c++17", ".cpp").split("|")
    assert version and int(size) == 192
