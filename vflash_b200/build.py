"""Build the sm_100a shared library ``libvflash_b200.so`` in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled to an object for
``-gencode arch=compute_100a,code=sm_100a`` (in parallel), then the objects
are linked into one shared library next to this file with the CUDA runtime
linked statically, so the library needs only the driver at run time.
No CUDA device is needed to build.

    python -m vflash_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
BUILD_DIR = PACKAGE.parent / "_build"
LIBRARY = PACKAGE / "libvflash_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    candidates = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for candidate in candidates:
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build vflash_b200")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(path.stat().st_mtime > mtime for path in inputs)


def _compile(nvcc: str, source: Path, obj: Path, verbose: bool, extra: list[str]) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c",
           str(source), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(f"--- {source.name}\n{result.stdout}{result.stderr}", file=sys.stderr)


def build_library(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile (if stale) and link the library; returns its path."""
    extra = list(extra or [])
    sources = _sources()
    headers = _headers()
    if not force and not _stale(LIBRARY, sources + headers + [Path(__file__)]):
        return LIBRARY
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    objects = [BUILD_DIR / (src.stem + ".o") for src in sources]
    jobs = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        for src, obj in zip(sources, objects, strict=True):
            if force or verbose or _stale(obj, [src, *headers, Path(__file__)]):
                jobs.append(pool.submit(_compile, nvcc, src, obj, verbose, extra))
        for job in jobs:
            job.result()
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
           *map(str, objects)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = parser.parse_args()
    print(build_library(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
