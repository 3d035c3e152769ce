"""Build FlashInfer's sm_100a NVFP4 modules from their source, for the GPU parity tests.

The reference's NVFP4 arithmetic lives in FlashInfer (Hansimov/vflash pins
``flashinfer-python==0.6.18``; this image has 0.6.11.post2).  FlashInfer
compiles these CUDA modules just in time with nvcc; a fresh GPU box would
rebuild them on every test run.  This script builds them once, here (no GPU
needed), into ``tests/.flashinfer_ref`` (git-ignored; it travels with the
working tree), and the tests point FlashInfer's workspace there:

    python tests/golden/build_flashinfer_reference.py [--gemm]

``--gemm`` also builds the CUTLASS FP4 GEMM behind ``mm_fp4(backend="cutlass")``
(several minutes).  The modules are only run as the checker, never read.
"""

from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

WORKSPACE = Path(__file__).resolve().parent.parent / ".flashinfer_ref"
ARCH_LIST = "10.0a"


def configure_environment() -> None:
    """Point FlashInfer's JIT workspace at the in-tree cache (call before importing flashinfer)."""
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(WORKSPACE))
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", ARCH_LIST)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gemm", action="store_true")
    args = parser.parse_args()
    configure_environment()
    from flashinfer.jit.fp4_quantization import gen_fp4_quantization_sm100_module

    specs = [gen_fp4_quantization_sm100_module()]
    if args.gemm:
        from flashinfer.jit.gemm.core import gen_gemm_sm100_module_cutlass_fp4

        specs.append(gen_gemm_sm100_module_cutlass_fp4())
    for spec in specs:
        t0 = time.time()
        spec.build(verbose=False)
        print(f"built {spec.name} in {time.time() - t0:.0f} s", file=sys.stderr)


if __name__ == "__main__":
    main()
