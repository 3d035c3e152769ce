"""CPU oracle for the vflash quantised-linear hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference
(Hansimov/vflash) for the FP8 / NVFP4 linear layers and their BF16
epilogues.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm may import it, and only as the checker or the
timed CPU baseline; the product package ``vflash_b200`` never imports it.

Pinning: ``fp8.quantize_activation`` and ``fp8.weight_only_linear`` are
checked bit-for-bit against golden vectors that ``tests/golden/make_golden.py``
produced by importing the reference itself (``tests/test_oracle_golden.py``).
The NVFP4 restatement (``nvfp4``) has no reference CPU path or golden vector
to pin it: its quantiser parity is checked on the GPU against FlashInfer when
that library runs there, otherwise it is unpinned.
"""
