"""vflash_b200 — B200-native (sm_100a) quantised linear layers for the H3 DiT blocks.

Drop-in replacements for the FP8 / NVFP4 linear path of Hansimov/vflash:

* ``vflash_b200.native.h3_fp8_linear``      RowFP8Execution, RowFP8Linear
* ``vflash_b200.native.h3_fp8_activation``  quantize_activation
* ``vflash_b200.native.h3_fused_ops``       strict-BF16 elementwise ops

All arithmetic runs in the native library ``libvflash_b200.so`` (hand-written
CUDA for sm_100a, C ABI in include/vflash_b200.h); there is no host fallback.
"""

__version__ = "0.1.0"
