"""Namespace mirroring ``antigravity-engine/src/dequant.py`` exactly, including its
alias ``quantize_fp16_to_int4 = quantize_weights_int4`` (:62), which differs from the
top-level ``src/dequant.py`` function of the same name."""

from .dequant import (  # noqa: F401
    arithmetic_dequantize,
    build_dequant_lut,
    lut_dequantize,
    quantize_weights_int4,
    repack_to_superblocks,
    unpack_superblock,
)

quantize_fp16_to_int4 = quantize_weights_int4
