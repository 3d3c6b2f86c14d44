"""moat_b200 — B200-native (sm_100a) INT4 super-block batched GEMM and exp-LUT decode
attention, a drop-in for the data-parallel hot path of chzchzchzchz/moat
("Project Antigravity").

Modules:
  dequant         quantize / pack / dequantize (src/dequant.py + engine dequant API)
  engine_dequant  antigravity-engine/src/dequant.py namespace (with its alias)
  attention       ExponentialLUT, safe_softmax_lut, reference_softmax, decode_attention
  gemm            batched_gemm (fused INT4 weight-streaming kernel)
  dist            column / head sharding across GPUs joined by an all-gather

The top-level names mirror ``src/__init__.py:3-17`` of the reference.
"""

from .dequant import (  # noqa: F401
    calculate_memory_footprint,
    ensure_aligned_array,
    lut_dequantize_fp16,
    quantize_fp16_to_int4,
    repack_weights_to_superblock,
    unpack_superblock_weights,
)

__all__ = [
    "repack_weights_to_superblock",
    "lut_dequantize_fp16",
    "quantize_fp16_to_int4",
    "unpack_superblock_weights",
    "calculate_memory_footprint",
]

__version__ = "0.1.0"
