"""NumPy restatement of the reference's INT4 quantize / pack / dequantize / GEMM.

Test infrastructure only (see ``oracle/__init__.py``). Each function names the
reference file:line whose arithmetic it restates. The byte layout of one
super-block (256 weights) is:

    bytes   0..15   8 fp16 group scales, little-endian, group g at bytes 2g..2g+1
    bytes  16..143  128 nibble bytes; byte j holds element 2j in its low nibble
                    and element 2j+1 in its high nibble, each stored as q + 8

(``antigravity-engine/src/dequant.py:119-124``; ``src/dequant.py:128-139``;
Metal ``struct SuperBlock`` in ``antigravity-engine/src/shaders/batched_gemm.metal:17-20``).
Super-block ``i`` holds flat elements ``[256 i, 256 i + 256)`` of the row-major
``[K, M]`` weight (flat index ``k * M + m``, ``batched_gemm_fused.metal:39-45``).
"""

from __future__ import annotations

import numpy as np

GROUP = 32
SB_ELEMS = 256
SB_BYTES = 144


def quantize_engine(w: np.ndarray, group_size: int = GROUP):
    """Engine quantizer, ``antigravity-engine/src/dequant.py:22-60``.

    The fp32 scale ``max|w|/7`` (1.0 for an all-zero group) is rounded to fp16
    FIRST (:57) and the weights are divided by that fp16 scale (:58), then
    round-half-even and clip to [-8, 7]. 1-D input only (:45-50).
    """
    if w.ndim != 1:
        raise ValueError(f"Expected 1D array, got shape {w.shape}")
    if len(w) % group_size != 0:
        raise ValueError(f"Weight length {len(w)} is not divisible by group_size={group_size}")
    g = w.astype(np.float32).reshape(-1, group_size)
    alphas = np.max(np.abs(g), axis=1)
    scales = np.where(alphas == 0, 1.0, alphas / 7.0).astype(np.float16)
    q = np.clip(np.round(g / scales[:, None]), -8, 7).astype(np.int8)
    return q.reshape(-1), scales


def quantize_toplevel(w: np.ndarray, group_size: int = GROUP):
    """Top-level quantizer, ``src/dequant.py:26-55``.

    Any shape; divides by the UNROUNDED fp32 scale (:51-52) and only then stores
    the scale as fp16 (:53). Returns q with the input's shape.
    """
    flat = w.astype(np.float32).flatten()
    assert flat.size % group_size == 0
    g = flat.reshape(-1, group_size)
    max_abs = np.max(np.abs(g), axis=1, keepdims=True)
    scales = np.where(max_abs == 0, 1.0, max_abs / 7.0)
    q = np.clip(np.round(g / scales), -8, 7).astype(np.int8)
    return q.reshape(w.shape), scales.flatten().astype(np.float16)


def pack_superblocks(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """144-byte super-block stream from int8 q and fp16 scales.

    Nibble = q + 8, low nibble = even element, high = odd
    (``antigravity-engine/src/dequant.py:119-124``); the scales header precedes
    the payload (``:79-82``; ``src/dequant.py:128-130``).
    """
    q = np.asarray(q, dtype=np.int8).reshape(-1)
    if q.size % SB_ELEMS != 0:
        raise ValueError(f"Weight length {q.size} not divisible by super-block size {SB_ELEMS}")
    nsb = q.size // SB_ELEMS
    u = (q.astype(np.int16) + 8).astype(np.uint8).reshape(nsb, 128, 2)
    payload = (u[:, :, 0] & 0x0F) | ((u[:, :, 1] & 0x0F) << 4)
    header = np.ascontiguousarray(scales.astype(np.float16).reshape(nsb, 8)).view(np.uint8)
    out = np.empty((nsb, SB_BYTES), dtype=np.uint8)
    out[:, :16] = header
    out[:, 16:] = payload
    return out.reshape(-1)


def unpack_q(stream: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Super-block stream -> (int8 q, fp16 scales), ``antigravity-engine/src/dequant.py:135-156``."""
    sb = np.asarray(stream, dtype=np.uint8).reshape(-1, SB_BYTES)
    scales = np.ascontiguousarray(sb[:, :16]).view(np.float16).reshape(-1)
    pay = sb[:, 16:]
    q = np.empty((sb.shape[0], 128, 2), dtype=np.int8)
    q[:, :, 0] = (pay & 0x0F).astype(np.int8) - 8
    q[:, :, 1] = ((pay >> 4) & 0x0F).astype(np.int8) - 8
    return q.reshape(-1), scales


def dequant(q: np.ndarray, scales: np.ndarray, group_size: int = GROUP) -> np.ndarray:
    """fp16(fp32(q) * fp32(s)), ``antigravity-engine/src/dequant.py:223-252``.

    The product of a 4-bit integer and an fp16 scale is exact in fp32, so this
    single rounding equals the 16-entry LUT of ``:163-220`` bit for bit.
    """
    q32 = np.asarray(q).astype(np.float32).reshape(-1, group_size)
    s32 = np.asarray(scales).astype(np.float32).reshape(-1, 1)
    return (q32 * s32).astype(np.float16).reshape(-1)


def unpack_superblock_weights(stream: np.ndarray) -> np.ndarray:
    """144-byte stream -> fp16 weights, ``src/dequant.py:116-147``."""
    q, s = unpack_q(stream)
    return dequant(q, s)


def gemm(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """fp32 matmul then cast to the weight dtype, ``antigravity-engine/tests/test_batched_speed.py:39-42``."""
    res = x.astype(np.float32) @ w.astype(np.float32)
    return res.astype(w.dtype)


def make_weights(K: int, M: int, seed: int, std: float = 0.02) -> np.ndarray:
    """Seeded fp32 N(0, std) weight [K, M] (the BASELINE configs' weight init)."""
    return np.random.default_rng(seed).normal(0.0, std, size=(K, M)).astype(np.float32)


def make_activations(N: int, K: int, seed: int) -> np.ndarray:
    """Seeded fp16 N(0, 1) activations [N, K]."""
    return np.random.default_rng(seed + 7919).normal(0.0, 1.0, size=(N, K)).astype(np.float16)


def quantize_pack_matrix(w: np.ndarray) -> np.ndarray:
    """Row-major [K, M] weight -> super-block stream via the engine quantizer."""
    q, s = quantize_engine(w.reshape(-1))
    return pack_superblocks(q, s)


def column_shard(stream: np.ndarray, K: int, M: int, c0: int, c1: int) -> np.ndarray:
    """Columns [c0, c1) of a packed [K, M] weight, re-packed as its own [K, c1-c0] stream.

    Bit-identical weights: q and the group scales move unchanged. Needs group-aligned
    boundaries (c0, c1 multiples of 32, M % 32 == 0) and K*(c1-c0) % 256 == 0.
    """
    q, s = unpack_q(stream)
    q = q.reshape(K, M)[:, c0:c1]
    s = s.reshape(K, M // GROUP)[:, c0 // GROUP:c1 // GROUP]
    return pack_superblocks(np.ascontiguousarray(q).reshape(-1), np.ascontiguousarray(s).reshape(-1))
