"""INT4 group-32 quantization, 144-byte super-block packing and LUT dequantization.

Drop-in for the reference's two dequant modules, with the work done by the sm_100a
kernels of ``libmoat_b200.so``:

* top-level ``src/dequant.py`` (re-exported by ``src/__init__.py:3-17``):
  ``ensure_aligned_array``, ``quantize_fp16_to_int4``, ``repack_weights_to_superblock``,
  ``lut_dequantize_fp16``, ``unpack_superblock_weights``, ``calculate_memory_footprint``;
* engine ``antigravity-engine/src/dequant.py``: ``quantize_weights_int4``,
  ``repack_to_superblocks``, ``unpack_superblock``, ``build_dequant_lut``,
  ``lut_dequantize``, ``arithmetic_dequantize`` (its alias
  ``quantize_fp16_to_int4 = quantize_weights_int4`` lives in ``moat_b200.engine_dequant``).

NumPy in -> NumPy out (the data makes a round trip through the GPU); torch CUDA
tensors in -> torch CUDA tensors out. The two quantizers keep the reference's
different semantics: the engine one divides by the fp16-rounded scale, the
top-level one by the unrounded fp32 scale. Besides the 144-byte wire form, the
functions also return the reference's own container types (list of dicts,
``(nsb, 8, 32)`` int8 arrays).
"""

from __future__ import annotations

from typing import Dict, Tuple, Union

import numpy as np

from . import _lib
from ._lib import check, lib, ptr, stream_of, to_device

GROUP_SIZE = 32
SUPERBLOCK_ELEMS = 256
SUPERBLOCK_BYTES = 144


def _out(t, was_np):
    if not was_np:
        return t
    a = t.cpu().numpy()
    return a


def _f16_out(t, was_np):
    if not was_np:
        return t.view(_lib.torch().float16)
    return t.cpu().numpy().view(np.float16)


# ---------------------------------------------------------------------------
# host-side utilities (no device work in the reference either)
# ---------------------------------------------------------------------------
def ensure_aligned_array(arr: np.ndarray, alignment: int = 128) -> np.ndarray:
    """C-contiguous copy whose data pointer is ``alignment``-byte aligned
    (``src/dequant.py:9-23``)."""
    a = np.ascontiguousarray(arr)
    if a.ctypes.data % alignment == 0:
        return a
    buf = np.empty(a.nbytes + alignment, dtype=np.uint8)
    off = (alignment - buf.ctypes.data % alignment) % alignment
    view = buf[off:off + a.nbytes].view(a.dtype).reshape(a.shape)
    np.copyto(view, a)
    return view


def calculate_memory_footprint(num_params: int, group_size: int = 32, bits: int = 4) -> Dict[str, Union[int, float, bool]]:
    """Weight + fp16 scale bytes under group quantization (``src/dequant.py:150-187``)."""
    weight_bytes = num_params * (bits / 8.0)
    scale_bytes = (num_params // group_size) * 2.0
    total = weight_bytes + scale_bytes
    ram_limit_gb = 4.5
    return {
        "num_params": num_params,
        "weight_bytes": weight_bytes,
        "scale_bytes": scale_bytes,
        "total_bytes": total,
        "total_mb": total / (1024 ** 2),
        "total_gb": total / (1024 ** 3),
        "ram_limit_gb": ram_limit_gb,
        "fits_in_ram": total / (1024 ** 3) <= ram_limit_gb,
        "bytes_per_param_effective": total / num_params,
    }


def build_dequant_lut(scale) -> np.ndarray:
    """16-entry table ``LUT[k+8] = fp16(k * scale)`` (``antigravity-engine/src/dequant.py:163-180``)."""
    return (np.arange(-8, 8, dtype=np.float32) * float(scale)).astype(np.float16)


# ---------------------------------------------------------------------------
# quantizers
# ---------------------------------------------------------------------------
def _quantize(weights, variant: int, want_q=True, want_s=True, want_sb=False):
    t = _lib.torch()
    w, was_np = to_device(weights)
    if w.dtype == t.float16:
        is16 = 1
    else:
        w = w.to(t.float32)
        is16 = 0
    n = w.numel()
    dev = w.device
    q = t.empty(n, dtype=t.int8, device=dev) if want_q else None
    s = t.empty(n // GROUP_SIZE, dtype=t.int16, device=dev) if want_s else None
    sb = t.empty(n // SUPERBLOCK_ELEMS * SUPERBLOCK_BYTES, dtype=t.uint8, device=dev) if want_sb else None
    check(lib().mb_int4_quantize(ptr(w), is16, n, variant, ptr(q) if q is not None else None,
                                 ptr(s) if s is not None else None, ptr(sb) if sb is not None else None,
                                 stream_of(dev)), "mb_int4_quantize")
    return q, s, sb, was_np


def quantize_weights_int4(weights_fp16, group_size: int = 32) -> Tuple[np.ndarray, np.ndarray]:
    """Engine quantizer (``antigravity-engine/src/dequant.py:22-60``): 1-D input only,
    scale = fp16(max|w| / 7) (1.0 for a zero group), q = clip(round(w / scale), -8, 7)."""
    if len(weights_fp16.shape) != 1:
        raise ValueError(f"Expected 1D array, got shape {tuple(weights_fp16.shape)}")
    if weights_fp16.shape[0] % group_size != 0:
        raise ValueError(f"Weight length {weights_fp16.shape[0]} is not divisible by group_size={group_size}")
    if group_size != GROUP_SIZE:
        raise NotImplementedError("the super-block format fixes group_size = 32")
    q, s, _, was_np = _quantize(weights_fp16, 0)
    return _out(q, was_np), _f16_out(s, was_np)


def quantize_fp16_to_int4(weights_fp16, group_size: int = 32) -> Tuple[np.ndarray, np.ndarray]:
    """Top-level quantizer (``src/dequant.py:26-55``): any shape, divides by the
    unrounded fp32 scale, returns q with the input's shape and fp16 scales."""
    size = int(np.prod(weights_fp16.shape))
    assert size % group_size == 0, (
        f"Weight array length ({size}) must be a multiple of group_size ({group_size}).")
    if group_size != GROUP_SIZE:
        raise NotImplementedError("the super-block format fixes group_size = 32")
    q, s, _, was_np = _quantize(weights_fp16, 1)
    q = _out(q, was_np)
    return q.reshape(tuple(weights_fp16.shape)), _f16_out(s, was_np)


def quantize_to_superblocks(weights, variant: str = "engine"):
    """Quantize (engine or top-level semantics) straight into the 144-byte stream.

    Not in the reference as one call; equals ``repack_to_superblocks`` applied to
    the quantizer's output. Returns uint8[n/256*144].
    """
    v = {"engine": 0, "toplevel": 1}[variant]
    n = int(np.prod(weights.shape))
    if n % SUPERBLOCK_ELEMS != 0:
        raise ValueError(f"Weight length {n} not divisible by super-block size {SUPERBLOCK_ELEMS}")
    _, _, sb, was_np = _quantize(weights, v, want_q=False, want_s=False, want_sb=True)
    return _out(sb, was_np)


# ---------------------------------------------------------------------------
# packing
# ---------------------------------------------------------------------------
def pack_superblocks(q_weights, scales):
    """int8 q + fp16 scales -> contiguous 144-byte super-block stream (uint8)."""
    t = _lib.torch()
    q, was_np = to_device(q_weights, t.int8)
    s, _ = to_device(np.asarray(scales).astype(np.float16).view(np.int16) if not isinstance(scales, t.Tensor)
                     else scales.view(t.int16), None, q.device)
    n = q.numel()
    if n % SUPERBLOCK_ELEMS != 0:
        raise ValueError(f"Weight length {n} not divisible by super-block size {SUPERBLOCK_ELEMS}")
    out = t.empty(n // SUPERBLOCK_ELEMS * SUPERBLOCK_BYTES, dtype=t.uint8, device=q.device)
    check(lib().mb_int4_pack(ptr(q), ptr(s), n, ptr(out), stream_of(q.device)), "mb_int4_pack")
    return _out(out, was_np)


def repack_to_superblocks(q_weights, scales, group_size: int = 32, groups_per_superblock: int = 8) -> list:
    """List of ``{'scales', 'packed_nibbles', 'raw_int4'}`` dicts, one per super-block
    (``antigravity-engine/src/dequant.py:69-132``); the bytes come from the GPU packer."""
    elems = group_size * groups_per_superblock
    n = len(q_weights)
    if n % elems != 0:
        raise ValueError(f"Weight length {n} not divisible by super-block size {elems}")
    if group_size != GROUP_SIZE or groups_per_superblock != 8:
        raise NotImplementedError("the super-block format fixes 8 groups of 32")
    stream = np.asarray(pack_superblocks(q_weights, scales) if not _is_torch(q_weights)
                        else pack_superblocks(q_weights, scales).cpu().numpy())
    sbs = stream.reshape(-1, SUPERBLOCK_BYTES)
    q_host = np.asarray(q_weights.cpu().numpy() if _is_torch(q_weights) else q_weights)
    out = []
    for i in range(sbs.shape[0]):
        out.append({
            "scales": sbs[i, :16].copy().view(np.float16),
            "packed_nibbles": sbs[i, 16:].copy(),
            "raw_int4": q_host[i * elems:(i + 1) * elems].copy(),
        })
    return out


def superblocks_to_stream(superblocks: list) -> np.ndarray:
    """The 144-byte wire form (Metal ``struct SuperBlock``) of a dict list."""
    return np.concatenate([np.concatenate([np.asarray(sb["scales"], np.float16).view(np.uint8),
                                           np.asarray(sb["packed_nibbles"], np.uint8)]) for sb in superblocks])


def unpack_superblock(superblock: dict, group_size: int = 32) -> np.ndarray:
    """A super-block dict's nibbles -> int8[256] in [-8, 7]
    (``antigravity-engine/src/dequant.py:135-156``)."""
    t = _lib.torch()
    raw = np.zeros(SUPERBLOCK_BYTES, dtype=np.uint8)
    raw[16:] = np.asarray(superblock["packed_nibbles"], dtype=np.uint8)
    d, _ = to_device(raw)
    q = t.empty(SUPERBLOCK_ELEMS, dtype=t.int8, device=d.device)
    check(lib().mb_int4_unpack(ptr(d), 1, ptr(q), None, stream_of(d.device)), "mb_int4_unpack")
    return q.cpu().numpy()


def unpack_superblocks(stream_bytes):
    """144-byte stream -> (int8 q, fp16 scales)."""
    t = _lib.torch()
    d, was_np = to_device(stream_bytes, t.uint8)
    nsb = d.numel() // SUPERBLOCK_BYTES
    q = t.empty(nsb * SUPERBLOCK_ELEMS, dtype=t.int8, device=d.device)
    s = t.empty(nsb * 8, dtype=t.int16, device=d.device)
    check(lib().mb_int4_unpack(ptr(d), nsb, ptr(q), ptr(s), stream_of(d.device)), "mb_int4_unpack")
    return _out(q, was_np), _f16_out(s, was_np)


def repack_weights_to_superblock(weights_int4, group_size: int = 32):
    """``(num_superblocks, 8, group_size)`` int8 view, 128-byte aligned
    (``src/dequant.py:58-76``). A reshape, no arithmetic."""
    if _is_torch(weights_int4):
        flat = weights_int4.reshape(-1)
        assert flat.numel() % 256 == 0, "Weight array length must be a multiple of 256."
        return flat.reshape(-1, 8, group_size).to(_lib.torch().int8).contiguous()
    flat = np.asarray(weights_int4).flatten()
    assert len(flat) % 256 == 0, "Weight array length must be a multiple of 256."
    return ensure_aligned_array(flat.reshape(len(flat) // 256, 8, group_size).astype(np.int8), alignment=128)


# ---------------------------------------------------------------------------
# dequantization (bit-exact: fp16(q * s), one rounding)
# ---------------------------------------------------------------------------
def unpack_superblock_weights(superblock_bytes, num_superblocks: int):
    """144-byte stream -> fp16[num_superblocks * 256] (``src/dequant.py:116-147``;
    Metal ``dequantize_superblocks_kernel``, batched_gemm.metal:41-66)."""
    t = _lib.torch()
    d, was_np = to_device(superblock_bytes, t.uint8)
    if d.numel() != num_superblocks * SUPERBLOCK_BYTES:
        raise ValueError(f"expected {num_superblocks * SUPERBLOCK_BYTES} bytes, got {d.numel()}")
    out = t.empty(num_superblocks * SUPERBLOCK_ELEMS, dtype=t.int16, device=d.device)
    check(lib().mb_int4_dequant(ptr(d), ptr(out), num_superblocks, stream_of(d.device)), "mb_int4_dequant")
    return _f16_out(out, was_np)


def _dequant_q(q_weights, scales, group_size):
    t = _lib.torch()
    q, was_np = to_device(q_weights, t.int8)
    s, _ = to_device(np.asarray(scales).astype(np.float16).view(np.int16) if not _is_torch(scales)
                     else scales.view(t.int16), None, q.device)
    n = q.numel()
    ng = n // group_size
    if ng == 0:
        return _f16_out(t.zeros(n, dtype=t.int16, device=q.device), was_np)
    n_used = ng * group_size
    out = t.zeros(n, dtype=t.int16, device=q.device)
    check(lib().mb_int4_dequant_q(ptr(q), ptr(s), n_used, group_size, ptr(out), stream_of(q.device)),
          "mb_int4_dequant_q")
    return _f16_out(out, was_np)


def lut_dequantize(q_weights, scales, group_size: int = 32):
    """Per-group 16-entry LUT dequant (``antigravity-engine/src/dequant.py:183-220``).
    ``LUT[k+8] = fp16(k * s)`` is exactly ``fp16(q * s)``, which the kernel computes."""
    return _dequant_q(q_weights, scales, group_size)


def arithmetic_dequantize(q_weights, scales, group_size: int = 32):
    """``fp16(q * s)`` (``antigravity-engine/src/dequant.py:223-252``)."""
    return _dequant_q(q_weights, scales, group_size)


def _lut_indices(q_weights, max_idx: int) -> np.ndarray:
    """Index rule of ``lut_dequantize_fp16`` (``src/dequant.py:86-94``)."""
    q = np.asarray(q_weights)
    if q.dtype == np.int8:
        idx = q.astype(np.int32) + 8
    elif np.issubdtype(q.dtype, np.signedinteger):
        idx = q.astype(np.int32) + 8 if q.size and np.min(q) < 0 else q.astype(np.int32)
    else:
        idx = q.astype(np.int32)
    return idx


def lut_dequantize_fp16(q_weights, lut):
    """Table-gather dequantization with a 1-D, 2-D (per group) or 3-D (per
    super-block and group) fp16 LUT (``src/dequant.py:79-113``)."""
    lut_np = np.asarray(lut)
    lut16 = lut_np.astype(np.float16) if lut_np.dtype != np.float16 else lut_np
    if lut16.ndim not in (1, 2, 3):
        raise ValueError(f"Unsupported LUT shape {lut_np.shape}. Must be 1D, 2D, or 3D.")
    q_np = np.asarray(q_weights.cpu().numpy() if _is_torch(q_weights) else q_weights)
    cols = lut16.shape[-1]
    idx = _lut_indices(q_np, cols - 1)
    rows = 1 if lut16.ndim == 1 else int(np.prod(lut16.shape[:-1]))
    n = idx.size
    group_len = max(1, n // rows) if rows > 1 else max(1, n)
    t = _lib.torch()
    di, _ = to_device(idx.reshape(-1))
    dl, _ = to_device(np.ascontiguousarray(lut16.reshape(-1)).view(np.int16), None, di.device)
    out = t.empty(n, dtype=t.int16, device=di.device)
    if n:
        check(lib().mb_lut_gather_f16(ptr(di), n, ptr(dl), rows, cols, group_len, ptr(out), stream_of(di.device)),
              "mb_lut_gather_f16")
    return out.cpu().numpy().view(np.float16).reshape(q_np.shape)


def extract_columns(superblocks, K: int, M: int, c0: int, c1: int):
    """Columns [c0, c1) of a packed [K, M] weight as their own [K, c1-c0] stream
    (bit-identical q and scales). Used to column-shard M across GPUs."""
    t = _lib.torch()
    d, was_np = to_device(superblocks, t.uint8)
    out = t.empty(K * (c1 - c0) // SUPERBLOCK_ELEMS * SUPERBLOCK_BYTES, dtype=t.uint8, device=d.device)
    check(lib().mb_int4_extract_columns(ptr(d), K, M, c0, c1, ptr(out), stream_of(d.device)),
          "mb_int4_extract_columns")
    return _out(out, was_np)


def _is_torch(x) -> bool:
    try:
        import torch
    except ImportError:  # pragma: no cover
        return False
    return isinstance(x, torch.Tensor)
