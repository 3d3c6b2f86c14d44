"""32,768-entry fp16 exp LUT, LUT safe softmax and LUT decode attention.

Drop-in for ``antigravity-engine/src/attention.py`` (``ExponentialLUT``,
``safe_softmax_lut``, ``reference_softmax``) plus ``decode_attention``, the decode
attention the reference composes from ``gqa_attention_scores_kernel``
(``transformer_ops.metal:94-123``), the LUT softmax and ``attention_value_kernel``
(``transformer_ops.metal:186-214``).

The table is built on the host with NumPy exactly as the reference builds it (the
device never re-evaluates ``exp``), copied once per device, and looked up by the
sm_100a kernels with the reference's index rule (IEEE fp32 divide, truncation).
"""

from __future__ import annotations

from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, lib, ptr, stream_of, to_device

_pool = _lib.WorkspacePool()


class ExponentialLUT:
    """fp16 table of ``exp`` over ``[-range_max, 0]`` with ``size`` entries
    (``attention.py:21-90``)."""

    def __init__(self, size: int = 32768, range_max: float = 10.0):
        if size < 2:
            raise ValueError(f"LUT size must be >= 2, got {size}")
        if range_max <= 0:
            raise ValueError(f"range_max must be positive, got {range_max}")
        self.size = size
        self.range_max = range_max
        self.inputs = np.linspace(-range_max, 0.0, size, dtype=np.float32)
        self.lut = np.exp(self.inputs).astype(np.float16)
        self.step = range_max / (size - 1)
        assert abs(float(self.lut[-1]) - 1.0) < 0.01, f"LUT endpoint should be ~1.0, got {self.lut[-1]}"
        self._dev = {}

    def device_table(self, device):
        key = str(device)
        tbl = self._dev.get(key)
        if tbl is None:
            tbl, _ = to_device(self.lut.view(np.int16), None, device)
            self._dev[key] = tbl
        return tbl

    def lookup(self, x_shifted):
        """``table[size-1-trunc(clip(|x| / step, 0, size-1))]`` on the GPU (``attention.py:60-85``)."""
        t = _lib.torch()
        x, was_np = to_device(x_shifted, t.float32)
        out = t.empty(x.shape, dtype=t.int16, device=x.device)
        if x.numel():
            check(lib().mb_exp_lut_lookup(ptr(self.device_table(x.device)), self.size, float(self.range_max),
                                          ptr(x), x.numel(), ptr(out), stream_of(x.device)), "mb_exp_lut_lookup")
        if was_np:
            return out.cpu().numpy().view(np.float16).reshape(np.shape(x_shifted))
        return out.view(t.float16)

    @property
    def memory_bytes(self) -> int:
        return self.lut.nbytes


def safe_softmax_lut(x, exp_lut: ExponentialLUT, axis: int = -1):
    """LUT softmax along ``axis``: fp32 max-subtract, LUT exp, fp32 sum, fp16 result
    (``attention.py:97-134``)."""
    t = _lib.torch()
    xd, was_np = to_device(x, t.float32)
    nd = xd.dim()
    ax = axis % nd if nd else 0
    moved = xd.movedim(ax, -1).contiguous() if nd and ax != nd - 1 else xd
    cols = moved.shape[-1] if nd else 1
    rows = moved.numel() // max(cols, 1)
    out = t.empty(moved.shape, dtype=t.int16, device=xd.device)
    if rows:
        check(lib().mb_lut_softmax(ptr(moved), rows, cols, ptr(exp_lut.device_table(xd.device)), exp_lut.size,
                                   float(exp_lut.range_max), ptr(out), stream_of(xd.device)), "mb_lut_softmax")
    out = out.view(t.float16)
    if nd and ax != nd - 1:
        out = out.movedim(-1, ax).contiguous()
    if was_np:
        return out.cpu().numpy()
    return out


def reference_softmax(x, axis: int = -1):
    """Exact-exp softmax used for validation (``attention.py:141-158``)."""
    if isinstance(x, np.ndarray):
        xf = x.astype(np.float32)
        e = np.exp(xf - np.max(xf, axis=axis, keepdims=True))
        return (e / np.sum(e, axis=axis, keepdims=True)).astype(np.float16)
    t = _lib.torch()
    xf = x.float()
    return t.softmax(xf, dim=axis).to(t.float16)


def decode_attention(q, k_cache, v_cache, exp_lut: ExponentialLUT, scale: Optional[float] = None, out=None):
    """LUT-softmax attention of one query token per (trace, head).

    q ``[T, H, d]``, k_cache / v_cache ``[T, H, L, d]`` fp16 -> out ``[T, H, d]`` fp16:
    ``s = (q . k) * scale`` (fp32, default ``1/sqrt(d)``), ``p = safe_softmax_lut(s)``
    (fp16), ``out = sum_l p_l v_l`` (fp32 accumulation).
    """
    t = _lib.torch()
    qd, was_np = to_device(q, t.float16)
    kd, _ = to_device(k_cache, t.float16, qd.device)
    vd, _ = to_device(v_cache, t.float16, qd.device)
    T, H, d = qd.shape
    L = kd.shape[2]
    if tuple(kd.shape) != (T, H, L, d) or tuple(vd.shape) != (T, H, L, d):
        raise ValueError("k_cache / v_cache must be [T, H, L, d] matching q [T, H, d]")
    sc = float(np.float32(1.0 / np.sqrt(d))) if scale is None else float(scale)
    if out is None:
        out = t.empty((T, H, d), dtype=t.float16, device=qd.device)
    st = stream_of(qd.device)
    nbytes = int(lib().mb_decode_attn_workspace_size(T, H, L, d))
    ws = _pool.get(qd.device, st, nbytes)
    check(lib().mb_decode_attn(ptr(qd), ptr(kd), ptr(vd), ptr(out), T, H, L, d, sc,
                               ptr(exp_lut.device_table(qd.device)), exp_lut.size, float(exp_lut.range_max),
                               ptr(ws), ws.numel(), st), "mb_decode_attn")
    if was_np:
        return out.cpu().numpy()
    return out


def attention_bytes(T: int, H: int, L: int, d: int) -> int:
    """Algorithmic HBM bytes of one decode attention call: K and V once, q and out."""
    return 2 * T * H * L * d * 2 + 2 * T * H * d * 2


__all__ = ["ExponentialLUT", "safe_softmax_lut", "reference_softmax", "decode_attention", "attention_bytes"]
