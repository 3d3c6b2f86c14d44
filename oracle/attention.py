"""NumPy restatement of the reference's exp-LUT safe softmax and decode attention.

Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import numpy as np


def exp_table(size: int = 32768, range_max: float = 10.0) -> np.ndarray:
    """fp16(exp(linspace(-r, 0, size, f32))), ``antigravity-engine/src/attention.py:50-51``."""
    xs = np.linspace(-range_max, 0.0, size, dtype=np.float32)
    return np.exp(xs).astype(np.float16)


def step32(size: int, range_max: float) -> np.float32:
    """``step = r / (size - 1)`` (:54), a Python float that NumPy 2 casts to fp32
    before dividing an fp32 array by it (NEP 50 weak scalar)."""
    return np.float32(range_max / (size - 1))


def lut_lookup(table: np.ndarray, range_max: float, x: np.ndarray) -> np.ndarray:
    """``ExponentialLUT.lookup``, ``attention.py:60-85``.

    idx = trunc(clip(|x| / step, 0, size-1)) with an IEEE fp32 divide; result is
    ``table[size - 1 - idx]`` (fp16).
    """
    size = table.shape[0]
    ax = np.abs(np.asarray(x).astype(np.float32))
    idx = np.clip(ax / step32(size, range_max), 0, size - 1).astype(np.intp)
    return table[size - 1 - idx]


def safe_softmax_lut(x: np.ndarray, table: np.ndarray, range_max: float, axis: int = -1) -> np.ndarray:
    """``safe_softmax_lut``, ``attention.py:97-134``: fp32 max-subtract, LUT exp,
    fp32 sum with a zero-sum guard, fp32 divide, fp16 result."""
    xf = np.asarray(x).astype(np.float32)
    m = np.max(xf, axis=axis, keepdims=True)
    e = lut_lookup(table, range_max, xf - m).astype(np.float32)
    s = np.sum(e, axis=axis, keepdims=True)
    s = np.where(s > 0, s, np.float32(1.0))
    return (e / s).astype(np.float16)


def reference_softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Exact-exp softmax, ``attention.py:141-158``."""
    xf = np.asarray(x).astype(np.float32)
    e = np.exp(xf - np.max(xf, axis=axis, keepdims=True))
    return (e / np.sum(e, axis=axis, keepdims=True)).astype(np.float16)


def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, table: np.ndarray,
                     range_max: float, scale: float | None = None, exact: bool = False) -> np.ndarray:
    """LUT-softmax decode attention for one query token per (trace, head).

    The reference composes it from three pieces: fp32 scores ``q . k / sqrt(d)``
    (``antigravity-engine/src/shaders/transformer_ops.metal:94-123``), the LUT
    softmax above producing fp16 probabilities (``attention.py:97-134``; its
    decode call sites are ``batch_generator.py:226,234``), and the fp32
    probability-weighted sum of V (``transformer_ops.metal:186-214``) stored as fp16.

    q [T, H, d], k/v [T, H, L, d] fp16 -> out [T, H, d] fp16.
    ``exact=True`` swaps in the exact-exp softmax (``attention.py:141-158``).
    """
    d = q.shape[-1]
    sc = np.float32(1.0 / np.sqrt(d)) if scale is None else np.float32(scale)
    s = np.einsum("thd,thld->thl", q.astype(np.float32), k.astype(np.float32)) * sc
    p = reference_softmax(s) if exact else safe_softmax_lut(s, table, range_max)
    out = np.einsum("thl,thld->thd", p.astype(np.float32), v.astype(np.float32))
    return out.astype(np.float16)


def make_attention_inputs(T: int, H: int, L: int, d: int, seed: int):
    """Seeded fp16 N(0,1) q [T,H,d] and K, V [T,H,L,d] (BASELINE config 4 init)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, H, d), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((T, H, L, d), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((T, H, L, d), dtype=np.float32).astype(np.float16)
    return q, k, v
