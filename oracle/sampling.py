"""CPU oracle (test infrastructure only) for token choice: greedy over a column-split
vocabulary, and the reference's batched sampler.

Greedy choice in the reference is ``numpy.argmax`` over one row of logits
(antigravity-engine/src/batch_generator.py:224-227; the torch branch at :203-206):
the first index of the largest value, a NaN counting as the largest, -0 equal to +0.
With the vocabulary split over tensor-parallel ranks, each rank reduces its columns to
one 64-bit key, ``code << 32 | (0xFFFFFFFF - column)``, where ``code`` is an
order-preserving 16-bit image of the fp16 value; the integer maximum of the keys of
all ranks names the same column as numpy.argmax of the whole row.

The sampler (``sample_tokens``) restates ``BatchedRolloutCoordinator.sample_tokens``
(NumPy branch, batch_generator.py:187-253) with its random draws given. Only
``tests/``, ``smoke()`` and the bench's CPU arms import this module.
"""

from __future__ import annotations

import numpy as np


def argmax_code(bits: np.ndarray) -> np.ndarray:
    """Order-preserving code (uint32 in [0, 0xFFFF]) of fp16 bit patterns."""
    h = np.asarray(bits, dtype=np.uint16).astype(np.uint32)
    nan = ((h & 0x7C00) == 0x7C00) & ((h & 0x03FF) != 0)
    h = np.where(h == 0x8000, 0, h)
    code = np.where((h & 0x8000) != 0, (~h) & 0xFFFF, h | 0x8000)
    return np.where(nan, 0xFFFF, code).astype(np.uint32)


def argmax_keys(logits: np.ndarray, col0: int = 0) -> np.ndarray:
    """int64 [N]: the best key of each row of fp16 ``logits [N, V]`` whose first column
    is global column ``col0``."""
    x = np.ascontiguousarray(logits, dtype=np.float16)
    code = argmax_code(x.view(np.uint16)).astype(np.uint64)
    cols = np.arange(col0, col0 + x.shape[1], dtype=np.uint64)
    keys = (code << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - cols)
    return keys.max(axis=1).astype(np.int64)


def keys_to_ids(keys: np.ndarray) -> np.ndarray:
    k = np.asarray(keys, dtype=np.int64).astype(np.uint64)
    return (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int32)


def reference_argmax(logits: np.ndarray) -> np.ndarray:
    """numpy.argmax of the fp16 rows, the reference's greedy choice."""
    return np.argmax(np.asarray(logits, dtype=np.float16), axis=-1).astype(np.int32)


# ---------------------------------------------------------------------------
# Batched sampling: BatchedRolloutCoordinator.sample_tokens, NumPy branch
# (antigravity-engine/src/batch_generator.py:187-253)
# ---------------------------------------------------------------------------
TOP_K = 50


def scaled_logits(logits: np.ndarray, temperature: float) -> np.ndarray:
    """``logits / max(temperature, 1e-5)`` with NumPy 2 scalar rules (:232): an fp16
    array stays fp16 (the temperature rounded to fp16, the quotient of the fp32 values
    rounded to fp16); an fp32 array is divided by the fp32 temperature. Temperature
    <= 0 leaves the logits as they are (the greedy branch, :224-228)."""
    x = np.asarray(logits)
    if temperature <= 0:
        return x
    t = max(float(temperature), 1e-5)
    with np.errstate(over="ignore"):
        if x.dtype == np.float16:
            return (x.astype(np.float32) / np.float32(np.float16(t))).astype(np.float16)
        return x.astype(np.float32) / np.float32(t)


def lut_probs16(x: np.ndarray, table: np.ndarray, range_max: float) -> np.ndarray:
    """``safe_softmax_lut`` (attention.py:97-134) of each row: fp32 shift by the row
    maximum, the table index ``trunc(min(|x - m| / step, S-1))`` in fp32, fp16 output.
    The row sum of the fp16 table values is formed exactly and rounded to fp32 once
    (every table value is a multiple of 2^-24, so the float64 sum is exact); NumPy's
    pairwise float32 sum in the reference can differ from it in the last place."""
    from .attention import step32
    S = table.shape[0]
    xf = np.asarray(x).astype(np.float32)
    m = xf.max(axis=-1, keepdims=True)
    a = np.abs(xf - m)
    idx = np.clip(a / step32(S, range_max), 0, S - 1).astype(np.int64)
    e = table[S - 1 - idx].astype(np.float32)
    tot = e.astype(np.float64).sum(axis=-1, keepdims=True).astype(np.float32)
    tot = np.where(tot > 0, tot, np.float32(1.0))
    return (e / tot).astype(np.float16)


def top_candidates(p16_row: np.ndarray, k: int) -> np.ndarray:
    """Column indices of the k largest fp16 probabilities of one row, ordered by
    probability (descending) then column (ascending). The reference takes the same
    set with ``np.argpartition`` (:242), whose order among equal values is unspecified;
    this fixed order is the one the kernel implements."""
    cols = np.arange(p16_row.shape[0])
    order = np.lexsort((cols, -p16_row.astype(np.float32)))
    return order[:k]


def sample_tokens(logits: np.ndarray, temperature: float, table: np.ndarray, range_max: float,
                  uniforms: np.ndarray, top_k: int = TOP_K):
    """Restatement of ``sample_tokens`` (NumPy branch) with the random draws given.

    Greedy (temperature <= 0, :224-228): the first index of the largest logit; its
    log-probability ``log(max(p, fp16(1e-10)))`` evaluated on the fp16 probability and
    rounded to fp16, as NumPy does for an fp16 array.
    Temperature > 0 (:230-253): the fp16 LUT probabilities of the scaled logits; the
    ``min(top_k, V)`` largest (``top_candidates`` order) renormalised by their fp32
    sum; the token is the first candidate whose running fp32 sum exceeds
    ``u * total`` (``u`` in [0, 1), one per row; the reference draws it inside
    ``np.random.choice``), or the last one; a zero total picks candidate
    ``floor(u * k)``. Its log-probability is ``log(max(p, 1e-10))`` of the
    un-renormalised probability, in fp32.
    Returns (tokens int32 [N], logprobs float32 [N]).
    """
    x = np.asarray(logits)
    N, V = x.shape
    if temperature <= 0:
        tok = np.argmax(x, axis=-1)
        p16 = lut_probs16(x, table, range_max)
        pt = p16[np.arange(N), tok]
        lp = np.log(np.maximum(pt, np.float16(1e-10)).astype(np.float32)).astype(np.float16).astype(np.float32)
        return tok.astype(np.int32), lp
    p16 = lut_probs16(scaled_logits(x, temperature), table, range_max)
    k = min(top_k, V)
    toks = np.zeros(N, dtype=np.int32)
    lps = np.zeros(N, dtype=np.float32)
    for n in range(N):
        cand = top_candidates(p16[n], k)
        pk = p16[n, cand].astype(np.float32)
        run = np.cumsum(pk, dtype=np.float32)
        total = run[-1]
        u = np.float32(uniforms[n])
        if total > 0:
            hit = np.nonzero(run > u * total)[0]
            j = int(hit[0]) if hit.size else k - 1
        else:
            j = min(int(np.floor(u * np.float32(k))), k - 1)
        toks[n] = cand[j]
        lps[n] = np.log(max(np.float32(p16[n, cand[j]]), np.float32(1e-10)))
    return toks, lps


def splitmix64(z: np.ndarray) -> np.ndarray:
    """SplitMix64 finaliser (Steele, Lea and Flood 2014) on uint64 values."""
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniforms(seed: int, counter: int, n: int) -> np.ndarray:
    """The kernel's per-row uniform draws in [0, 1): the top 24 bits of
    splitmix64(splitmix64(seed ^ counter * 0xD1B54A32D192ED03) + row), scaled by 2^-24."""
    with np.errstate(over="ignore"):
        base = splitmix64(np.uint64(seed) ^ (np.uint64(counter) * np.uint64(0xD1B54A32D192ED03)))
        h = splitmix64(base + np.arange(n, dtype=np.uint64))
    return ((h >> np.uint64(40)).astype(np.float64) * 2.0 ** -24).astype(np.float32)


def make_logits(N: int, V: int, seed: int, scale: float = 3.0, dtype=np.float32) -> np.ndarray:
    """Seeded N(0, scale^2) logits (the sampler fixtures' inputs)."""
    return (np.random.default_rng(seed).standard_normal((N, V)) * scale).astype(dtype)
