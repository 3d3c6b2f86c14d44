"""Generate ``tests/golden/sampling_vectors.npz`` by running the REFERENCE's sampler.

Run once, in a container where the reference tree is mounted read-only:

    python tests/golden/make_sampling_golden.py /path/to/reference

It imports ``antigravity-engine/src/batch_generator.py`` (``BatchedRolloutCoordinator
.sample_tokens``, NumPy branch) and ``antigravity-engine/src/attention.py``
(``ExponentialLUT``, ``safe_softmax_lut``) and records, on seeded logits from
``oracle.sampling.make_logits``:

* greedy tokens and log-probabilities (fp32 and fp16 logits, zero and huge logits);
* the fp16 LUT probabilities of the temperature-scaled logits (whole arrays for small
  vocabularies; for the 151936-column case the top-64 (probability, column) pairs of
  each row and a SHA-256 digest of the array), and which cases make the reference
  raise (fp16 quotients that overflow);
* the reference's own random draws under ``np.random.seed``: its chosen tokens and
  log-probabilities, and token counts over 20000 draws from one row, so the tests can
  check that a draw lies in the top-50 set, carries the right log-probability and that
  the draws follow the renormalised top-50 distribution.
Nothing at test or bench time reads the reference tree.
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.sampling import make_logits  # noqa: E402  (input generator only)

TEMPS = [1e-10, 1e-5, 0.01, 0.7, 1.0, 10.0, 100.0]


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def top64(p16: np.ndarray):
    cols = np.arange(p16.shape[1])
    out_p, out_i = [], []
    for row in p16:
        order = np.lexsort((cols, -row.astype(np.float32)))[:64]
        out_p.append(row[order])
        out_i.append(order)
    return np.stack(out_p), np.stack(out_i).astype(np.int32)


def main(ref_root: str) -> None:
    src = os.path.join(ref_root, "antigravity-engine/src")
    sys.path.insert(0, src)
    att = _load("attention", os.path.join(src, "attention.py"))
    bg = _load("ref_batch_generator", os.path.join(src, "batch_generator.py"))
    assert not bg.HAS_TORCH_MPS  # the NumPy branch
    arrays, meta = {}, {"generator": "tests/golden/make_sampling_golden.py", "numpy": np.__version__,
                        "temps": TEMPS, "cases": {}, "raises": []}
    coord = bg.BatchedRolloutCoordinator(n_channels=8, vocab_size=1000, hidden_dim=256)
    lut = coord.exp_lut
    assert lut.size == 32768 and lut.range_max == 10.0

    # 1. greedy
    greedy = {"g32": (8, 1000, 1, 3.0, np.float32), "g16": (4, 151936, 2, 3.0, np.float16),
              "gzero": (8, 1000, None, 0.0, np.float32), "ghuge": (8, 1000, 3, 1e8, np.float32)}
    for name, (N, V, seed, scale, dt) in greedy.items():
        x = np.zeros((N, V), dt) if seed is None else make_logits(N, V, seed, scale, dt)
        tok, lp = coord.sample_tokens(x, temperature=0.0)
        arrays[name + "_tok"] = np.asarray(tok, np.int32)
        arrays[name + "_lp"] = np.asarray(lp, np.float32)
        meta["cases"][name] = {"N": N, "V": V, "seed": seed, "scale": scale, "dtype": np.dtype(dt).name}

    # 2. LUT probabilities of scaled logits, and the reference's own draws
    for dt, tag in ((np.float32, "32"), (np.float16, "16")):
        x = make_logits(8, 1000, 10, 3.0, dt)
        for i, t in enumerate(TEMPS):
            scaled = x / max(t, 1e-5)
            if not np.all(np.isfinite(scaled)):  # fp16 overflow: the reference raises
                try:
                    coord.sample_tokens(x, temperature=t)
                    raise AssertionError("expected the reference to fail on non-finite scaled logits")
                except IndexError:
                    meta["raises"].append(f"{tag}_{i}")
                continue
            arrays[f"p{tag}_{i}"] = att.safe_softmax_lut(scaled, lut)
            np.random.seed(1000 + i)
            tok, lp = coord.sample_tokens(x, temperature=t)
            arrays[f"s{tag}_{i}_tok"] = np.asarray(tok, np.int32)
            arrays[f"s{tag}_{i}_lp"] = np.asarray(lp, np.float32)
    x = make_logits(4, 151936, 11, 3.0, np.float16)
    p = att.safe_softmax_lut(x / 0.7, lut)
    arrays["big_top_p"], arrays["big_top_i"] = top64(p)
    meta["big_sha"] = sha(p)
    np.random.seed(77)
    tok, lp = coord.sample_tokens(x, temperature=0.7)
    arrays["big_tok"], arrays["big_lp"] = np.asarray(tok, np.int32), np.asarray(lp, np.float32)

    # 3. distribution of the reference's draws: one row of 60 columns, 20000 draws
    row = make_logits(1, 60, 12, 1.0, np.float32)
    xs = np.repeat(row, 20000, axis=0)
    np.random.seed(5)
    tok, _ = coord.sample_tokens(xs, temperature=1.0)
    arrays["dist_counts"] = np.bincount(np.asarray(tok), minlength=60).astype(np.int64)

    np.savez_compressed(os.path.join(HERE, "sampling_vectors.npz"), **arrays)
    with open(os.path.join(HERE, "sampling_vectors.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/reference")
