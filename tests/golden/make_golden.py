"""Generate the golden vectors in ``tests/golden/`` by running the REFERENCE's own code.

Run once, in a container where the reference tree is mounted read-only:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference modules (``antigravity-engine/src/dequant.py``,
``antigravity-engine/src/attention.py``, ``src/dequant.py`` and the CPU GEMM of
``antigravity-engine/tests/test_batched_speed.py``) and records their outputs on
seeded inputs. Inputs are regenerated at test time from the same seeds with
``oracle.int4.make_weights`` / ``make_activations`` and
``oracle.attention.make_attention_inputs``, so only outputs (or SHA-256 digests of
large outputs) are stored. Nothing at test or bench time reads the reference tree.
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

from oracle import int4 as O  # noqa: E402  (input generators only)
from oracle import attention as OA  # noqa: E402


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def stream_from_dicts(sbs) -> np.ndarray:
    """The 144-byte wire form (Metal ``struct SuperBlock``) of the reference's dict list."""
    return np.concatenate([np.concatenate([sb["scales"].astype(np.float16).view(np.uint8),
                                           sb["packed_nibbles"].astype(np.uint8)]) for sb in sbs])


def main(ref_root: str) -> None:
    eng = _load("ref_engine_dequant", os.path.join(ref_root, "antigravity-engine/src/dequant.py"))
    top = _load("ref_top_dequant", os.path.join(ref_root, "src/dequant.py"))
    att = _load("ref_attention", os.path.join(ref_root, "antigravity-engine/src/attention.py"))
    sys.path.insert(0, os.path.join(ref_root, "antigravity-engine/src"))
    speed = _load("ref_speed", os.path.join(ref_root, "antigravity-engine/tests/test_batched_speed.py"))

    arrays: dict[str, np.ndarray] = {}
    meta: dict = {"generator": "tests/golden/make_golden.py", "numpy": np.__version__}

    # 1. Quantizer known answers (engine + top-level), small seeded and edge inputs.
    qcases = {
        "randn1024": np.random.default_rng(1).standard_normal(1024).astype(np.float16),
        "uniform_pm2": np.random.default_rng(2).uniform(-2, 2, 1024).astype(np.float16),
        "zeros": np.zeros(256, np.float16),
        "const35": np.full(256, 3.5, np.float16),
        "alt_pm10": np.tile(np.array([10.0, -10.0], np.float16), 128),
        "tiny": np.full(256, 1e-4, np.float16),
        "outlier": np.concatenate([np.array([1e4], np.float16), np.zeros(255, np.float16)]),
        "x100": (np.random.default_rng(3).standard_normal(1024) * 100).astype(np.float16),
        "fp32_02": np.random.default_rng(4).normal(0, 0.02, 4096).astype(np.float32),
    }
    for name, w in qcases.items():
        arrays[f"qin_{name}"] = w
        q, s = eng.quantize_weights_int4(w)
        arrays[f"qeng_q_{name}"], arrays[f"qeng_s_{name}"] = q, s
        q2, s2 = top.quantize_fp16_to_int4(w)
        arrays[f"qtop_q_{name}"], arrays[f"qtop_s_{name}"] = q2, s2
        stream = stream_from_dicts(eng.repack_to_superblocks(q, s))
        arrays[f"stream_{name}"] = stream
        arrays[f"deq_{name}"] = top.unpack_superblock_weights(stream, len(stream) // 144)
        arrays[f"lutdeq_{name}"] = eng.lut_dequantize(q, s)

    # 2. W[2048,2048] N(0,0.02) seed 1, X[8,2048] N(0,1).
    K, M, N, seed = 2048, 2048, 8, 1
    w = O.make_weights(K, M, seed)
    q, s = eng.quantize_weights_int4(w.reshape(-1))
    stream = stream_from_dicts(eng.repack_to_superblocks(q, s))
    deq = top.unpack_superblock_weights(stream, len(stream) // 144)
    lut = eng.lut_dequantize(q, s)
    arith = eng.arithmetic_dequantize(q, s)
    assert np.array_equal(deq, lut) and np.array_equal(lut, arith)
    x = O.make_activations(N, K, seed)
    wmat = deq.reshape(K, M)
    arrays["cfg1_gemm"] = speed.simulate_gemm(wmat, x)
    arrays["cfg1_gemv"] = np.vstack([speed.simulate_gemv(wmat, x[i]) for i in range(N)])
    q_top, s_top = top.quantize_fp16_to_int4(w)
    meta["cfg1"] = {"K": K, "M": M, "N": N, "seed": seed,
                    "stream_sha256": sha(stream), "q_sha256": sha(q), "scales_sha256": sha(s),
                    "deq_sha256": sha(deq),
                    "toplevel_q_sha256": sha(q_top), "toplevel_scales_sha256": sha(s_top),
                    "toplevel_vs_engine_q_mismatches": int(np.sum(q_top.reshape(-1) != q))}

    # 3. Odd GEMM shapes (M not a multiple of 256, or of 32).
    odd = [(64, 160, 3, 11), (96, 384, 5, 12), (256, 1376, 17, 13), (64, 100, 2, 14),
           (32, 2048, 1, 15), (512, 5504, 32, 16)]
    meta["odd"] = []
    for (k_, m_, n_, sd) in odd:
        w_ = O.make_weights(k_, m_, sd)
        q_, s_ = eng.quantize_weights_int4(w_.reshape(-1))
        st_ = stream_from_dicts(eng.repack_to_superblocks(q_, s_))
        d_ = top.unpack_superblock_weights(st_, len(st_) // 144).reshape(k_, m_)
        x_ = O.make_activations(n_, k_, sd)
        tag = f"odd_{k_}x{m_}_n{n_}"
        arrays[f"{tag}_gemm"] = speed.simulate_gemm(d_, x_)
        meta["odd"].append({"K": k_, "M": m_, "N": n_, "seed": sd, "stream_sha256": sha(st_)})

    # 4. Exp LUT tables, lookups and LUT softmax.
    for r in (10.0, 16.0):
        e = att.ExponentialLUT(range_max=r)
        meta[f"exp_table_r{int(r)}_sha256"] = sha(e.lut)
        xs = -np.random.default_rng(21).random(20000).astype(np.float32) * (r * 1.5)
        xs[:6] = [0.0, -0.0, -r, -r * 2, -1e-7, -1000.0]
        arrays[f"lookup_in_r{int(r)}"] = xs
        arrays[f"lookup_out_r{int(r)}"] = e.lookup(xs)
    e10 = att.ExponentialLUT()
    for name, (shape, sd, mul) in {"s4x16": ((4, 16), 42, 1.0), "s32x128": ((32, 128), 99, 1.0),
                                   "s8x4096": ((8, 4096), 5, 3.0), "s3x7": ((3, 7), 6, 20.0),
                                   "s2x1": ((2, 1), 7, 1.0)}.items():
        xin = (np.random.default_rng(sd).standard_normal(shape) * mul).astype(np.float16)
        arrays[f"sm_in_{name}"] = xin
        arrays[f"sm_out_{name}"] = att.safe_softmax_lut(xin, e10)
        arrays[f"smref_out_{name}"] = att.reference_softmax(xin)

    # 5. Reduced BASELINE config 4: LUT decode attention T=2, H=4, L=512, d=128, r=16.
    T, H, L, d, sd = 2, 4, 512, 128, 31
    qa, ka, va = OA.make_attention_inputs(T, H, L, d, sd)
    e16 = att.ExponentialLUT(range_max=16.0)
    scale = np.float32(1.0 / np.sqrt(d))
    scores = np.einsum("thd,thld->thl", qa.astype(np.float32), ka.astype(np.float32)) * scale
    probs = att.safe_softmax_lut(scores, e16)
    out = np.einsum("thl,thld->thd", probs.astype(np.float32), va.astype(np.float32)).astype(np.float16)
    arrays["attn_out"] = out
    arrays["attn_probs"] = probs
    meta["attn"] = {"T": T, "H": H, "L": L, "d": d, "seed": sd, "range_max": 16.0}

    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **arrays)
    with open(os.path.join(HERE, "reference_vectors.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/reference")
