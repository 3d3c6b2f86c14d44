"""Pin the NumPy oracle against golden vectors produced by the reference itself.

The vectors come from ``tests/golden/make_golden.py`` (which imports the
reference's ``dequant.py``, ``attention.py`` and the CPU GEMM of
``test_batched_speed.py``). Integer, byte and fp16-dequant results must match bit
for bit; the fp32 CPU GEMM to a tight tolerance (BLAS summation order may differ
between hosts).
"""

import hashlib

import numpy as np
import pytest

from oracle import int4 as O
from oracle import attention as OA

QCASES = ["randn1024", "uniform_pm2", "zeros", "const35", "alt_pm10", "tiny", "outlier", "x100", "fp32_02"]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", QCASES)
def test_quantizers_and_packing_bit_exact(golden, name):
    w = golden[f"qin_{name}"]
    q, s = O.quantize_engine(w)
    np.testing.assert_array_equal(q, golden[f"qeng_q_{name}"])
    np.testing.assert_array_equal(s.view(np.uint16), golden[f"qeng_s_{name}"].view(np.uint16))
    q2, s2 = O.quantize_toplevel(w)
    np.testing.assert_array_equal(q2, golden[f"qtop_q_{name}"])
    np.testing.assert_array_equal(s2.view(np.uint16), golden[f"qtop_s_{name}"].view(np.uint16))
    st = O.pack_superblocks(q, s)
    np.testing.assert_array_equal(st, golden[f"stream_{name}"])
    deq = O.unpack_superblock_weights(st)
    np.testing.assert_array_equal(deq.view(np.uint16), golden[f"deq_{name}"].view(np.uint16))
    np.testing.assert_array_equal(deq.view(np.uint16), golden[f"lutdeq_{name}"].view(np.uint16))
    q3, s3 = O.unpack_q(st)
    np.testing.assert_array_equal(q3, q)


def test_config1_stream_and_dequant_digests(golden, golden_meta):
    m = golden_meta["cfg1"]
    w = O.make_weights(m["K"], m["M"], m["seed"])
    q, s = O.quantize_engine(w.reshape(-1))
    assert sha(q) == m["q_sha256"]
    assert sha(s) == m["scales_sha256"]
    st = O.pack_superblocks(q, s)
    assert sha(st) == m["stream_sha256"]
    deq = O.unpack_superblock_weights(st)
    assert sha(deq) == m["deq_sha256"]
    qt, stt = O.quantize_toplevel(w)
    assert sha(qt) == m["toplevel_q_sha256"]
    assert sha(stt) == m["toplevel_scales_sha256"]
    assert int(np.sum(qt.reshape(-1) != q)) == m["toplevel_vs_engine_q_mismatches"]
    x = O.make_activations(m["N"], m["K"], m["seed"])
    y = O.gemm(x, deq.reshape(m["K"], m["M"]))
    np.testing.assert_allclose(y.astype(np.float32), golden["cfg1_gemm"].astype(np.float32), rtol=1e-3, atol=1e-3)
    # GEMM(N=8) == 8 sequential GEMVs, the reference's own criterion (test_batched_speed.py:55-70)
    np.testing.assert_allclose(golden["cfg1_gemm"].astype(np.float32), golden["cfg1_gemv"].astype(np.float32),
                               rtol=1e-2, atol=1e-2)


def test_odd_gemm_shapes(golden, golden_meta):
    for c in golden_meta["odd"]:
        K, M, N, sd = c["K"], c["M"], c["N"], c["seed"]
        st = O.quantize_pack_matrix(O.make_weights(K, M, sd))
        assert sha(st) == c["stream_sha256"]
        y = O.gemm(O.make_activations(N, K, sd), O.unpack_superblock_weights(st).reshape(K, M))
        np.testing.assert_allclose(y.astype(np.float32), golden[f"odd_{K}x{M}_n{N}_gemm"].astype(np.float32),
                                   rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("r", [10, 16])
def test_exp_table_and_lookup(golden, golden_meta, r):
    t = OA.exp_table(32768, float(r))
    assert sha(t) == golden_meta[f"exp_table_r{r}_sha256"]
    out = OA.lut_lookup(t, float(r), golden[f"lookup_in_r{r}"])
    np.testing.assert_array_equal(out.view(np.uint16), golden[f"lookup_out_r{r}"].view(np.uint16))


@pytest.mark.parametrize("name", ["s4x16", "s32x128", "s8x4096", "s3x7", "s2x1"])
def test_lut_softmax(golden, name):
    t = OA.exp_table(32768, 10.0)
    x = golden[f"sm_in_{name}"]
    np.testing.assert_array_equal(OA.safe_softmax_lut(x, t, 10.0).view(np.uint16),
                                  golden[f"sm_out_{name}"].view(np.uint16))
    np.testing.assert_array_equal(OA.reference_softmax(x).view(np.uint16),
                                  golden[f"smref_out_{name}"].view(np.uint16))


def test_attention_reduced_config4(golden, golden_meta):
    a = golden_meta["attn"]
    q, k, v = OA.make_attention_inputs(a["T"], a["H"], a["L"], a["d"], a["seed"])
    t = OA.exp_table(32768, a["range_max"])
    out = OA.decode_attention(q, k, v, t, a["range_max"])
    np.testing.assert_allclose(out.astype(np.float32), golden["attn_out"].astype(np.float32), rtol=1e-3, atol=1e-3)
    exact = OA.decode_attention(q, k, v, t, a["range_max"], exact=True)
    rel = np.linalg.norm(out.astype(np.float32) - exact.astype(np.float32)) / np.linalg.norm(exact.astype(np.float32))
    assert rel < 1e-2


def test_column_shard_preserves_weights():
    K, M = 64, 512
    st = O.quantize_pack_matrix(O.make_weights(K, M, 3))
    full = O.unpack_superblock_weights(st).reshape(K, M)
    for c0, c1 in [(0, 256), (256, 512), (128, 384), (32, 160)]:
        sh = O.column_shard(st, K, M, c0, c1)
        np.testing.assert_array_equal(O.unpack_superblock_weights(sh).reshape(K, c1 - c0).view(np.uint16),
                                      full[:, c0:c1].view(np.uint16))
