"""GPU parity of quantize / pack / unpack / dequant against the reference's golden
vectors and the NumPy oracle. Integer and byte results: bit-exact."""

import hashlib

import numpy as np
import pytest

from oracle import int4 as O

pytestmark = pytest.mark.gpu

QCASES = ["randn1024", "uniform_pm2", "zeros", "const35", "alt_pm10", "tiny", "outlier", "x100", "fp32_02"]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", QCASES)
def test_quantizers_match_reference(cuda, golden, name):
    from moat_b200 import dequant as D
    w = golden[f"qin_{name}"]
    q, s = D.quantize_weights_int4(w)
    np.testing.assert_array_equal(q, golden[f"qeng_q_{name}"])
    np.testing.assert_array_equal(s.view(np.uint16), golden[f"qeng_s_{name}"].view(np.uint16))
    q2, s2 = D.quantize_fp16_to_int4(w)
    np.testing.assert_array_equal(q2, golden[f"qtop_q_{name}"])
    np.testing.assert_array_equal(s2.view(np.uint16), golden[f"qtop_s_{name}"].view(np.uint16))
    st = D.pack_superblocks(q, s)
    np.testing.assert_array_equal(st, golden[f"stream_{name}"])
    np.testing.assert_array_equal(D.quantize_to_superblocks(w), golden[f"stream_{name}"])
    deq = D.unpack_superblock_weights(st, len(st) // 144)
    np.testing.assert_array_equal(deq.view(np.uint16), golden[f"deq_{name}"].view(np.uint16))
    np.testing.assert_array_equal(D.lut_dequantize(q, s).view(np.uint16), golden[f"lutdeq_{name}"].view(np.uint16))
    np.testing.assert_array_equal(D.arithmetic_dequantize(q, s).view(np.uint16),
                                  golden[f"lutdeq_{name}"].view(np.uint16))
    q3, s3 = D.unpack_superblocks(st)
    np.testing.assert_array_equal(q3, q)
    np.testing.assert_array_equal(s3.view(np.uint16), s.view(np.uint16))


def test_config1_digests_on_gpu(cuda, golden_meta):
    """BASELINE config 1 (2048x2048, N(0,0.02), seed 1): packed stream and dequant
    digests equal the ones the reference produced."""
    import torch
    from moat_b200 import dequant as D
    m = golden_meta["cfg1"]
    w = O.make_weights(m["K"], m["M"], m["seed"])
    wd = torch.from_numpy(w.reshape(-1)).cuda()
    q, s = D.quantize_weights_int4(wd)
    assert sha(q.cpu().numpy()) == m["q_sha256"]
    assert sha(s.cpu().numpy()) == m["scales_sha256"]
    st = D.quantize_to_superblocks(wd)
    assert sha(st.cpu().numpy()) == m["stream_sha256"]
    deq = D.unpack_superblock_weights(st, st.numel() // 144)
    assert sha(deq.cpu().numpy()) == m["deq_sha256"]
    qt, stt = D.quantize_fp16_to_int4(torch.from_numpy(w).cuda())
    assert sha(qt.cpu().numpy()) == m["toplevel_q_sha256"]


def test_reference_api_shapes_and_errors(cuda):
    from moat_b200 import dequant as D
    from moat_b200 import engine_dequant as E
    with pytest.raises(ValueError):
        D.quantize_weights_int4(np.zeros(33, np.float16))
    with pytest.raises(ValueError):
        D.quantize_weights_int4(np.zeros((4, 32), np.float16))
    with pytest.raises(ValueError):
        D.repack_to_superblocks(np.zeros(200, np.int8), np.ones(7, np.float16))
    with pytest.raises(AssertionError):
        D.repack_weights_to_superblock(np.zeros(200, np.int8))
    q = np.random.default_rng(0).integers(-8, 8, 512, dtype=np.int8)
    s = np.random.default_rng(1).random(16).astype(np.float16)
    sbs = D.repack_to_superblocks(q, s)
    assert len(sbs) == 2 and sbs[0]["packed_nibbles"].dtype == np.uint8 and len(sbs[0]["packed_nibbles"]) == 128
    for i, sb in enumerate(sbs):
        np.testing.assert_array_equal(D.unpack_superblock(sb), q[i * 256:(i + 1) * 256])
        np.testing.assert_array_equal(sb["scales"].view(np.uint16), s[i * 8:(i + 1) * 8].view(np.uint16))
    np.testing.assert_array_equal(D.superblocks_to_stream(sbs), O.pack_superblocks(q, s))
    r = D.repack_weights_to_superblock(q)
    assert r.shape == (2, 8, 32) and r.ctypes.data % 128 == 0
    assert E.quantize_fp16_to_int4 is E.quantize_weights_int4
    # lut_dequantize_fp16 index rule (src/dequant.py:86-94; tests/test_quantization.py:100-112)
    lut = np.arange(10, 26, dtype=np.float16)
    np.testing.assert_array_equal(D.lut_dequantize_fp16(np.array([-8, -7, 0, 7], np.int8), lut),
                                  np.array([10, 11, 18, 25], np.float16))
    np.testing.assert_array_equal(D.lut_dequantize_fp16(np.array([-10, 20, 5, 0], np.int32), lut),
                                  lut[np.clip(np.array([-2, 28, 13, 8]), 0, 15)])
    # 2-D per-group LUT
    w = np.random.default_rng(2).uniform(-1, 1, 256).astype(np.float16)
    qq, ss = D.quantize_fp16_to_int4(w)
    lut2 = ss.astype(np.float32)[:, None] * np.arange(-8, 8, dtype=np.float32)[None, :]
    got = D.lut_dequantize_fp16(qq.reshape(8, 32), lut2)
    np.testing.assert_array_equal(got.reshape(-1).view(np.uint16), O.dequant(qq, ss).view(np.uint16))


def test_large_stream_dequant_bit_exact(cuda):
    """25 M weights (3072x8192): GPU dequant == oracle bit for bit."""
    import torch
    from moat_b200 import dequant as D
    K, M = 3072, 8192
    w = O.make_weights(K, M, 3)
    st = O.quantize_pack_matrix(w)
    ref = O.unpack_superblock_weights(st)
    got = D.unpack_superblock_weights(torch.from_numpy(st).cuda(), st.size // 144).cpu().numpy()
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    st_gpu = D.quantize_to_superblocks(torch.from_numpy(w.reshape(-1)).cuda()).cpu().numpy()
    assert np.array_equal(st_gpu, st)


def test_extract_columns_bit_exact(cuda):
    import torch
    from moat_b200 import dequant as D
    K, M = 96, 1024
    st = O.quantize_pack_matrix(O.make_weights(K, M, 4))
    d = torch.from_numpy(st).cuda()
    for c0, c1 in [(0, 512), (512, 1024), (32, 288), (96, 736)]:
        got = D.extract_columns(d, K, M, c0, c1).cpu().numpy()
        np.testing.assert_array_equal(got, O.column_shard(st, K, M, c0, c1))


def test_empty_inputs(cuda):
    from moat_b200 import dequant as D
    q, s = D.quantize_weights_int4(np.zeros(0, np.float16))
    assert q.size == 0 and s.size == 0
    assert D.unpack_superblock_weights(np.zeros(0, np.uint8), 0).size == 0


def test_nan_inf_groups_follow_reference(cuda):
    from moat_b200 import dequant as D
    w = np.zeros(64, np.float16)
    w[0] = np.inf
    w[33] = np.nan
    w[40] = 1.0
    q, s = D.quantize_weights_int4(w)
    assert np.all(q == 0)
    assert np.isinf(s[0]) and np.isnan(s[1])
