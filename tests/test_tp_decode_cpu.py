"""Host logic of the tensor-parallel decode step, on CPU.

* The distributed greedy choice: per-shard 64-bit keys (oracle restatement of the
  kernel's encoding) combined by an integer maximum give numpy.argmax of the whole row
  (the reference's greedy choice, batch_generator.py:224-227), NaN, ties and signed
  zeros included; and the same combine as a gloo all-reduce over two ranks.
* The Megatron split of config 5 over 1/2/4/8 ranks: head, FFN and vocabulary ranges
  cover their dimension, are whole 128-column units, and give every rank's GEMMs
  widths the fast kernel plan takes.
* The LM head's zero-column padding (to whole 256-column strips) leaves the INT4 codes
  and scales of the real columns bit for bit as they were (oracle quantizer).
"""

import os
import socket

import numpy as np
import pytest

from oracle import sampling as S


def _shard_keys(x, bounds):
    keys = [S.argmax_keys(x[:, c0:c1], c0) for c0, c1 in bounds]
    return S.keys_to_ids(np.maximum.reduce(keys))


def test_keys_match_numpy_argmax_over_any_split():
    rng = np.random.default_rng(0)
    N, V = 8, 1000
    x = rng.standard_normal((N, V)).astype(np.float16)
    x[1, 10] = x[1, 900] = 9.0                  # tie across shards: first column
    x[2, 500] = np.float16("nan")               # NaN is the largest
    x[2, 700] = np.float16("nan")
    x[3, :] = -2.0                              # all equal
    x[4, :] = 0.0
    x[4, :5] = np.float16(-0.0)                 # -0 == +0: column 0
    x[5, 3] = np.float16("inf")
    x[6, :] = np.float16("-inf")
    x[7, 999] = 50.0                            # last column
    ref = S.reference_argmax(x)
    assert ref[1] == 10 and ref[2] == 500 and ref[3] == 0 and ref[4] == 0 and ref[6] == 0 and ref[7] == 999
    for bounds in ([(0, V)], [(0, 500), (500, V)], [(0, 96), (96, 512), (512, 992), (992, V)]):
        np.testing.assert_array_equal(_shard_keys(x, bounds), ref)


def test_code_is_order_preserving():
    v = np.array([-np.inf, -65504, -1.5, -1e-7, -0.0, 0.0, 1e-7, 1.5, 65504, np.inf], dtype=np.float16)
    c = S.argmax_code(v.view(np.uint16))
    assert np.all(np.diff(c.astype(np.int64)[[0, 1, 2, 3, 4, 6, 7, 8, 9]]) > 0)
    assert c[4] == c[5]
    assert S.argmax_code(np.array([0x7E00, 0xFE01], dtype=np.uint16)).tolist() == [0xFFFF, 0xFFFF]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _keys_input():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((6, 640)).astype(np.float16)
    x[0, 100] = x[0, 600] = 7.0
    x[1, 639] = np.float16("nan")
    return x


def _keys_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        x = _keys_input()
        c0, c1 = [(0, 384), (384, 640)][rank]
        keys = torch.from_numpy(S.argmax_keys(x[:, c0:c1], c0))
        dist.all_reduce(keys, op=dist.ReduceOp.MAX)
        q.put((rank, S.keys_to_ids(keys.numpy()).tolist()))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_key_all_reduce_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_keys_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=120) for _ in range(2))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    ref = S.reference_argmax(_keys_input()).tolist()
    assert res[0] == ref and res[1] == ref, res
    assert ref[0] == 100 and ref[1] == 639


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config5_split(world):
    from moat_b200.decode import DecoderConfig, tp_shards
    cfg = DecoderConfig()
    sh = tp_shards(cfg, world)
    for name, total in (("heads", cfg.heads), ("ffn", cfg.ffn), ("vocab", cfg.vocab)):
        b = sh[name]
        assert len(b) == world and b[0][0] == 0 and b[-1][1] == total
        assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
        if name != "heads" and world > 1:
            assert all(c0 % 128 == 0 and (c1 - c0) % 128 == 0 for c0, c1 in b)
    if world == 8:
        assert [c1 - c0 for c0, c1 in sh["ffn"]] == [768] * 3 + [640] * 5
        assert sh["heads"] == [(2 * r, 2 * r + 2) for r in range(8)]
    # every rank's GEMM shapes: K a multiple of 8, M a multiple of 128 (fast plan)
    D, dh = cfg.hidden, cfg.head_dim
    for r in range(world):
        Hl = sh["heads"][r][1] - sh["heads"][r][0]
        Fl = sh["ffn"][r][1] - sh["ffn"][r][0]
        Vl = sh["vocab"][r][1] - sh["vocab"][r][0]
        for K, M in ((D, 3 * Hl * dh), (Hl * dh, D), (D, 2 * Fl), (Fl, D), (D, Vl)):
            assert K % 8 == 0 and M % 128 == 0 and (K * M) % 256 == 0, (r, K, M)


def test_small_vocab_split_falls_back_to_groups():
    from moat_b200.decode import DecoderConfig, tp_shards
    sh = tp_shards(DecoderConfig(vocab=1056, ffn=512), 2)
    assert sh["vocab"] == [(0, 544), (544, 1056)]
    assert sh["ffn"] == [(0, 256), (256, 512)]


def test_lm_head_padding_keeps_codes_and_scales():
    from moat_b200.decode import DecoderConfig, lm_head_cols, tp_shards
    from oracle import int4 as O
    cfg = DecoderConfig()
    for world in (1, 2, 4, 8):
        for c0, c1 in tp_shards(cfg, world)["vocab"]:
            cols = lm_head_cols(c1 - c0)
            assert cols % 256 == 0 or (c1 - c0) % 256 != 128
            assert cols - (c1 - c0) in (0, 128)
    assert lm_head_cols(151936) == 152064 and lm_head_cols(76032) == 76032 and lm_head_cols(1000) == 1000
    K, V = 64, 1152  # 9 x 128 columns -> 1280
    w = O.make_weights(K, V, 31)
    Vp = lm_head_cols(V)
    wp = np.concatenate([w, np.zeros((K, Vp - V), np.float32)], axis=1)
    plain = O.unpack_superblock_weights(O.quantize_pack_matrix(w)).reshape(K, V)
    padded = O.unpack_superblock_weights(O.quantize_pack_matrix(wp)).reshape(K, Vp)
    np.testing.assert_array_equal(padded[:, :V].view(np.uint16), plain.view(np.uint16))
    assert not np.any(padded[:, V:])
