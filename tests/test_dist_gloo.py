"""Multi-rank host logic of the column / head sharding on CPU: gloo ranks (world size
2 and 3) each compute their shard with the NumPy oracle and join through the same
``gather_columns`` / ``gather_heads`` the NCCL path uses. The joined result must equal
the unsharded oracle result bit for bit (a shard's columns are computed by the same
fp32 GEMM on bit-identical re-packed weights)."""

import os
import socket

import numpy as np
import pytest

from moat_b200.dist import column_bounds, head_bounds


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gemm_rank(rank, world, port, K, M, N, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from moat_b200.dist import ColumnShardedGemm
    from oracle import int4 as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        st = O.quantize_pack_matrix(O.make_weights(K, M, 12))
        x = O.make_activations(N, K, 3)
        bounds = column_bounds(M, world, K)
        c0, c1 = bounds[rank]
        shard = O.column_shard(st, K, M, c0, c1)

        def local(xx):
            w = O.unpack_superblock_weights(shard).reshape(K, c1 - c0)
            return torch.from_numpy(O.gemm(xx, w).astype(np.float32))

        layer = ColumnShardedGemm(st, K, M, rank, world, local_fn=local)
        q.put((rank, layer(x).numpy()))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _heads_rank(rank, world, port, T, H, L, d, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from moat_b200.dist import HeadShardedAttention
    from oracle import attention as OA

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        qq, k, v = OA.make_attention_inputs(T, H, L, d, 21)
        table = OA.exp_table(32768, 16.0)
        h0, h1 = head_bounds(H, world)[rank]

        def local(qs, ks, vs, lut, scale):
            return torch.from_numpy(OA.decode_attention(qs, ks, vs, lut, 16.0).astype(np.float32))

        attn = HeadShardedAttention(H, rank, world, local_fn=local)
        q.put((rank, attn(qq[:, h0:h1], k[:, h0:h1], v[:, h0:h1], table).numpy()))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _run(target, world, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, y = q.get(timeout=120)
            results[r] = y
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errors = {r: y for r, y in results.items() if isinstance(y, str)}
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return results


@pytest.mark.parametrize("world", [2, 3])
def test_column_sharded_gemm_gloo(world):
    K, M, N = 512, 1536, 4  # 48 groups: uneven split at world 3 is still group aligned
    res = _run(_gemm_rank, world, K, M, N)
    from oracle import int4 as O
    st = O.quantize_pack_matrix(O.make_weights(K, M, 12))
    ref = O.gemm(O.make_activations(N, K, 3), O.unpack_superblock_weights(st).reshape(K, M)).astype(np.float32)
    for r in range(world):
        assert res[r].shape == (N, M)
        np.testing.assert_array_equal(res[r], ref)


def test_head_sharded_attention_gloo():
    T, H, L, d = 2, 5, 256, 32  # 5 heads over 2 ranks: uneven split
    res = _run(_heads_rank, 2, T, H, L, d)
    from oracle import attention as OA
    qq, k, v = OA.make_attention_inputs(T, H, L, d, 21)
    ref = OA.decode_attention(qq, k, v, OA.exp_table(32768, 16.0), 16.0).astype(np.float32)
    for r in range(2):
        np.testing.assert_array_equal(res[r], ref)


def test_bounds_are_group_aligned_and_cover():
    for M, world in [(8192, 8), (5504, 8), (5504, 3), (2048, 2)]:
        b = column_bounds(M, world)
        assert b[0][0] == 0 and b[-1][1] == M
        assert all(c1 - c0 > 0 and c0 % 32 == 0 and c1 % 32 == 0 for c0, c1 in b)
        assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
        widths = [c1 - c0 for c0, c1 in b]
        assert max(widths) - min(widths) <= 32
    assert head_bounds(16, 8) == [(2 * i, 2 * i + 2) for i in range(8)]
    with pytest.raises(ValueError):
        column_bounds(100, 2)
    with pytest.raises(ValueError):
        head_bounds(2, 4)
