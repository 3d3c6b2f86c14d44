"""Two ranks on two GPUs (skipped with fewer): the column-sharded config-3 GEMM joined by
an NCCL all-gather and the head-sharded config-4 LUT attention joined the same way,
each against the CPU oracle of the reference's path on the whole unsharded problem.

* GEMM: every rank keeps its group-aligned column range of the packed weight (re-packed
  bit-identically), multiplies it with the local kernel and ``gather_columns`` joins the
  shards; N = 1 and 32 against the oracle's fp32 GEMM of the dequantized weight (the
  north-star bar 1e-2 relative, and relative L2 <= 1e-3).
* Attention: every rank runs the heads ``head_bounds`` gives it and ``gather_heads``
  joins the outputs; all 256 (trace, head) rows against the oracle's composition
  (einsum scores, exp-LUT softmax, einsum with V).
"""

import os
import socket

import numpy as np
import pytest

from oracle import attention as OA
from oracle import int4 as O

pytestmark = pytest.mark.gpu

K3, M3 = 3072, 8192


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _needs_two_gpus():
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from moat_b200.attention import ExponentialLUT
    from moat_b200.dist import ColumnShardedGemm, HeadShardedAttention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        out = {}
        st = torch.from_numpy(O.quantize_pack_matrix(O.make_weights(K3, M3, 41))).to(dev)
        sharded = ColumnShardedGemm(st, K3, M3, rank, world)
        for n in (1, 32):
            x = torch.from_numpy(O.make_activations(n, K3, 50 + n)).to(dev)
            out[f"gemm{n}"] = sharded(x).float().cpu().numpy()
        T, H, L, d = 16, 16, 4096, 128
        qn, kn, vn = OA.make_attention_inputs(T, H, L, d, 43)
        att = HeadShardedAttention(H, rank, world)
        h0, h1 = att.h0, att.h1
        loc = [torch.from_numpy(np.ascontiguousarray(a[:, h0:h1])).to(dev) for a in (qn, kn, vn)]
        out["attn"] = att(*loc, ExponentialLUT(range_max=16.0)).float().cpu().numpy()
        out["bounds"] = (sharded.bounds, att.bounds)
        torch.cuda.synchronize()
        q.put((rank, out))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_gemm_and_attention_match_oracle():
    _needs_two_gpus()
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, y = q.get(timeout=300)
            res[r] = y
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    errors = {r: y for r, y in res.items() if isinstance(y, str)}
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    w = O.unpack_superblock_weights(O.quantize_pack_matrix(O.make_weights(K3, M3, 41))).reshape(K3, M3)
    for n in (1, 32):
        ref = O.gemm(O.make_activations(n, K3, 50 + n), w).astype(np.float32)
        for r in range(world):  # every rank holds the whole joined product
            got = res[r][f"gemm{n}"]
            np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2)
            assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-3
    qn, kn, vn = OA.make_attention_inputs(16, 16, 4096, 128, 43)
    ref = OA.decode_attention(qn, kn, vn, OA.exp_table(32768, 16.0), 16.0).astype(np.float32)
    for r in range(world):
        got = res[r]["attn"]
        np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2)
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-3
    assert res[0]["bounds"][0] == [(0, 4096), (4096, 8192)] and res[0]["bounds"][1] == [(0, 8), (8, 16)]
