"""GPU parity of the tensor-parallel decode step and its exchanges.

* ``mb_argmax_key_f16`` / ``mb_argmax_keys_to_ids`` against the oracle's keys, bit for
  bit (NaN, ties across shards, signed zeros).
* A rank's weights are exact slices of the one-GPU decoder's weights: q/k/v columns and
  o_proj rows of its heads, gate/up columns and down rows of its FFN range, lm_head
  columns of its vocabulary range (whole groups, so identical codes and scales).
* The NVLink peer exchange on one GPU: with one rank it equals ``mb_add_rmsnorm`` and
  ``mb_argmax_f16`` bit for bit over several epochs, and so does the row-parallel GEMM
  whose epilogue stores its rows into the exchange buffers followed by the join over
  them; a peer that never delivers makes the bounded wait expire into the error word.
* Two ranks (needs 2 GPUs), joined by the NVLink peer exchange (fused into the GEMM or
  not) or by NCCL: eager and
  graph-captured TP steps against the one-GPU decoder fed the same token ids. Logits
  within 2e-2 (the row-parallel partial products are rounded to fp16 before they are
  summed, instead of one fp32 accumulation); the residual stream identical on both
  ranks; greedy ids equal wherever the one-GPU logits' top-2 gap exceeds that noise.
  And the exchange kernels directly against NumPy.
"""

import ctypes
import os
import socket

import numpy as np
import pytest

from oracle import int4 as O
from oracle import sampling as S

pytestmark = pytest.mark.gpu


def _st():
    import torch
    return torch.cuda.current_stream().cuda_stream


def test_argmax_keys_match_oracle(cuda):
    import torch
    from moat_b200._lib import lib
    L = lib()
    N, V, col0 = 5, 19072, 37 * 128
    g = torch.Generator(device=cuda)
    g.manual_seed(3)
    x = torch.randn((N, V), generator=g, device=cuda).half()
    x[1, 5] = x[1, 18000] = 9.0
    x[2, 77] = float("nan")
    x[3, :] = 0.0
    x[3, :9] = -0.0
    x[4, :] = float("-inf")
    keys = torch.zeros(N, dtype=torch.int64, device=cuda)
    ids = torch.zeros(N, dtype=torch.int32, device=cuda)
    assert L.mb_argmax_key_f16(x.data_ptr(), N, V, col0, keys.data_ptr(), _st()) == 0
    assert L.mb_argmax_keys_to_ids(keys.data_ptr(), N, ids.data_ptr(), _st()) == 0
    torch.cuda.synchronize()
    xn = x.cpu().numpy()
    np.testing.assert_array_equal(keys.cpu().numpy(), S.argmax_keys(xn, col0))
    assert ids.cpu().numpy().tolist() == (S.reference_argmax(xn) + col0).tolist()
    assert ids.cpu().numpy().tolist()[1:] == [col0 + 5, col0 + 77, col0, col0]


def _small_cfg():
    from moat_b200.decode import DecoderConfig
    return DecoderConfig(layers=2, hidden=512, heads=4, head_dim=128, ffn=1024, vocab=4096, max_len=64)


def _deq(sb, K, M):
    return O.unpack_superblock_weights(sb.cpu().numpy()).reshape(K, M)


def test_rank_weights_are_slices_of_one_gpu_weights(cuda):
    from moat_b200.decode import Int4Decoder, tp_shards
    cfg = _small_cfg()
    D, dh, F, V = cfg.hidden, cfg.head_dim, cfg.ffn, cfg.vocab
    one = Int4Decoder(cfg, 2, device=cuda, seed=11)
    for world in (2, 4):
        sh = tp_shards(cfg, world)
        for rank in range(world):
            tp = Int4Decoder(cfg, 2, device=cuda, seed=11, rank=rank, world=world)
            h0, h1 = tp.head_range
            f0, f1 = sh["ffn"][rank]
            v0, v1 = sh["vocab"][rank]
            Dl, Fl = (h1 - h0) * dh, f1 - f0
            for a, b in zip(one.layers, tp.layers):
                full = _deq(a["wqkv"], D, 3 * D)
                want = np.concatenate([full[:, j * D + h0 * dh:j * D + h1 * dh] for j in range(3)], axis=1)
                np.testing.assert_array_equal(_deq(b["wqkv"], D, 3 * Dl), want)
                np.testing.assert_array_equal(_deq(b["wo"], Dl, D), _deq(a["wo"], D, D)[h0 * dh:h1 * dh])
                full = _deq(a["wgu"], D, 2 * F)
                want = np.concatenate([full[:, f0:f1], full[:, F + f0:F + f1]], axis=1)
                np.testing.assert_array_equal(_deq(b["wgu"], D, 2 * Fl), want)
                np.testing.assert_array_equal(_deq(b["wd"], Fl, D), _deq(a["wd"], F, D)[f0:f1])
            np.testing.assert_array_equal(_deq(tp.lm_head, D, v1 - v0), _deq(one.lm_head, D, V)[:, v0:v1])
            assert np.array_equal(tp.embed.cpu().numpy(), one.embed.cpu().numpy())


# ---------------------------------------------------------------------------
# the NVLink peer exchange kernels on one GPU, called through the C ABI
# ---------------------------------------------------------------------------
def _exchange_buffers(cuda, n, rows, D):
    import torch
    from moat_b200._lib import lib
    nb = int(lib().mb_peer_buffer_bytes(rows, D))
    assert nb > 0
    return [torch.zeros(nb, dtype=torch.uint8, device=cuda) for _ in range(n)]


def _ptrs(bufs):
    return (ctypes.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])


def test_peer_exchange_one_rank_equals_local_kernels(cuda):
    """world = 1: the exchange joins one partial, so x and h equal mb_add_rmsnorm's and
    the ids mb_argmax_f16's bit for bit, over several epochs (both parities)."""
    import torch
    from moat_b200._lib import lib
    L = lib()
    N, D, V = 16, 2048, 5000
    g = torch.Generator(device=cuda)
    g.manual_seed(4)
    bufs = _exchange_buffers(cuda, 1, N, D)
    state = torch.zeros(128, dtype=torch.int32, device=cuda)  # 64 row epochs per exchange kind
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    x_a = torch.randn((N, D), generator=g, device=cuda)
    x_b = x_a.clone()
    w = 1.0 + 0.1 * torch.randn(D, generator=g, device=cuda)
    h_a = torch.empty((N, D), dtype=torch.float16, device=cuda)
    h_b = torch.empty_like(h_a)
    ids_a = torch.empty(N, dtype=torch.int32, device=cuda)
    ids_b = torch.empty_like(ids_a)
    for _ in range(5):
        y = torch.randn((N, D), generator=g, device=cuda).half()
        assert L.mb_peer_add_rmsnorm(_ptrs(bufs), 1, 0, N * D, 10**9, y.data_ptr(), x_a.data_ptr(), w.data_ptr(), N,
                                     D, 1e-6, h_a.data_ptr(), state.data_ptr(), err.data_ptr(), _st()) == 0
        assert L.mb_add_rmsnorm(x_b.data_ptr(), y.data_ptr(), w.data_ptr(), N, D, 1e-6, h_b.data_ptr(), _st()) == 0
        logits = torch.randn((N, V), generator=g, device=cuda).half()
        assert L.mb_peer_argmax(_ptrs(bufs), 1, 0, N * D, 10**9, logits.data_ptr(), N, V, 0, ids_a.data_ptr(),
                                state.data_ptr() + 256, err.data_ptr(), _st()) == 0
        assert L.mb_argmax_f16(logits.data_ptr(), N, V, ids_b.data_ptr(), _st()) == 0
        torch.cuda.synchronize()
        assert torch.equal(x_a, x_b) and torch.equal(h_a, h_b) and torch.equal(ids_a, ids_b)
    assert int(err.item()) == 0
    epochs = state.cpu().tolist()
    assert epochs[:N] == [5] * N and epochs[64:64 + N] == [5] * N and not any(epochs[N:64] + epochs[64 + N:])


@pytest.mark.parametrize("N", [16, 40])
def test_fused_gemm_join_one_rank_equals_local_kernels(cuda, N):
    """world = 1: the row-parallel GEMM whose epilogue stores its rows as exchange words
    (mb_int4_gemm_peer), then the join over the stored rows (mb_peer_sum_rmsnorm), give
    x and h bit for bit as mb_int4_gemm + mb_add_rmsnorm, over six epochs (both
    parities) alternating with the unfused peer join on the same epoch state. N = 40
    runs the GEMM as two launches (32 + 8 batch rows)."""
    import torch
    from moat_b200._lib import lib
    from moat_b200.dequant import quantize_to_superblocks
    L = lib()
    K, D = 1024, 2048
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    sb = quantize_to_superblocks((0.02 * torch.randn((K, D), generator=g, device=cuda)).reshape(-1))
    bufs = _exchange_buffers(cuda, 1, 64, D)
    slot = 64 * D
    state = torch.zeros(128, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    x_a = torch.randn((N, D), generator=g, device=cuda)
    x_b = x_a.clone()
    w = 1.0 + 0.1 * torch.randn(D, generator=g, device=cuda)
    h_a = torch.empty((N, D), dtype=torch.float16, device=cuda)
    h_b = torch.empty_like(h_a)
    y = torch.empty((N, D), dtype=torch.float16, device=cuda)
    for e in range(6):
        act = torch.randn((N, K), generator=g, device=cuda).half()
        assert L.mb_int4_gemm(act.data_ptr(), sb.data_ptr(), y.data_ptr(), N, K, D, err.data_ptr(), _st()) == 0
        if e % 2 == 0:
            assert L.mb_int4_gemm_peer(act.data_ptr(), sb.data_ptr(), N, K, D, _ptrs(bufs), 1, 0, slot,
                                       state.data_ptr(), err.data_ptr(), _st()) == 0
            assert L.mb_peer_sum_rmsnorm(_ptrs(bufs), 1, 0, slot, 10**9, x_a.data_ptr(), w.data_ptr(), N, D, 1e-6,
                                         h_a.data_ptr(), state.data_ptr(), err.data_ptr(), _st()) == 0
        else:
            assert L.mb_peer_add_rmsnorm(_ptrs(bufs), 1, 0, slot, 10**9, y.data_ptr(), x_a.data_ptr(),
                                         w.data_ptr(), N, D, 1e-6, h_a.data_ptr(), state.data_ptr(),
                                         err.data_ptr(), _st()) == 0
        assert L.mb_add_rmsnorm(x_b.data_ptr(), y.data_ptr(), w.data_ptr(), N, D, 1e-6, h_b.data_ptr(), _st()) == 0
        torch.cuda.synchronize()
        assert torch.equal(x_a, x_b) and torch.equal(h_a, h_b), e
    assert int(err.item()) == 0
    assert state.cpu().tolist()[:N] == [6] * N
    # off the fast plan (M % 128 != 0): refused before any launch
    assert L.mb_int4_gemm_peer(act.data_ptr(), sb.data_ptr(), N, 2048, 1000 // 8 * 8, _ptrs(bufs), 1, 0, slot,
                               state.data_ptr(), err.data_ptr(), _st()) == -6


def test_peer_wait_gives_up_with_error_bit(cuda):
    """A rank whose peer never delivers (a second buffer whose flags nothing sets):
    the bounded wait expires, the kernel sets MB_DEVERR_TIMEOUT and returns, and the
    context stays usable."""
    import time

    import torch
    from moat_b200._lib import lib
    L = lib()
    N, D = 2, 256
    bufs = _exchange_buffers(cuda, 2, N, D)
    state = torch.zeros(128, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    x = torch.zeros((N, D), device=cuda)
    w = torch.ones(D, device=cuda)
    h = torch.empty((N, D), dtype=torch.float16, device=cuda)
    y = torch.ones((N, D), dtype=torch.float16, device=cuda)
    t0 = time.perf_counter()
    assert L.mb_peer_add_rmsnorm(_ptrs(bufs), 2, 0, N * D, 20_000_000, y.data_ptr(), x.data_ptr(), w.data_ptr(), N,
                                 D, 1e-6, h.data_ptr(), state.data_ptr(), err.data_ptr(), _st()) == 0
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(err.item()) & 1
    assert float(torch.ones(1, device=cuda).sum()) == 1.0


# ---------------------------------------------------------------------------
# two ranks on two GPUs
# ---------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(target, world, *args, timeout=300):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, y = q.get(timeout=timeout)
            res[r] = y
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    errors = {r: y for r, y in res.items() if isinstance(y, str)}
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return res


def _needs_two_gpus():
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


def _tp_worker(rank, world, port, exchange, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from moat_b200.decode import Int4Decoder
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    tp = one = None
    try:
        cfg, N = _small_cfg(), 4
        tp = Int4Decoder(cfg, N, device=dev, seed=11, rank=rank, world=world,
                         exchange="nccl" if exchange == "nccl" else "peer", fused_join=exchange != "peer_unfused",
                         exchange_timeout_s=2.0)
        tp.fill_prompt_cache(20, seed=12)
        if rank == 0:
            one = Int4Decoder(cfg, N, device=dev, seed=11)
            one.fill_prompt_cache(20, seed=12)
        ids = torch.tensor([3, 1000, 4095, 17], dtype=torch.int32, device=dev)
        recs = []

        def record(nxt, ids_in):
            rec = {"ids": nxt.cpu().numpy().copy(), "logits": tp.logits.float().cpu().numpy(),
                   "x": tp.x.cpu().numpy(), "err": int(tp.err.item())}
            if one is not None:  # the one-GPU decoder on the same input ids
                rec["ref_ids"] = one.step(ids_in).cpu().numpy().copy()
                rec["ref_logits"] = one.logits.float().cpu().numpy()
                rec["ref_x"] = one.x.cpu().numpy()
            recs.append(rec)

        for _ in range(3):  # eager steps
            nxt = tp.step(ids)
            record(nxt, ids)
            ids = nxt.clone()
        tp.ids.copy_(ids)
        tp.capture()
        for _ in range(3):  # graph replays (length read on the device)
            ids_in = tp.ids.clone()
            nxt = tp.step_graphed()
            torch.cuda.synchronize()
            record(nxt, ids_in)
        q.put((rank, recs))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))
    finally:
        if tp is not None:
            tp.close()  # graph and exchange buffers go before the process group
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["peer", "peer_unfused", "nccl"])
def test_tp_decode_two_gpus_matches_one_gpu(exchange):
    _needs_two_gpus()
    res = _spawn(_tp_worker, 2, exchange)
    for s, (a, b) in enumerate(zip(res[0], res[1])):
        assert a["err"] == 0 and b["err"] == 0
        np.testing.assert_array_equal(a["ids"], b["ids"])      # every rank chose the same tokens
        np.testing.assert_array_equal(a["x"], b["x"])          # replicated residual stream
        logits = np.concatenate([a["logits"], b["logits"]], axis=1)
        ref = a["ref_logits"]
        np.testing.assert_allclose(logits, ref, rtol=2e-2, atol=2e-2, err_msg=f"step {s}")
        np.testing.assert_allclose(a["x"], a["ref_x"], rtol=2e-2, atol=2e-2)
        top2 = np.sort(ref, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 4e-2
        assert np.array_equal(a["ids"][clear], a["ref_ids"][clear]), (s, a["ids"], a["ref_ids"])


def _exchange_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from moat_b200.peer import PeerExchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    px = None
    try:
        N, D, V = 16, 2048, 3000
        px = PeerExchange(N, D, dev, timeout_s=2.0)
        rng = np.random.default_rng(100)
        x0 = rng.standard_normal((N, D)).astype(np.float32)
        w = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        x = torch.from_numpy(x0).to(dev)
        wt = torch.from_numpy(w).to(dev)
        h = torch.empty((N, D), dtype=torch.float16, device=dev)
        ids = torch.empty(N, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        out = []
        for step in range(4):
            parts = [np.random.default_rng(1000 * step + r).standard_normal((N, D)).astype(np.float16)
                     for r in range(world)]
            px.add_rmsnorm(torch.from_numpy(parts[rank]).to(dev), x, wt, 1e-6, h, err)
            logits = np.random.default_rng(77 + step).standard_normal((N, world * V)).astype(np.float16)
            logits[step, 5] = logits[step, V + 5] = 9.0  # tie across the two ranks' ranges
            px.argmax(torch.from_numpy(np.ascontiguousarray(logits[:, rank * V:(rank + 1) * V])).to(dev), rank * V,
                      ids, err)
            torch.cuda.synchronize()
            out.append({"x": x.cpu().numpy(), "h": h.float().cpu().numpy(), "ids": ids.cpu().numpy().copy(),
                        "parts": parts, "logits": logits})
        q.put((rank, {"steps": out, "x0": x0, "w": w, "err": int(err.item())}))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        if px is not None:
            px.close()
        dist.destroy_process_group()


def test_peer_exchange_two_gpus_matches_numpy():
    """Two ranks: x += fp16(P_0 + P_1 summed in fp32) bit for bit against NumPy on both
    ranks; h = RMSNorm(x) * w within fp16 rounding; ids = numpy.argmax of the joined
    logits (ties across the ranks' ranges to the first column)."""
    _needs_two_gpus()
    res = _spawn(_exchange_worker, 2)
    x = res[0]["x0"].copy()
    w = res[0]["w"]
    for s in range(4):
        a, b = res[0]["steps"][s], res[1]["steps"][s]
        d = (a["parts"][0].astype(np.float32) + a["parts"][1].astype(np.float32)).astype(np.float16)
        x = x + d.astype(np.float32)
        np.testing.assert_array_equal(a["x"], x)
        np.testing.assert_array_equal(b["x"], x)
        np.testing.assert_array_equal(a["h"], b["h"])
        ref_h = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * w
        np.testing.assert_allclose(a["h"], ref_h.astype(np.float16).astype(np.float32), rtol=2e-3, atol=2e-3)
        ref_ids = S.reference_argmax(a["logits"])
        assert a["ids"].tolist() == ref_ids.tolist() == b["ids"].tolist()
        assert ref_ids[s] == 5
    assert res[0]["err"] == 0 and res[1]["err"] == 0


def _fused_join_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from moat_b200.dequant import quantize_to_superblocks
    from moat_b200.gemm import batched_gemm
    from moat_b200.peer import PeerExchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    px = None
    try:
        N, K, D = 16, 1024, 2048
        px = PeerExchange(N, D, dev, timeout_s=2.0)
        rng = np.random.default_rng(200 + rank)
        sb = quantize_to_superblocks(torch.from_numpy((0.02 * rng.standard_normal(K * D)).astype(np.float32)).to(dev))
        x0 = np.random.default_rng(300).standard_normal((N, D)).astype(np.float32)
        w = torch.ones(D, device=dev)
        x = torch.from_numpy(x0).to(dev)
        h = torch.empty((N, D), dtype=torch.float16, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        out = []
        for step in range(4):
            act = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float16)).to(dev)
            y = batched_gemm(act, sb, K, D)  # this rank's partial, unfused, for the check
            if step % 2 == 0:
                assert px.gemm(act, sb, K, D, err)
                px.sum_rmsnorm(x, w, 1e-6, h, err)
            else:
                px.add_rmsnorm(y, x, w, 1e-6, h, err)
            torch.cuda.synchronize()
            out.append({"x": x.cpu().numpy(), "h": h.float().cpu().numpy(), "y": y.cpu().numpy()})
        q.put((rank, {"steps": out, "x0": x0, "err": int(err.item())}))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        if px is not None:
            px.close()
        dist.destroy_process_group()


def test_fused_gemm_join_two_gpus_matches_numpy():
    """Two ranks, alternating the fused row-parallel GEMM + join (epochs 1, 3) with the
    unfused peer join (2, 4): x += fp16(Y_0 + Y_1 summed in fp32), with Y_r rank r's
    own mb_int4_gemm partial, bit for bit on both ranks; identical h on both ranks."""
    _needs_two_gpus()
    res = _spawn(_fused_join_worker, 2)
    x = res[0]["x0"].copy()
    for s in range(4):
        a, b = res[0]["steps"][s], res[1]["steps"][s]
        d = (a["y"].astype(np.float32) + b["y"].astype(np.float32)).astype(np.float16)
        x = x + d.astype(np.float32)
        np.testing.assert_array_equal(a["x"], x, err_msg=f"step {s}")
        np.testing.assert_array_equal(b["x"], x, err_msg=f"step {s}")
        np.testing.assert_array_equal(a["h"], b["h"])
    assert res[0]["err"] == 0 and res[1]["err"] == 0


def _tp_sample_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from moat_b200.decode import Int4Decoder
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    tp = None
    try:
        tp = Int4Decoder(_small_cfg(), 4, device=dev, seed=11, rank=rank, world=world, exchange_timeout_s=2.0,
                         temperature=0.8, sample_seed=5)
        tp.fill_prompt_cache(20, seed=12)
        tp.ids.copy_(torch.tensor([3, 1000, 4095, 17], dtype=torch.int32, device=dev))
        recs = []
        for c in range(3):  # an eager step, then graph replays
            if c == 0:
                tp.step(tp.ids)
            else:
                if c == 1:
                    tp.capture()
                tp.step_graphed()
            torch.cuda.synchronize()
            recs.append({"ids": tp.ids.cpu().numpy().copy(), "lp": tp.logprobs.cpu().numpy().copy(),
                         "logits": tp.logits_full.float().cpu().numpy(), "err": int(tp.err.item())})
        q.put((rank, recs))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        if tp is not None:
            tp.close()
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_tp_sampled_decode_two_gpus():
    """Temperature sampling with the vocabulary split over two ranks: both ranks gather
    the same logits and draw the same token, the oracle's draw from those logits with
    the device stream's uniforms (counter = step)."""
    _needs_two_gpus()
    from oracle import attention as OA
    res = _spawn(_tp_sample_worker, 2)
    table = OA.exp_table(32768, 10.0)
    for c, (a, b) in enumerate(zip(res[0], res[1])):
        assert a["err"] == 0 and b["err"] == 0
        np.testing.assert_array_equal(a["logits"], b["logits"])
        np.testing.assert_array_equal(a["ids"], b["ids"])
        otok, olp = S.sample_tokens(a["logits"].astype(np.float16), 0.8, table, 10.0, S.uniforms(5, c, 4))
        np.testing.assert_array_equal(a["ids"], otok)
        np.testing.assert_allclose(a["lp"], olp, rtol=1e-6, atol=1e-6)
