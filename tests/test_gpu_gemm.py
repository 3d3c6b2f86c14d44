"""GPU parity of the fused INT4 batched GEMM against the reference's CPU GEMM
(golden vectors) and the NumPy oracle.

Tolerance: the north-star bar, 1e-2 relative with fp32 accumulation
(``rtol = atol = 1e-2`` as in antigravity-engine/tests/test_batched_speed.py:66-70),
and a relative L2 error of at most 1e-3 over the whole output. The kernel sums
``q * fp16(x * s)`` in fp32 (the group scale is applied to the activations, one fp16
rounding per product) where the reference sums ``x * fp16(q * s)``: both carry one
fp16 rounding per product, so results agree to about 3e-4 relative L2, not bit for
bit. Dequantization itself is bit-exact and tested as such (test_gpu_int4.py).
"""

import numpy as np
import pytest

from oracle import int4 as O

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2


def close(got, ref):
    g, r = got.astype(np.float32), ref.astype(np.float32)
    np.testing.assert_allclose(g, r, rtol=RTOL, atol=ATOL)
    rel = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    assert rel <= 1e-3, f"relative L2 error {rel:.3e}"


def run(x, st, K, M):
    import torch
    from moat_b200.gemm import batched_gemm
    return batched_gemm(torch.from_numpy(x).cuda(), torch.from_numpy(st).cuda(), K, M).cpu().numpy()


def test_config1_against_reference_golden(cuda, golden, golden_meta):
    m = golden_meta["cfg1"]
    K, M, N = m["K"], m["M"], m["N"]
    st = O.quantize_pack_matrix(O.make_weights(K, M, m["seed"]))
    x = O.make_activations(N, K, m["seed"])
    got = run(x, st, K, M)
    close(got, golden["cfg1_gemm"])
    # GEMM(N=8) vs 8 sequential GEMVs through the same kernel (test_batched_speed.py:55-70)
    gemv = np.vstack([run(x[i:i + 1], st, K, M) for i in range(N)])
    np.testing.assert_allclose(got.astype(np.float32), gemv.astype(np.float32), rtol=RTOL, atol=ATOL)
    close(gemv, golden["cfg1_gemv"])


def test_odd_shapes_against_reference_golden(cuda, golden, golden_meta):
    for c in golden_meta["odd"]:
        K, M, N, sd = c["K"], c["M"], c["N"], c["seed"]
        st = O.quantize_pack_matrix(O.make_weights(K, M, sd))
        got = run(O.make_activations(N, K, sd), st, K, M)
        close(got, golden[f"odd_{K}x{M}_n{N}_gemm"])


@pytest.mark.parametrize("K,M", [(2048, 5504), (3072, 8192)])
@pytest.mark.parametrize("N", [1, 2, 4, 8, 16, 32])
def test_baseline_configs_n_sweep(cuda, K, M, N):
    """BASELINE configs 2 and 3 at every N of the sweep, against the oracle."""
    st = O.quantize_pack_matrix(O.make_weights(K, M, 100 + K))
    w = O.unpack_superblock_weights(st).reshape(K, M)
    x = O.make_activations(N, K, N)
    close(run(x, st, K, M), O.gemm(x, w))


@pytest.mark.parametrize("N,K,M", [(3, 16, 256), (5, 40, 512), (1, 8, 256), (7, 1000, 768), (33, 256, 512),
                                   (70, 64, 256), (12, 4104, 256), (9, 24, 4096)])
def test_ragged_shapes(cuda, N, K, M):
    """K not a multiple of the 16-row slice or 64-row stage, N not a multiple of 8, N > 32."""
    st = O.quantize_pack_matrix(O.make_weights(K, M, N * 7 + K))
    w = O.unpack_superblock_weights(st).reshape(K, M)
    x = O.make_activations(N, K, K)
    close(run(x, st, K, M), O.gemm(x, w))


_WIDE = {}


def _wide(K, M):
    if (K, M) not in _WIDE:
        st = O.quantize_pack_matrix(O.make_weights(K, M, 7 + K))
        _WIDE[(K, M)] = (st, O.unpack_superblock_weights(st).reshape(K, M))
    return _WIDE[(K, M)]


@pytest.mark.parametrize("K,M", [(256, 151936), (512, 76032), (520, 75904)])
@pytest.mark.parametrize("N", [1, 16, 32])
def test_many_strips_without_k_split(cuda, N, K, M):
    """More strips than the GPU holds CTAs at once, and no K split: the config-5 LM head
    (1187 strips of 128 columns) and its two tensor-parallel shards (594 and 593 strips
    of 128) run in several waves of one CTA per strip; K = 520 ends every strip with a
    one-slice stage. Against the oracle."""
    from moat_b200.gemm import plan
    pl = plan(N, K, M)
    assert pl["kind"] == 1 and pl["cluster"] == 1 and pl["grid"] > 148, pl
    st, w = _wide(K, M)
    x = O.make_activations(N, K, K + N)
    close(run(x, st, K, M), O.gemm(x, w))


@pytest.mark.parametrize("N", [32, 40])
def test_rows_in_blocks_of_16_where_32_do_not_fit(cuda, N):
    """K = 2048 without a K split: the activations of the whole K for a 32-row block
    leave no shared memory for the weight ring (the 32-row plan is not fast), so the
    rows run as 16-row blocks of the fast kernel. Against the oracle."""
    from moat_b200.gemm import plan
    K, M = 2048, 19200
    assert plan(32, K, M)["kind"] == 0 and plan(16, K, M)["kind"] == 1
    st, w = _wide(K, M)
    x = O.make_activations(N, K, 3 + N)
    close(run(x, st, K, M), O.gemm(x, w))


def test_metal_known_answers(cuda):
    """KATs of antigravity-engine/tests/test_metal_kernels.cpp restated for the INT4 path:
    byte 0x7F with scale 0.5 dequantizes to +3.5 (even) / -0.5 (odd) (:68-91), and
    all-ones activations against a constant 0.5 weight over K=16 give 8.0 (:97-130)."""
    import torch
    from moat_b200 import dequant as D
    from moat_b200.gemm import batched_gemm
    sb = np.zeros(144, np.uint8)
    sb[:16] = np.full(8, 0.5, np.float16).view(np.uint8)
    sb[16:] = 0x7F
    deq = D.unpack_superblock_weights(sb, 1)
    assert float(deq[0]) == 3.5 and float(deq[1]) == -0.5
    # constant 0.5 weights: q = 1 with scale 0.5 -> nibble 9
    K, M, N = 16, 256, 8
    st = np.zeros(K * M // 256 * 144, np.uint8).reshape(-1, 144)
    st[:, :16] = np.full(8, 0.5, np.float16).view(np.uint8)
    st[:, 16:] = 0x99
    y = batched_gemm(torch.ones(N, K, dtype=torch.float16, device="cuda"), torch.from_numpy(st.reshape(-1)).cuda(),
                     K, M).cpu().numpy()
    assert np.all(y == 8.0)
    assert not np.any(np.isnan(y)) and not np.any(np.isinf(y))


@pytest.mark.parametrize("N", [1, 8, 16, 32])
def test_repeated_calls_are_deterministic(cuda, N):
    """The split-K partial sums are reduced in a fixed order on chip: 20 back-to-back
    calls on one stream give bit-identical results and the device error word stays 0."""
    import torch
    from moat_b200.gemm import batched_gemm
    K, M = 3072, 8192
    st = torch.from_numpy(O.quantize_pack_matrix(O.make_weights(K, M, 5))).cuda()
    x = torch.from_numpy(O.make_activations(N, K, 5)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    first = batched_gemm(x, st, K, M, dev_err=err).clone()
    for _ in range(20):
        y = batched_gemm(x, st, K, M, dev_err=err)
    torch.cuda.synchronize()
    assert torch.equal(y, first)
    assert int(err.item()) == 0


def test_numpy_host_inputs_end_to_end(cuda):
    from moat_b200.gemm import batched_gemm
    K, M, N = 512, 1024, 4
    st = O.quantize_pack_matrix(O.make_weights(K, M, 9))
    x = O.make_activations(N, K, 9)
    y = batched_gemm(x, st, K, M)
    assert isinstance(y, np.ndarray) and y.dtype == np.float16 and y.shape == (N, M)
    close(y, O.gemm(x, O.unpack_superblock_weights(st).reshape(K, M)))



@pytest.mark.parametrize("N", [1, 5, 32, 40])
def test_host_buffer_path_matches_device_path(cuda, N):
    """mb_int4_gemm_host (pinned host activations in, host output out, one C call)
    gives the device path's bits; asynchronous calls on one stream reuse the staging
    buffers in order."""
    import torch
    from moat_b200.gemm import batched_gemm
    K, M = 512, 1024
    st = O.quantize_pack_matrix(O.make_weights(K, M, 5))
    sb = torch.from_numpy(st).cuda()
    xs = [O.make_activations(N, K, 10 + i) for i in range(3)]
    refs = [batched_gemm(torch.from_numpy(x).cuda(), sb, K, M).cpu().numpy() for x in xs]
    hx = [torch.from_numpy(x).pin_memory() for x in xs]
    hy = [torch.empty((N, M), dtype=torch.float16).pin_memory() for _ in xs]
    got = batched_gemm(hx[0], sb, K, M, out=hy[0])  # synchronous
    np.testing.assert_array_equal(got.numpy().view(np.uint16), refs[0].view(np.uint16))
    for i in range(3):
        batched_gemm(hx[i], sb, K, M, out=hy[i], sync=False)
    torch.cuda.synchronize()
    for i in range(3):
        np.testing.assert_array_equal(hy[i].numpy().view(np.uint16), refs[i].view(np.uint16))
    close(hy[2].numpy(), O.gemm(xs[2], O.unpack_superblock_weights(st).reshape(K, M)))


def test_overlapped_host_calls_across_slots_shapes_and_growth(cuda):
    """Host-buffer calls with sync=False: more calls than staging slots, mixed batch
    sizes (N > 32 included) and weights, and one call large enough to grow the
    staging (which first waits for the calls in flight); after host_wait every
    output equals the device path's bits."""
    import torch
    from moat_b200.gemm import batched_gemm, host_wait
    shapes = [(512, 1024), (2048, 8192)]
    sbs = {s: torch.from_numpy(O.quantize_pack_matrix(O.make_weights(s[0], s[1], 7 + i))).cuda()
           for i, s in enumerate(shapes)}
    calls = [(shapes[0], n) for n in (1, 7, 32, 40, 3, 16, 1, 9)] + [(shapes[1], 200)] + \
            [(shapes[0], n) for n in (2, 33, 5)]
    xs, hys, refs = [], [], []
    for i, ((K, M), n) in enumerate(calls):
        x = O.make_activations(n, K, 100 + i)
        refs.append(batched_gemm(torch.from_numpy(x).cuda(), sbs[(K, M)], K, M).cpu().numpy())
        xs.append(torch.from_numpy(x).pin_memory())
        hys.append(torch.empty((n, M), dtype=torch.float16).pin_memory())
    torch.cuda.synchronize()
    for i, ((K, M), n) in enumerate(calls):
        batched_gemm(xs[i], sbs[(K, M)], K, M, out=hys[i], sync=False)
    host_wait()
    for i in range(len(calls)):
        np.testing.assert_array_equal(hys[i].numpy().view(np.uint16), refs[i].view(np.uint16), err_msg=str(calls[i]))
