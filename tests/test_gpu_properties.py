"""Size-independent properties at the full BASELINE sizes, where running the NumPy
oracle on every case would take too long: exact scaling, additivity, shard / join
consistency, pack / unpack identity, and argmax agreement of the LUT attention.
"""

import numpy as np
import pytest

from oracle import attention as OA
from oracle import int4 as O

pytestmark = pytest.mark.gpu

K3, M3 = 3072, 8192


@pytest.fixture(scope="module")
def cfg3(cuda):
    import torch
    from moat_b200.dequant import quantize_to_superblocks
    g = torch.Generator(device=cuda).manual_seed(33)
    w = torch.randn((K3, M3), generator=g, device=cuda) * 0.02
    return quantize_to_superblocks(w.reshape(-1))


@pytest.mark.parametrize("N", [1, 8, 32])
def test_power_of_two_scaling_is_exact(cuda, cfg3, N):
    """gemm(2x) == 2 gemm(x) bit for bit: doubling an fp16 input doubles every scaled
    activation fp16(x s), every fp32 product and partial sum exactly, whatever the
    summation order, and the fp16 rounding commutes with the doubling outside the
    subnormal range. The activations keep |x| >= 1/4 so that no x s is an fp16
    subnormal (group scales here are above 1e-3), where rounding does not commute with
    doubling."""
    import torch
    from moat_b200.gemm import batched_gemm
    g = torch.Generator(device=cuda).manual_seed(N)
    x = torch.randn((N, K3), generator=g, device=cuda)
    x = (torch.sign(x) * x.abs().clamp(min=0.25)).half()
    y1 = batched_gemm(x, cfg3, K3, M3).float()
    y2 = batched_gemm(x * 2, cfg3, K3, M3).float()
    normal = y1.abs() >= 2.0 ** -14
    assert torch.equal(y2[normal], 2 * y1[normal])


@pytest.mark.parametrize("N", [4, 32])
def test_additivity(cuda, cfg3, N):
    """gemm(a + b) == gemm(a) + gemm(b) within the 1e-2 bar (fp16 rounding of a + b
    and of the three outputs is the only difference)."""
    import torch
    from moat_b200.gemm import batched_gemm
    g = torch.Generator(device=cuda).manual_seed(100 + N)
    a = torch.randn((N, K3), generator=g, device=cuda).half()
    b = torch.randn((N, K3), generator=g, device=cuda).half()
    lhs = batched_gemm(a + b, cfg3, K3, M3).float()
    rhs = batched_gemm(a, cfg3, K3, M3).float() + batched_gemm(b, cfg3, K3, M3).float()
    torch.testing.assert_close(lhs, rhs, rtol=1e-2, atol=1e-2)
    assert ((lhs - rhs).norm() / rhs.norm()).item() < 1e-3


@pytest.mark.parametrize("world", [2, 4, 8])
def test_column_shards_join_to_the_full_product(cuda, cfg3, world):
    """The multi-GPU layout on one GPU: every rank's group-aligned column shard,
    re-packed and multiplied on its own, joins to the unsharded product."""
    import torch
    from moat_b200.dequant import extract_columns
    from moat_b200.dist import column_bounds
    from moat_b200.gemm import batched_gemm
    N = 16
    g = torch.Generator(device=cuda).manual_seed(world)
    x = torch.randn((N, K3), generator=g, device=cuda).half()
    full = batched_gemm(x, cfg3, K3, M3).float()
    parts = []
    for c0, c1 in column_bounds(M3, world, K3):
        shard = extract_columns(cfg3, K3, M3, c0, c1)
        parts.append(batched_gemm(x, shard, K3, c1 - c0).float())
    joined = torch.cat(parts, dim=1)
    torch.testing.assert_close(joined, full, rtol=1e-2, atol=1e-2)
    assert ((joined - full).norm() / full.norm()).item() < 1e-3


def test_pack_unpack_identity_full_size(cuda, cfg3):
    """stream -> (q, scales) -> stream is the identity on the 14 MB config-3 stream,
    and dequant equals q * scale rounded once to fp16."""
    import torch
    from moat_b200.dequant import pack_superblocks, unpack_superblock_weights, unpack_superblocks
    q, s = unpack_superblocks(cfg3)
    again = pack_superblocks(q, s)
    assert torch.equal(again, cfg3)
    assert int(q.min()) >= -8 and int(q.max()) <= 7
    deq = unpack_superblock_weights(cfg3, K3 * M3 // 256)
    ref = (q.float().reshape(-1, 32) * s.float().reshape(-1, 1)).half().reshape(-1)
    assert torch.equal(deq.view(torch.int16), ref.view(torch.int16))


def test_attention_argmax_agreement_config4(cuda):
    """per (trace, head), the argmax over the head dimension of
    the LUT attention output agrees with exact-exp attention on >= 99% of rows."""
    import torch
    from moat_b200.attention import ExponentialLUT, decode_attention
    T, H, L, d = 16, 16, 4096, 128
    q, k, v = OA.make_attention_inputs(T, H, L, d, 9)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = decode_attention(qd, kd, vd, ExponentialLUT(range_max=16.0)).float()
    s = torch.einsum("thd,thld->thl", qd.float(), kd.float()) / np.sqrt(d)
    exact = torch.einsum("thl,thld->thd", torch.softmax(s, -1), vd.float())
    agree = (out.argmax(-1) == exact.argmax(-1)).float().mean().item()
    assert agree >= 0.99, agree


def test_gemm_matches_oracle_on_a_full_size_sample(cuda, cfg3):
    """A column sample of the full config-3 product against the oracle's fp32 GEMM
    of the same dequantized weights (the oracle runs on 512 columns only)."""
    import torch
    from moat_b200.dequant import extract_columns
    from moat_b200.gemm import batched_gemm
    N = 32
    x = O.make_activations(N, K3, 5)
    y = batched_gemm(torch.from_numpy(x).cuda(), cfg3, K3, M3).float().cpu().numpy()
    c0, c1 = 4096, 4608
    st = extract_columns(cfg3, K3, M3, c0, c1).cpu().numpy()
    w = O.unpack_superblock_weights(st).reshape(K3, c1 - c0)
    ref = O.gemm(x, w).astype(np.float32)
    np.testing.assert_allclose(y[:, c0:c1], ref, rtol=1e-2, atol=1e-2)
