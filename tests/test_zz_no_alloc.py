"""The fixed-scratch decode attention entry point (``mb_decode_attn_noalloc``).

It runs the same kernels as ``mb_decode_attn`` on a scratch array owned by the
library, so on the same inputs its output must match the workspace entry point.
Two calls in a row with different shapes, both on the three-pass path that uses the
scratch, check that what the first call leaves in the scratch (statistics, arrival
counters) does not leak into the second. This file sorts last so the test also
runs after every other GPU test has used the device.
"""

import ctypes

import numpy as np
import pytest

from moat_b200 import _lib

NOALLOC_LIMIT = 16 << 20  # MB_ATTN_NOALLOC_SCRATCH_BYTES


@pytest.fixture(scope="module")
def L():
    return _lib.lib()


def test_noalloc_host_side_validation(L):
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first
    assert L.mb_decode_attn_noalloc(None, fake, fake, fake, 1, 1, 16, 128, 1.0, fake, 32768, 16.0, None) == -1
    assert L.mb_decode_attn_noalloc(fake, fake, fake, fake, 1, 1, 16, 100, 1.0, fake, 32768, 16.0, None) == -2
    assert L.mb_decode_attn_noalloc(ctypes.c_void_p(0x10008), fake, fake, fake, 1, 1, 16, 128, 1.0, fake,
                                    32768, 16.0, None) == -5
    # beyond the fixed scratch: MB_ERR_WORKSPACE, before any CUDA call
    T, H, Lk, d = 16, 16, 16384, 128
    assert L.mb_decode_attn_workspace_size(T, H, Lk, d) > NOALLOC_LIMIT
    assert L.mb_decode_attn_noalloc(fake, fake, fake, fake, T, H, Lk, d, 1.0, fake, 32768, 16.0, None) == -3
    # the shapes the GPU test below uses fit
    assert L.mb_decode_attn_workspace_size(16, 16, 4096, 128) <= NOALLOC_LIMIT


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point(L, cuda):
    import torch
    from moat_b200.attention import ExponentialLUT

    lut = ExponentialLUT(range_max=16.0)
    table = lut.device_table(cuda)
    st = torch.cuda.current_stream(cuda).cuda_stream
    rng = np.random.default_rng(11)
    # two calls in a row, both on the three-pass path (caches longer than the
    # 2048-position one-CTA-per-row path): config 4 (16 traces x 16 heads x 4096 x 128),
    # then a ragged shape with other row and chunk counts, so the second call's
    # statistics and arrival counters start from what the first call left in the scratch
    for T, H, Lk, d in ((16, 16, 4096, 128), (3, 5, 2600, 64)):
        q = torch.from_numpy(rng.standard_normal((T, H, d)).astype(np.float16)).to(cuda)
        k = torch.from_numpy(rng.standard_normal((T, H, Lk, d)).astype(np.float16)).to(cuda)
        v = torch.from_numpy(rng.standard_normal((T, H, Lk, d)).astype(np.float16)).to(cuda)
        scale = float(np.float32(1.0 / np.sqrt(d)))
        nbytes = int(L.mb_decode_attn_workspace_size(T, H, Lk, d))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
        ref = torch.empty((T, H, d), dtype=torch.float16, device=cuda)
        got = torch.full((T, H, d), float("nan"), dtype=torch.float16, device=cuda)
        rc = L.mb_decode_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), T, H, Lk, d, scale,
                              table.data_ptr(), lut.size, 16.0, ws.data_ptr(), nbytes, st)
        assert rc == 0
        rc = L.mb_decode_attn_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(), T, H, Lk, d,
                                      scale, table.data_ptr(), lut.size, 16.0, st)
        assert rc == 0
        torch.cuda.synchronize(cuda)
        g = got.float().cpu().numpy()
        r = ref.float().cpu().numpy()
        assert np.all(np.isfinite(g))
        np.testing.assert_allclose(g, r, rtol=1e-2, atol=1e-2)
        # same kernels, same order of sums: identical bits
        np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), ref.cpu().numpy().view(np.uint16))
