"""The C-ABI library loads, exports every symbol ``include/moat_b200.h`` declares, and
rejects bad arguments on the host (no GPU needed: validation happens before any
CUDA call)."""

import ctypes
import os
import re

import pytest

from moat_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moat_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(_lib.LIB_PATH):
        from moat_b200.build import build
        build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(L):
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/moat_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature in moat_b200/_lib.py"


def test_binding_covers_only_declared(L):
    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_gemm_plans(L):
    """Host-side planning of the GEMM launch for the BASELINE shapes; needs no GPU
    (148 SMs assumed when none is visible)."""
    info = (ctypes.c_int32 * 8)()
    for (N, K, M) in [(8, 2048, 2048), (1, 3072, 8192), (32, 3072, 8192), (16, 2048, 5504), (16, 2048, 151936),
                      (16, 5504, 2048), (24, 3072, 8192)]:
        assert L.mb_int4_gemm_plan(N, K, M, info) == 0
        kind, strip, ck, grid, stages, smem = list(info)[:6]
        assert kind == 1, (N, K, M)
        assert smem <= 227 * 1024 and stages >= 1
        assert strip in (128, 256) and M % strip == 0 and 1 <= ck <= 8
        assert grid == (M // strip) * ck and (ck == 1 or grid <= 148)
    assert L.mb_int4_gemm_plan(8, 12, 64, info) == 0 and info[0] == 0  # generic path
    # no K split and K = 2048: 32 rows of activations over the whole K leave no room for
    # the weight ring, 16 rows do (the GEMM then runs 16-row blocks of the fast kernel)
    for M in (19200, 151936):
        assert L.mb_int4_gemm_plan(32, 2048, M, info) == 0 and info[0] == 0
        assert L.mb_int4_gemm_plan(16, 2048, M, info) == 0 and info[0] == 1 and info[2] == 1


def test_cluster_owner_ranges():
    """The cluster kernel's final reduction gives strip group g (32 columns) to CTA
    (g Ck) // GS of a Ck-CTA cluster, and CTA q adds the groups [ceil(q GS / Ck),
    ceil((q + 1) GS / Ck)): every group has exactly one owner rank < Ck, the owner's
    range contains it, the ranges tile the strip, and no CTA owns more than
    ceil(GS / Ck) groups (the receive-slot width). The planner may pick any Ck from 1
    to 8 for GS = 8 (256-wide strips) or 4 (128-wide)."""
    for GS in (4, 8):
        for Ck in range(1, 9):
            first = [(q * GS + Ck - 1) // Ck for q in range(Ck + 1)]
            assert first[0] == 0 and first[-1] == GS
            for g in range(GS):
                own = g * Ck // GS
                assert own < Ck and first[own] <= g < first[own + 1]
            assert max(first[q + 1] - first[q] for q in range(Ck)) <= -(-GS // Ck)


def test_version_and_status_strings(L):
    assert L.mb_abi_version() == 1
    assert L.mb_status_string(0) == b"ok"
    assert L.mb_status_string(-2) == b"invalid arguments"
    assert L.mb_status_string(-99) == b"unknown status"


def test_workspace_sizes(L):
    ws = L.mb_decode_attn_workspace_size(16, 16, 4096, 128)
    assert ws >= 16 * 16 * 4096 * 4  # fp32 scores
    assert L.mb_decode_attn_workspace_size(0, 16, 4096, 128) == 0


def test_host_side_argument_validation(L):
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first
    # null pointers -> MB_ERR_NULL (-1)
    assert L.mb_int4_gemm(None, fake, fake, 8, 2048, 2048, None, None) == -1
    assert L.mb_int4_gemm_host(fake, fake, fake, 8, 2048, 2048, None, fake, None, None) == -1
    assert L.mb_embed(None, 4, fake, 10, 16, fake, None, None) == -1
    assert L.mb_add_rmsnorm(fake, None, fake, 0, 16, 1e-6, fake, None) == -2
    assert L.mb_rope_append(fake, 2, 2, 7, fake, fake, 16, fake, fake, fake, None, None) == -2   # odd head dim
    assert L.mb_swiglu(fake, 2, 0, fake, None) == -2
    assert L.mb_argmax_f16(None, 2, 10, fake, None) == -1
    assert L.mb_decode_attn_cache(fake, fake, fake, fake, 1, 1, 20, 10, 128, 1.0, fake, 32768, 16.0, fake,
                                  1 << 30, None) == -2  # L > Lmax
    assert L.mb_int4_gemm_host(fake, fake, fake, 8, 3, 5, fake, fake, None, None) == -2
    # overlapped host calls: staging is MB_HOST_SLOTS (4) fixed-size slots
    slot = (32 * 3072 * 2 + 255) // 256 * 256 + (32 * 8192 * 2 + 255) // 256 * 256
    assert L.mb_int4_gemm_host_staging_bytes(32, 3072, 8192) == 4 * slot
    assert L.mb_int4_gemm_host_staging_bytes(0, 3072, 8192) == 0
    big = ctypes.c_void_p(0x100000)
    assert L.mb_int4_gemm_host_overlap(fake, fake, fake, 32, 3072, 8192, None, 4 * slot, None, None) == -1
    assert L.mb_int4_gemm_host_overlap(fake, fake, fake, 8, 3, 5, big, 4 * slot, None, None) == -2
    assert L.mb_int4_gemm_host_overlap(fake, fake, fake, 32, 3072, 8192, ctypes.c_void_p(0x100010), 4 * slot,
                                       None, None) == -5  # staging not 256-byte aligned
    assert L.mb_int4_gemm_host_overlap(fake, fake, fake, 32, 3072, 8192, big, 4 * slot - 256, None, None) == -3
    assert L.mb_int4_dequant(None, fake, 1, None) == -1
    assert L.mb_decode_attn(None, fake, fake, fake, 1, 1, 16, 128, 1.0, fake, 32768, 16.0, fake, 1 << 30, None) == -1
    # bad shapes -> MB_ERR_ARGS (-2)
    assert L.mb_int4_gemm(fake, fake, fake, 8, 3, 5, None, None) == -2   # K*M % 256 != 0
    assert L.mb_int4_gemm(fake, fake, fake, 0, 2048, 2048, None, None) == -2
    assert L.mb_int4_quantize(fake, 0, 33, 0, fake, None, None, None) == -2
    assert L.mb_int4_quantize(fake, 0, 32, 0, None, None, fake, None) == -2       # packing needs n % 256
    assert L.mb_int4_quantize(fake, 0, 256, 2, fake, None, None, None) == -2      # unknown variant
    assert L.mb_int4_extract_columns(fake, 64, 512, 16, 256, fake, None) == -2    # not group aligned
    assert L.mb_decode_attn(fake, fake, fake, fake, 1, 1, 16, 100, 1.0, fake, 32768, 16.0, fake, 1 << 30, None) == -2
    assert L.mb_exp_lut_lookup(fake, 1, 10.0, fake, 4, fake, None) == -2
    # workspace too small -> MB_ERR_WORKSPACE (-3)
    assert L.mb_decode_attn(fake, fake, fake, fake, 1, 1, 16, 128, 1.0, fake, 32768, 16.0, fake, 16, None) == -3
    # misaligned -> MB_ERR_ALIGN (-5)
    assert L.mb_int4_dequant(ctypes.c_void_p(0x10001), fake, 1, None) == -5


def test_tensor_parallel_and_sampling_entries_validate_on_the_host(L):
    fake = ctypes.c_void_p(0x10000)
    bufs = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    # key words, then two parities x 8 ranks of row slots; every 8-byte word carries
    # two fp16 payload values and the call's epoch
    assert L.mb_peer_buffer_bytes(16, 2048) == 16384 + 2 * 8 * (16 * 2048 // 2) * 8
    assert L.mb_peer_buffer_bytes(0, 2048) == 0 and L.mb_peer_buffer_bytes(65, 2048) == 0
    assert L.mb_peer_buffer_bytes(16, 100) == 0
    assert L.mb_argmax_key_f16(None, 2, 10, 0, fake, None) == -1
    assert L.mb_argmax_key_f16(fake, 2, 10, -1, fake, None) == -2
    assert L.mb_argmax_keys_to_ids(fake, 0, fake, None) == -2
    assert L.mb_ipc_alloc(1024, None, fake) == -1
    assert L.mb_ipc_open(None, fake) == -1
    # peer exchange: null pointers, too many rows, rows larger than a slot, bad rank / world
    assert L.mb_peer_add_rmsnorm(bufs, 2, 0, 4096, 10**9, None, fake, fake, 2, 2048, 1e-6, fake, fake, None,
                                 None) == -1
    assert L.mb_peer_add_rmsnorm(bufs, 2, 0, 65 * 2048, 10**9, fake, fake, fake, 65, 2048, 1e-6, fake, fake, None,
                                 None) == -2
    assert L.mb_peer_add_rmsnorm(bufs, 2, 0, 2048, 10**9, fake, fake, fake, 2, 2048, 1e-6, fake, fake, None,
                                 None) == -2
    assert L.mb_peer_add_rmsnorm(bufs, 2, 2, 4096, 10**9, fake, fake, fake, 2, 2048, 1e-6, fake, fake, None,
                                 None) == -2
    assert L.mb_peer_add_rmsnorm(bufs, 9, 0, 4096, 10**9, fake, fake, fake, 2, 2048, 1e-6, fake, fake, None,
                                 None) == -2
    # the row-parallel GEMM that stores into the exchange buffers, and its join
    assert L.mb_int4_gemm_peer(fake, fake, 16, 1024, 2048, bufs, 2, 0, 16 * 2048, None, None, None) == -1
    assert L.mb_int4_gemm_peer(fake, fake, 65, 1024, 2048, bufs, 2, 0, 65 * 2048, fake, None, None) == -2
    assert L.mb_int4_gemm_peer(fake, fake, 16, 1024, 2048, bufs, 2, 0, 2048, fake, None, None) == -2  # slot
    assert L.mb_int4_gemm_peer(fake, fake, 16, 1024, 2048, bufs, 2, 2, 16 * 2048, fake, None, None) == -2
    assert L.mb_int4_gemm_peer(ctypes.c_void_p(0x10008), fake, 16, 1024, 2048, bufs, 2, 0, 16 * 2048, fake, None,
                               None) == -6  # unaligned activations: off the fast plan
    assert L.mb_peer_sum_rmsnorm(bufs, 2, 0, 4096, 10**9, None, fake, 2, 2048, 1e-6, fake, fake, None, None) == -1
    assert L.mb_peer_sum_rmsnorm(bufs, 2, 0, 2048, 10**9, fake, fake, 2, 2048, 1e-6, fake, fake, None, None) == -2
    assert L.mb_peer_argmax(bufs, 2, 0, 4096, 0, fake, 2, 10, 0, fake, fake, None, None) == -2   # no timeout
    assert L.mb_peer_argmax(bufs, 2, 0, 4096, 10**9, fake, 2, 10, 0, None, fake, None, None) == -1
    # sampler: sizes, workspace, top_k range, dtype flag
    assert L.mb_sample_workspace_size(16, 151936) == (16 * 151936 * 2 + 255) // 256 * 256
    assert L.mb_sample_workspace_size(0, 10) == 0
    args = dict(T=0.7, k=50, size=32768, r=10.0)

    def samp(logits=fake, f32=0, N=2, V=100, k=50, ws_bytes=1 << 20, tokens=fake):
        return L.mb_sample_tokens(logits, f32, N, V, args["T"], k, fake, args["size"], args["r"], None, 0, fake,
                                  tokens, fake, fake, ws_bytes, None, None)
    assert samp(logits=None) == -1
    assert samp(tokens=None) == -1
    assert samp(k=0) == -2 and samp(k=65) == -2
    assert samp(f32=2) == -2
    assert samp(ws_bytes=16) == -3
