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


def test_version_and_status_strings(L):
    assert L.mb_abi_version() == 1
    assert L.mb_status_string(0) == b"ok"
    assert L.mb_status_string(-2) == b"invalid arguments"
    assert L.mb_status_string(-99) == b"unknown status"


def test_workspace_sizes(L):
    assert L.mb_int4_gemm_workspace_size(8, 2048, 2048) >= 8 * 2048 * 4
    assert L.mb_int4_gemm_workspace_size(64, 2048, 2048) == L.mb_int4_gemm_workspace_size(32, 2048, 2048)
    assert L.mb_int4_gemm_workspace_size(0, 2048, 2048) == 0
    ws = L.mb_decode_attn_workspace_size(16, 16, 4096, 128)
    assert ws >= 16 * 16 * 4096 * 4  # fp32 scores
    assert L.mb_decode_attn_workspace_size(0, 16, 4096, 128) == 0


def test_host_side_argument_validation(L):
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first
    # null pointers -> MB_ERR_NULL (-1)
    assert L.mb_int4_gemm(None, fake, fake, 8, 2048, 2048, fake, 1 << 20, None) == -1
    assert L.mb_int4_dequant(None, fake, 1, None) == -1
    assert L.mb_decode_attn(None, fake, fake, fake, 1, 1, 16, 128, 1.0, fake, 32768, 16.0, fake, 1 << 30, None) == -1
    # bad shapes -> MB_ERR_ARGS (-2)
    assert L.mb_int4_gemm(fake, fake, fake, 8, 3, 5, fake, 1 << 20, None) == -2   # K*M % 256 != 0
    assert L.mb_int4_gemm(fake, fake, fake, 0, 2048, 2048, fake, 1 << 20, None) == -2
    assert L.mb_int4_quantize(fake, 0, 33, 0, fake, None, None, None) == -2
    assert L.mb_int4_quantize(fake, 0, 32, 0, None, None, fake, None) == -2       # packing needs n % 256
    assert L.mb_int4_quantize(fake, 0, 256, 2, fake, None, None, None) == -2      # unknown variant
    assert L.mb_int4_extract_columns(fake, 64, 512, 16, 256, fake, None) == -2    # not group aligned
    assert L.mb_decode_attn(fake, fake, fake, fake, 1, 1, 16, 100, 1.0, fake, 32768, 16.0, fake, 1 << 30, None) == -2
    assert L.mb_exp_lut_lookup(fake, 1, 10.0, fake, 4, fake, None) == -2
    # workspace too small -> MB_ERR_WORKSPACE (-3)
    assert L.mb_int4_gemm(fake, fake, ctypes.c_void_p(0x10000), 8, 2048, 2048, ctypes.c_void_p(0x10000), 16,
                          None) == -3
    # misaligned -> MB_ERR_ALIGN (-5)
    assert L.mb_int4_dequant(ctypes.c_void_p(0x10001), fake, 1, None) == -5
