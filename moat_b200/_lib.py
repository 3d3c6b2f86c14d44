"""ctypes binding of the in-tree CUDA library (C ABI in ``include/moat_b200.h``).

There is no CPU fallback: if ``moat_b200/_lib/libmoat_b200.so`` is missing or does
not load, every accelerated entry point raises. Build it with
``python -m moat_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libmoat_b200.so")

_c_i32, _c_i64, _c_sz, _c_f, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float, ctypes.c_void_p

# name -> (restype, argtypes); one entry per function declared in include/moat_b200.h
SIGNATURES = {
    "mb_abi_version": (_c_i32, []),
    "mb_status_string": (ctypes.c_char_p, [_c_i32]),
    "mb_int4_quantize": (_c_i32, [_vp, _c_i32, _c_i64, _c_i32, _vp, _vp, _vp, _vp]),
    "mb_int4_pack": (_c_i32, [_vp, _vp, _c_i64, _vp, _vp]),
    "mb_int4_unpack": (_c_i32, [_vp, _c_i64, _vp, _vp, _vp]),
    "mb_int4_dequant": (_c_i32, [_vp, _vp, _c_i64, _vp]),
    "mb_int4_dequant_q": (_c_i32, [_vp, _vp, _c_i64, _c_i32, _vp, _vp]),
    "mb_lut_gather_f16": (_c_i32, [_vp, _c_i64, _vp, _c_i64, _c_i32, _c_i64, _vp, _vp]),
    "mb_int4_gemm": (_c_i32, [_vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _vp, _vp]),
    "mb_int4_gemm_host": (_c_i32, [_vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _vp, _vp, _vp, _vp]),
    "mb_int4_gemm_host_staging_bytes": (_c_sz, [_c_i32, _c_i32, _c_i32]),
    "mb_int4_gemm_host_overlap": (_c_i32, [_vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _vp, _c_sz, _vp, _vp]),
    "mb_int4_gemm_host_wait": (_c_i32, [_vp]),
    "mb_int4_gemm_plan": (_c_i32, [_c_i32, _c_i32, _c_i32, ctypes.POINTER(_c_i32)]),
    "mb_int4_extract_columns": (_c_i32, [_vp, _c_i32, _c_i32, _c_i32, _c_i32, _vp, _vp]),
    "mb_exp_lut_lookup": (_c_i32, [_vp, _c_i32, _c_f, _vp, _c_i64, _vp, _vp]),
    "mb_lut_softmax": (_c_i32, [_vp, _c_i64, _c_i64, _vp, _c_i32, _c_f, _vp, _vp]),
    "mb_decode_attn_workspace_size": (_c_sz, [_c_i32, _c_i32, _c_i32, _c_i32]),
    "mb_decode_attn": (_c_i32, [_vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32, _c_f, _vp, _c_i32, _c_f,
                                _vp, _c_sz, _vp]),
    "mb_decode_attn_cache": (_c_i32, [_vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f, _vp,
                                      _c_i32, _c_f, _vp, _c_sz, _vp]),
    "mb_decode_attn_cache_lens": (_c_i32, [_vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32, _vp, _c_i32, _c_f,
                                           _vp, _c_i32, _c_f, _vp, _c_sz, _vp]),
    "mb_embed": (_c_i32, [_vp, _c_i32, _vp, _c_i32, _c_i32, _vp, _vp, _vp]),
    "mb_add_rmsnorm": (_c_i32, [_vp, _vp, _vp, _c_i32, _c_i32, _c_f, _vp, _vp]),
    "mb_rope_append": (_c_i32, [_vp, _c_i32, _c_i32, _c_i32, _vp, _vp, _c_i32, _vp, _vp, _vp, _vp, _vp]),
    "mb_swiglu": (_c_i32, [_vp, _c_i32, _c_i32, _vp, _vp]),
    "mb_argmax_f16": (_c_i32, [_vp, _c_i32, _c_i32, _vp, _vp]),
    "mb_argmax_key_f16": (_c_i32, [_vp, _c_i32, _c_i32, _c_i32, _vp, _vp]),
    "mb_argmax_keys_to_ids": (_c_i32, [_vp, _c_i32, _vp, _vp]),
    "mb_advance_positions": (_c_i32, [_vp, _c_i32, _vp]),
    "mb_peer_buffer_bytes": (_c_sz, [_c_i32, _c_i32]),
    "mb_ipc_alloc": (_c_i32, [_c_sz, _vp, _vp]),
    "mb_ipc_open": (_c_i32, [_vp, _vp]),
    "mb_ipc_close": (_c_i32, [_vp]),
    "mb_ipc_free": (_c_i32, [_vp]),
    "mb_peer_add_rmsnorm": (_c_i32, [_vp, _c_i32, _c_i32, _c_i64, _c_i64, _vp, _vp, _vp, _c_i32, _c_i32, _c_f, _vp,
                                     _vp, _vp, _vp]),
    "mb_peer_argmax": (_c_i32, [_vp, _c_i32, _c_i32, _c_i64, _c_i64, _vp, _c_i32, _c_i32, _c_i32, _vp, _vp, _vp,
                                _vp]),
    "mb_int4_gemm_peer": (_c_i32, [_vp, _vp, _c_i32, _c_i32, _c_i32, _vp, _c_i32, _c_i32, _c_i64, _vp, _vp, _vp]),
    "mb_peer_sum_rmsnorm": (_c_i32, [_vp, _c_i32, _c_i32, _c_i64, _c_i64, _vp, _vp, _c_i32, _c_i32, _c_f, _vp, _vp,
                                     _vp, _vp]),
    "mb_sample_workspace_size": (_c_sz, [_c_i32, _c_i32]),
    "mb_sample_tokens": (_c_i32, [_vp, _c_i32, _c_i32, _c_i32, _c_f, _c_i32, _vp, _c_i32, _c_f, _vp, ctypes.c_uint64,
                                  _vp, _vp, _vp, _vp, _c_sz, _vp, _vp]),
    "mb_decode_attn_noalloc": (_c_i32, [_vp, _vp, _vp, _vp, _c_i32, _c_i32, _c_i32, _c_i32, _c_f, _vp, _c_i32,
                                        _c_f, _vp]),
}

_lock = threading.Lock()
_lib = None


class MoatError(RuntimeError):
    """A moat_b200 C-ABI call returned a non-zero status."""


def lib() -> ctypes.CDLL:
    """Load the CUDA library once; raise loudly if it is not there."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"moat_b200 CUDA library not built: {LIB_PATH} is missing "
                                      f"(run `python -m moat_b200.build`)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype, fn.argtypes = res, args
                _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().mb_status_string(rc).decode()
        raise MoatError(f"{what} failed: {msg} (status {rc})")


# ---------------------------------------------------------------------------
# tensor plumbing (torch is the device-memory / stream provider)
# ---------------------------------------------------------------------------
def torch():
    import torch as _t
    return _t


def require_cuda():
    t = torch()
    if not t.cuda.is_available():
        raise RuntimeError("moat_b200 kernels need a CUDA device (B200, sm_100a); none is visible")
    return t


def stream_of(device) -> int:
    """Raw handle of torch's current stream on ``device`` (a torch.device or index)."""
    t = torch()
    idx = device.index if hasattr(device, "index") else device
    if idx is None:
        idx = t.cuda.current_device()
    raw = getattr(t._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:  # the handle without building a Stream object
        return raw(idx)
    return t.cuda.current_stream(idx).cuda_stream


_NP2TORCH = {np.dtype(np.float16): "float16", np.dtype(np.float32): "float32", np.dtype(np.int8): "int8",
             np.dtype(np.uint8): "uint8", np.dtype(np.int32): "int32", np.dtype(np.int64): "int64",
             np.dtype(np.int16): "int16", np.dtype(np.uint16): "int16"}


def to_device(x, dtype=None, device=None):
    """numpy array or torch tensor -> contiguous torch CUDA tensor.

    Returns (tensor, was_numpy). ``dtype`` is a torch dtype to cast to (after the copy).
    """
    t = require_cuda()
    if isinstance(x, t.Tensor):
        was_np = False
        y = x
        if not y.is_cuda:
            y = y.to(device or "cuda")
    else:
        was_np = True
        a = np.ascontiguousarray(np.asarray(x))
        if a.dtype == np.uint16:
            a = a.view(np.int16)
        y = t.from_numpy(a).to(device or "cuda", non_blocking=False)
    if dtype is not None and y.dtype != dtype:
        y = y.to(dtype)
    return y.contiguous(), was_np


def ptr(tensor) -> int:
    return tensor.data_ptr()


class WorkspacePool:
    """Per-(device, stream) zero-initialised scratch buffers for kernels that need one.

    A buffer is only ever used by calls enqueued on its own stream, so calls that
    share it are ordered. Kernels leave the buffer zeroed again after each call.
    """

    def __init__(self):
        self._bufs = {}
        self._lock = threading.Lock()

    def get(self, device, stream: int, nbytes: int):
        t = torch()
        key = (str(device), stream)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                buf = t.zeros(size, dtype=t.uint8, device=device)
                self._bufs[key] = buf
            return buf
