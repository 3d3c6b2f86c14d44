"""The ``batched_gemm`` entry point: N decode traces x INT4 super-block weights.

``out[N, M] = activations[N, K] @ dequant(superblocks)[K, M]`` in fp16 with fp32
accumulation, computed by the fused weight-streaming sm_100a kernel (C ABI
``mb_int4_gemm``). Replaces the reference's Metal ``batched_gemm_simdgroup`` /
``fused_batched_gemm_int4`` (``antigravity-engine/src/shaders/batched_gemm.metal:74-169``,
buffers ``activations, weights, output, N, K, M``) whose CPU form is the decode
step's ``activations @ W`` (``antigravity-engine/src/batch_generator.py:290``).

The weights are the reference's 144-byte super-block stream of the row-major
``[K, M]`` matrix (flat index ``k*M + m``). Host (NumPy) inputs are copied to the
GPU and the result copied back, which is the end-to-end path; torch CUDA tensors stay
on the device.
"""

from __future__ import annotations

import numpy as np

from . import _lib
from ._lib import check, lib, ptr, stream_of, to_device

def plan(N: int, K: int, M: int) -> dict:
    """The launch plan the kernel uses for a shape (strip width, cluster K split, grid)."""
    import ctypes
    info = (ctypes.c_int32 * 8)()
    check(lib().mb_int4_gemm_plan(N, K, M, info), "mb_int4_gemm_plan")
    keys = ("kind", "strip", "cluster", "grid", "stages", "smem", "extra", "tiles")
    return dict(zip(keys, list(info)))


_staging = _lib.WorkspacePool()


def batched_gemm(activations, superblocks, K: int, M: int, out=None, dev_err=None, sync: bool = True):
    """fp16 ``[N, K] x int4[K, M] -> fp16 [N, M]`` with fp32 accumulation.

    activations: fp16 ``[N, K]`` (NumPy, torch CUDA, or torch CPU); superblocks:
    uint8 ``[K*M/256*144]`` super-block stream on the same device (or NumPy);
    ``out``: optional fp16 ``[N, M]`` tensor to write into; ``dev_err``: optional
    int32 CUDA tensor whose first word receives device error bits (bounded waits).

    Host path: with CPU torch ``activations`` and a CPU torch ``out`` (pinned memory
    for asynchronous copies) and the weights on a GPU, one C call enqueues the copy in,
    the GEMM (on the current stream) and the copy back (``mb_int4_gemm_host_overlap``:
    the copies run on library streams, so consecutive calls' copies overlap their
    neighbours' GEMMs); with ``sync=False`` it returns at once, and ``out`` is complete
    (and ``activations`` free to change) after ``host_wait()`` or a device synchronise.
    """
    t = _lib.torch()
    if type(activations) is t.Tensor and type(superblocks) is t.Tensor and superblocks.is_cuda:
        if activations.is_cuda:
            fast = _batched_gemm_device(t, activations, superblocks, K, M, out, dev_err)
            if fast is not None:
                return fast
        elif type(out) is t.Tensor and not out.is_cuda:
            return _batched_gemm_host(t, activations, superblocks, K, M, out, dev_err, sync)
    a, was_np = to_device(activations, t.float16)
    if a.dim() == 1:
        a = a.reshape(1, -1)
    N = a.shape[0]
    if a.shape[1] != K:
        raise ValueError(f"activations have {a.shape[1]} columns, expected K={K}")
    if (K * M) % 256 != 0:
        raise ValueError(f"K*M = {K * M} is not a multiple of 256")
    sb, _ = to_device(superblocks, t.uint8, a.device)
    if sb.numel() != K * M // 256 * 144:
        raise ValueError(f"superblock stream has {sb.numel()} bytes, expected {K * M // 256 * 144}")
    if out is None:
        out = t.empty((N, M), dtype=t.float16, device=a.device)
    elif out.shape != (N, M) or out.dtype != t.float16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous fp16 [N, M] tensor")
    check(lib().mb_int4_gemm(ptr(a), ptr(sb), ptr(out), N, K, M, ptr(dev_err) if dev_err is not None else None,
                             stream_of(a.device)), "mb_int4_gemm")
    if was_np:
        return out.cpu().numpy()
    return out


def _batched_gemm_device(t, a, sb, K: int, M: int, out, dev_err):
    """The common case with few Python-side checks: contiguous fp16 CUDA activations,
    uint8 CUDA weights on the same device. Returns None to fall back to the general
    path for anything else."""
    if a.dtype is not t.float16 or sb.dtype is not t.uint8 or a.device != sb.device or not a.is_contiguous():
        return None
    shape = a.shape
    if len(shape) == 2:
        N = shape[0]
        if shape[1] != K:
            raise ValueError(f"activations have {shape[1]} columns, expected K={K}")
    elif len(shape) == 1 and shape[0] == K:
        N = 1
    else:
        return None
    if (K * M) % 256 != 0:
        raise ValueError(f"K*M = {K * M} is not a multiple of 256")
    if sb.numel() != K * M // 256 * 144:
        raise ValueError(f"superblock stream has {sb.numel()} bytes, expected {K * M // 256 * 144}")
    dev = a.device
    if out is None:
        out = t.empty((N, M), dtype=t.float16, device=dev)
    elif out.dtype is not t.float16 or out.device != dev or out.numel() != N * M or not out.is_contiguous():
        raise ValueError("out must be a contiguous fp16 [N, M] tensor on the activations' device")
    rc = lib().mb_int4_gemm(a.data_ptr(), sb.data_ptr(), out.data_ptr(), N, K, M,
                            dev_err.data_ptr() if dev_err is not None else None, stream_of(dev))
    if rc != 0:
        check(rc, "mb_int4_gemm")
    return out


class _HostStaging:
    """Per-(device, stream) device staging of the overlapped host calls. It only grows,
    and first waits for the calls still using it (they run on library streams, which
    torch's allocator does not track)."""

    def __init__(self):
        import threading
        self._bufs = {}
        self._lock = threading.Lock()

    def get(self, device_index: int, stream: int, nbytes: int):
        key = (device_index, stream)
        buf = self._bufs.get(key)  # the common case: an existing buffer large enough
        if buf is not None and buf.numel() >= nbytes:
            return buf
        t = _lib.torch()
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                if buf is not None:
                    check(lib().mb_int4_gemm_host_wait(stream), "mb_int4_gemm_host_wait")
                buf = t.empty(max(nbytes, 4 << 20), dtype=t.uint8, device=t.device("cuda", device_index))
                self._bufs[key] = buf
            return buf


_host_staging = _HostStaging()
_HOST_SLOTS = 4  # MB_HOST_SLOTS


def _batched_gemm_host(t, a, sb, K: int, M: int, out, dev_err, sync: bool):
    if a.dim() == 1:
        a = a.reshape(1, -1)
    N = a.shape[0]
    if a.dtype != t.float16 or not a.is_contiguous() or a.shape[1] != K:
        raise ValueError(f"activations must be a contiguous fp16 [N, {K}] tensor")
    if out.dtype != t.float16 or not out.is_contiguous() or tuple(out.shape) != (N, M):
        raise ValueError(f"out must be a contiguous fp16 [{N}, {M}] tensor")
    if (K * M) % 256 != 0:
        raise ValueError(f"K*M = {K * M} is not a multiple of 256")
    if sb.dtype != t.uint8 or sb.numel() != K * M // 256 * 144:
        raise ValueError(f"superblock stream must be uint8 with {K * M // 256 * 144} bytes")
    dev = sb.get_device()
    st = stream_of(dev)
    slot = ((N * K * 2 + 255) // 256 + (N * M * 2 + 255) // 256) * 256
    buf = _host_staging.get(dev, st, _HOST_SLOTS * slot)
    L = lib()
    check(L.mb_int4_gemm_host_overlap(a.data_ptr(), sb.data_ptr(), out.data_ptr(), N, K, M, buf.data_ptr(),
                                      buf.numel(), ptr(dev_err) if dev_err is not None else None, st),
          "mb_int4_gemm_host_overlap")
    if sync:
        check(L.mb_int4_gemm_host_wait(st), "mb_int4_gemm_host_wait")
    return out


def host_wait(device=None) -> None:
    """Wait until every host-buffer ``batched_gemm(..., sync=False)`` call enqueued on
    the current stream of ``device`` has written its output."""
    t = _lib.torch()
    dev = t.device("cuda", t.cuda.current_device()) if device is None else t.device(device)
    check(lib().mb_int4_gemm_host_wait(stream_of(dev)), "mb_int4_gemm_host_wait")


def gemm_bytes(N: int, K: int, M: int) -> int:
    """Algorithmic HBM bytes of one call: packed weights + activations + output."""
    return K * M * 144 // 256 + 2 * N * K + 2 * N * M


def gemm_flops(N: int, K: int, M: int) -> int:
    return 2 * N * K * M


__all__ = ["batched_gemm", "host_wait", "plan", "gemm_bytes", "gemm_flops"]

_ = np  # numpy inputs are accepted through to_device
