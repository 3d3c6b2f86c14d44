"""NVLink peer-memory exchanges for the tensor-parallel decode step.

Each rank allocates one exchange buffer, shares it with the other ranks of the
process group through CUDA IPC (handles passed with ``all_gather_object``) and maps
theirs. ``add_rmsnorm`` and ``argmax`` then each run as one kernel per rank that stores
its rows into the peers' buffers and waits, bounded, for theirs (``mb_peer_add_rmsnorm``
and ``mb_peer_argmax`` in ``include/moat_b200.h``). They replace, on the decode path, a
library all-reduce of the row-parallel partial products followed by the residual add
and RMSNorm, and the all-reduce of the greedy keys of a column-split vocabulary.
``gemm`` + ``sum_rmsnorm`` fuse the row-parallel projection with its join: the GEMM's
epilogue stores the rows into the exchange buffers itself (``mb_int4_gemm_peer``).

Every rank must make the same calls in the same order, on its own GPU: the exchange
refuses a group in which two ranks share a device, because the two kernels that wait
on each other could not both run. A wait that expires sets ``MB_DEVERR_TIMEOUT`` in the
caller's device error word.
"""

from __future__ import annotations

import ctypes
from typing import Optional

from . import _lib
from ._lib import check, lib, stream_of

HANDLE_BYTES = 64
DEVERR_TIMEOUT = 1
ERR_UNSUPPORTED = -6  # MB_ERR_UNSUPPORTED
STATE_WORDS = 64  # MB_PEER_STATE_WORDS: one epoch word per row and exchange kind


class PeerExchange:
    """Exchange buffers of one process group, for up to ``max_rows`` rows of ``D`` fp16
    values per call. ``timeout_s`` bounds every wait on another rank."""

    def __init__(self, max_rows: int, D: int, device, group=None, timeout_s: float = 10.0):
        import torch.distributed as dist
        t = _lib.require_cuda()
        L = lib()
        self.dev = t.device(device)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("peer exchange supports up to 8 ranks")
        self.max_rows, self.D = max_rows, D
        self.nbytes = int(L.mb_peer_buffer_bytes(max_rows, D))
        if self.nbytes == 0:
            raise ValueError(f"unsupported exchange size: {max_rows} rows x D={D}")
        self.slot_elems = max_rows * D
        self.timeout_ns = int(timeout_s * 1e9)
        uuid = str(t.cuda.get_device_properties(self.dev).uuid)
        uuids = [None] * self.world
        dist.all_gather_object(uuids, uuid, group=group)
        if len(set(uuids)) != self.world:
            raise RuntimeError("peer exchange needs one GPU per rank; ranks share a device: " + repr(uuids))
        self._own = ctypes.c_void_p()
        self._opened = []
        handle = (ctypes.c_uint8 * HANDLE_BYTES)()
        with t.cuda.device(self.dev):
            check(L.mb_ipc_alloc(self.nbytes, ctypes.byref(self._own), handle), "mb_ipc_alloc")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs, failure = [], None
        try:
            with t.cuda.device(self.dev):
                for q, hq in enumerate(handles):
                    if q == self.rank:
                        ptrs.append(self._own.value)
                        continue
                    p = ctypes.c_void_p()
                    hb = (ctypes.c_uint8 * HANDLE_BYTES).from_buffer_copy(hq)
                    check(L.mb_ipc_open(hb, ctypes.byref(p)), f"mb_ipc_open(rank {q})")
                    self._opened.append(p.value)
                    ptrs.append(p.value)
        except Exception as e:  # reported to every rank below, so all of them raise together
            failure = f"rank {self.rank}: {e}"
        failures = [None] * self.world
        dist.all_gather_object(failures, failure, group=group)
        failures = [f for f in failures if f]
        if failures:
            self.close(barrier=False)
            raise RuntimeError("peer exchange could not map the other ranks' buffers: " + "; ".join(failures))
        self._bufs = (ctypes.c_void_p * self.world)(*ptrs)
        # every row's epoch per exchange kind (MB_PEER_STATE_WORDS each): add_rmsnorm, argmax
        self.state = t.zeros(2 * STATE_WORDS, dtype=t.int32, device=self.dev)
        t.cuda.synchronize(self.dev)
        dist.barrier(group=group)  # every buffer is zeroed and mapped before anyone stores

    def add_rmsnorm(self, partial, x, w, eps: float, h, err, stream: Optional[int] = None):
        """x += fp16(sum over ranks of ``partial``), h = RMSNorm(x) * w (every rank gets
        the same x and h)."""
        N, D = partial.shape
        st = stream_of(self.dev) if stream is None else stream
        check(lib().mb_peer_add_rmsnorm(self._bufs, self.world, self.rank, self.slot_elems, self.timeout_ns,
                                        partial.data_ptr(), x.data_ptr(), w.data_ptr(), N, D, float(eps),
                                        h.data_ptr(), self.state.data_ptr(), err.data_ptr(), st),
              "mb_peer_add_rmsnorm")

    def gemm(self, act, sb, K: int, M: int, err, stream: Optional[int] = None):
        """This rank's row-parallel partial ``act [N, K] x int4 sb [K, M]`` (M = D),
        stored by the GEMM's epilogue straight into every rank's exchange buffer; the
        next call must be ``sum_rmsnorm`` (``mb_int4_gemm_peer``). Returns False, having
        launched nothing, for a shape off the fast GEMM plan."""
        N = act.shape[0]
        st = stream_of(self.dev) if stream is None else stream
        rc = lib().mb_int4_gemm_peer(act.data_ptr(), sb.data_ptr(), N, K, M, self._bufs, self.world, self.rank,
                                     self.slot_elems, self.state.data_ptr(), err.data_ptr(), st)
        if rc == ERR_UNSUPPORTED:
            return False
        check(rc, "mb_int4_gemm_peer")
        return True

    def sum_rmsnorm(self, x, w, eps: float, h, err, stream: Optional[int] = None):
        """The join after ``gemm``: x += fp16(sum over ranks of the stored rows),
        h = RMSNorm(x) * w."""
        N, D = x.shape
        st = stream_of(self.dev) if stream is None else stream
        check(lib().mb_peer_sum_rmsnorm(self._bufs, self.world, self.rank, self.slot_elems, self.timeout_ns,
                                        x.data_ptr(), w.data_ptr(), N, D, float(eps), h.data_ptr(),
                                        self.state.data_ptr(), err.data_ptr(), st),
              "mb_peer_sum_rmsnorm")

    def argmax(self, logits, col0: int, ids, err, stream: Optional[int] = None):
        """ids = the global greedy choice over every rank's column range of the logits."""
        N, V = logits.shape
        st = stream_of(self.dev) if stream is None else stream
        state1 = self.state.data_ptr() + 4 * STATE_WORDS  # the argmax channel's row epochs
        check(lib().mb_peer_argmax(self._bufs, self.world, self.rank, self.slot_elems, self.timeout_ns,
                                   logits.data_ptr(), N, V, int(col0), ids.data_ptr(), state1, err.data_ptr(), st),
              "mb_peer_argmax")

    def close(self, barrier: bool = True):
        """Unmap the peers' buffers and free this rank's (after every rank has finished
        its exchanges: a barrier on both sides)."""
        import torch.distributed as dist
        t = _lib.torch()
        L = lib()
        t.cuda.synchronize(self.dev)
        if barrier:
            dist.barrier(group=self.group)
        with t.cuda.device(self.dev):
            for p in self._opened:
                L.mb_ipc_close(ctypes.c_void_p(p))
            self._opened = []
            if barrier:
                dist.barrier(group=self.group)
            if self._own.value:
                L.mb_ipc_free(self._own)
                self._own = ctypes.c_void_p()


__all__ = ["PeerExchange", "DEVERR_TIMEOUT"]
