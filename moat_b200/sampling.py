"""Batched token sampling on the GPU with the exp-LUT softmax.

Drop-in for ``BatchedRolloutCoordinator.sample_tokens(logits_batch, temperature=0.7,
top_p=0.9)`` (``antigravity-engine/src/batch_generator.py:187-253``, NumPy branch): N
rows of logits in, ``(token_ids, logprobs)`` out, greedy for ``temperature <= 0``,
otherwise a draw from the top-50 of the LUT softmax (``safe_softmax_lut`` with a
32,768-entry table over [-10, 0]) of the temperature-scaled logits. As in that branch,
``top_p`` is accepted and not used. The whole choice runs in one kernel
(``mb_sample_tokens``); the random draws come from a counter-based stream on the
device (``seed`` plus a counter the kernel advances), or are passed in as
``uniforms``. Token ids are int32, log-probabilities float32 (the greedy branch's fp16
value widened).
"""

from __future__ import annotations

from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, lib, stream_of

TOP_K = 50
DEVERR_NONFINITE = 4


class BatchSampler:
    """Device state for repeated sampling of [N, V] logits on one GPU: the exp table,
    the index workspace, the random-stream counter and the output buffers. Calls are
    capturable in a CUDA graph (the counter lives on the device)."""

    def __init__(self, N: int, V: int, device="cuda", seed: int = 0, range_max: float = 10.0, size: int = 32768,
                 top_k: int = TOP_K):
        t = _lib.require_cuda()
        from .attention import ExponentialLUT
        self.dev = t.device(device)
        if self.dev.index is None:
            self.dev = t.device("cuda", t.cuda.current_device())
        self.N, self.V, self.seed, self.top_k = N, V, int(seed) & 0xFFFFFFFFFFFFFFFF, top_k
        self.lut = ExponentialLUT(size=size, range_max=range_max)
        self.table = self.lut.device_table(self.dev)
        nb = int(lib().mb_sample_workspace_size(N, V))
        self.ws = t.empty(max(nb, 256), dtype=t.uint8, device=self.dev)
        self.rng_state = t.zeros(2, dtype=t.int32, device=self.dev)
        self.tokens = t.empty(N, dtype=t.int32, device=self.dev)
        self.logprobs = t.empty(N, dtype=t.float32, device=self.dev)
        self.err = t.zeros(1, dtype=t.int32, device=self.dev)

    def sample(self, logits, temperature: float, uniforms=None, tokens=None, logprobs=None, err=None,
               stream: Optional[int] = None):
        """Sample one token per row of ``logits`` (CUDA fp16 or fp32 [N, V]); returns the
        device (tokens, logprobs), by default this sampler's buffers."""
        t = _lib.torch()
        if logits.dtype not in (t.float16, t.float32) or tuple(logits.shape) != (self.N, self.V):
            raise ValueError(f"logits must be fp16/fp32 [{self.N}, {self.V}]")
        logits = logits.contiguous()
        tokens = self.tokens if tokens is None else tokens
        logprobs = self.logprobs if logprobs is None else logprobs
        err = self.err if err is None else err
        u = None if uniforms is None else uniforms.data_ptr()
        st = stream_of(self.dev) if stream is None else stream
        check(lib().mb_sample_tokens(logits.data_ptr(), 1 if logits.dtype == t.float32 else 0, self.N, self.V,
                                     float(temperature), self.top_k, self.table.data_ptr(), self.lut.size,
                                     float(self.lut.range_max), u, self.seed, self.rng_state.data_ptr(),
                                     tokens.data_ptr(), logprobs.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                                     err.data_ptr(), st), "mb_sample_tokens")
        return tokens, logprobs


def sample_tokens(logits_batch, temperature: float = 0.7, top_p: float = 0.9, *, seed: int = 0,
                  uniforms=None, top_k: int = TOP_K):
    """``sample_tokens`` of the reference: (token_ids [N] int32, logprobs [N] float32).

    NumPy input gives NumPy output (the rows are copied to the GPU; float64 logits are
    rounded to float32 first); a CUDA tensor gives CUDA tensors. ``uniforms`` (N values
    in [0, 1)) replaces the device random stream; ``seed`` seeds it otherwise. A row
    whose scaled maximum is not finite raises, as the reference does."""
    t = _lib.require_cuda()
    was_np = not isinstance(logits_batch, t.Tensor)
    if was_np:
        a = np.asarray(logits_batch)
        if a.dtype not in (np.float16, np.float32):
            a = a.astype(np.float32)
        x = t.from_numpy(np.ascontiguousarray(a)).cuda()
    else:
        x = logits_batch if logits_batch.is_cuda else logits_batch.cuda()
        if x.dtype not in (t.float16, t.float32):
            x = x.float()
    if x.dim() != 2:
        raise ValueError("logits_batch must be [N, V]")
    N, V = x.shape
    s = BatchSampler(N, V, device=x.device, seed=seed, top_k=top_k)
    u = None
    if uniforms is not None:
        u = t.as_tensor(np.asarray(uniforms, dtype=np.float32) if not isinstance(uniforms, t.Tensor) else uniforms,
                        dtype=t.float32).to(x.device).contiguous()
    tok, lp = s.sample(x, temperature, uniforms=u)
    if int(s.err.item()) & DEVERR_NONFINITE:
        raise FloatingPointError("sample_tokens: a row's scaled maximum logit is not finite")
    if was_np:
        return tok.cpu().numpy(), lp.cpu().numpy()
    return tok, lp


__all__ = ["BatchSampler", "sample_tokens", "TOP_K"]
