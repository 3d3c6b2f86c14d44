"""CPU restatement of the reference's decoder forward for N traces decoding in lockstep.

Test infrastructure and the CPU baseline of the decode bench only (see
``oracle/__init__.py``): nothing in ``moat_b200`` imports it. The model is the
reference's LLaMA block stack, ``antigravity-engine/src/transformer.py``, in fp32 torch
on the host cores, one token per trace per step with a KV cache:

* ``RMSNorm`` :26-37: ``x * rsqrt(mean(x^2) + eps) * weight`` in fp32;
* ``precompute_freqs_cis`` :39-44 / ``apply_rotary_emb`` :47-63: adjacent (even, odd)
  pairs of q and k rotated as complex numbers by the position's ``torch.polar``
  factor; the cache holds the rotated keys (:98-103);
* ``Attention.forward`` :85-122 with as many KV heads as query heads (BASELINE
  config 5 names no KV-head count): ``q k^T / sqrt(d)``, softmax, ``@ v``, o_proj;
* ``SwiGLUMLP`` :125-135: ``down(silu(gate x) * up x)``;
* ``TransformerBlock`` :137-158 and ``TinyLlamaModel.forward`` :200-220: embedding,
  blocks with two residual adds, final norm, LM head; greedy choice ``argmax``
  (``transformer.py:322``, ``batch_generator.py:224``).

The softmax is the reference's exact ``F.softmax`` (:117) or, with
``softmax="lut"``, the exp-table ``safe_softmax_lut`` its batched decode path applies
to attention scores (``batch_generator.py:226``; ``antigravity-engine/src/attention.py:
97-134``, restated in ``oracle/attention.py``).

Weights are dense fp32 tensors ``[K, M]`` (``out = x @ W``): the caller dequantizes the
INT4 super-block streams (bit-exact with ``oracle.int4.unpack_superblock_weights``).
"""

from __future__ import annotations

import math

import numpy as np


class CpuDecoder:
    """fp32 CPU decoder. ``layers``: list of dicts with ``wqkv [D, 3D]``, ``wo [D, D]``,
    ``wgu [D, 2F]`` (gate | up), ``wd [F, D]``, ``attn_norm [D]``, ``ffn_norm [D]``;
    ``final_norm [D]``, ``lm_head [D, V]``, ``embed [V, D]``; ``cis`` complex64
    ``[max_len, head_dim/2]`` RoPE factors."""

    def __init__(self, layers, final_norm, lm_head, embed, cis, heads: int, n_traces: int, max_len: int,
                 eps: float = 1e-6, softmax: str = "exact", lut=None, lut_range: float = 16.0):
        import torch
        if softmax not in ("exact", "lut"):
            raise ValueError("softmax must be 'exact' or 'lut'")
        self.torch = torch
        self.layers, self.final_norm, self.lm_head, self.embed, self.cis = layers, final_norm, lm_head, embed, cis
        self.D = embed.shape[1]
        self.H = heads
        self.dh = self.D // heads
        self.N, self.max_len, self.eps = n_traces, max_len, eps
        self.softmax, self.lut, self.lut_range = softmax, lut, lut_range
        shape = (n_traces, heads, max_len, self.dh)
        self.k_cache = [torch.zeros(shape, dtype=torch.float32) for _ in layers]
        self.v_cache = [torch.zeros(shape, dtype=torch.float32) for _ in layers]
        self.length = 0

    def load_cache(self, k_caches, v_caches, length: int):
        """Start from ``length`` cached positions (``[N, H, >= length, dh]`` tensors of
        any float dtype, one pair per layer)."""
        for dst, src in zip(self.k_cache, k_caches):
            dst[:, :, :length] = src[:, :, :length].float()
        for dst, src in zip(self.v_cache, v_caches):
            dst[:, :, :length] = src[:, :, :length].float()
        self.length = length

    def _rms(self, x, w):
        t = self.torch
        return x * t.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * w

    def _softmax(self, s):
        t = self.torch
        if self.softmax == "exact":
            return t.softmax(s, dim=-1)
        from . import attention as OA
        return t.from_numpy(OA.safe_softmax_lut(s.numpy(), self.lut, self.lut_range).astype(np.float32))

    def step(self, ids):
        """One step: token ids ``[N]`` in, fp32 logits ``[N, V]`` out; appends this
        position's keys and values to the cache."""
        t = self.torch
        N, H, dh, D, pos = self.N, self.H, self.dh, self.D, self.length
        if pos >= self.max_len:
            raise ValueError("KV cache is full")
        x = self.embed[t.as_tensor(ids).long()].float()
        rot = self.cis[pos]
        scale = 1.0 / math.sqrt(dh)
        for li, lw in enumerate(self.layers):
            h = self._rms(x, lw["attn_norm"])
            qkv = (h @ lw["wqkv"]).reshape(N, 3, H, dh)
            q = t.view_as_real(t.view_as_complex(qkv[:, 0].reshape(N, H, dh // 2, 2).contiguous()) * rot)
            k = t.view_as_real(t.view_as_complex(qkv[:, 1].reshape(N, H, dh // 2, 2).contiguous()) * rot)
            kc, vc = self.k_cache[li], self.v_cache[li]
            kc[:, :, pos] = k.reshape(N, H, dh)
            vc[:, :, pos] = qkv[:, 2]
            s = t.einsum("nhd,nhld->nhl", q.reshape(N, H, dh), kc[:, :, :pos + 1]) * scale
            att = t.einsum("nhl,nhld->nhd", self._softmax(s), vc[:, :, :pos + 1]).reshape(N, D)
            x = x + att @ lw["wo"]
            h = self._rms(x, lw["ffn_norm"])
            gu = h @ lw["wgu"]
            F = gu.shape[1] // 2
            x = x + (t.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ lw["wd"]
        self.length = pos + 1
        return self._rms(x, self.final_norm) @ self.lm_head


def argmax_agreement(a, b) -> float:
    """Fraction of equal entries of two id arrays of one shape."""
    a, b = np.asarray(a), np.asarray(b)
    return float(np.mean(a == b)) if a.size else 1.0
