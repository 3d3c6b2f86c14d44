"""INT4 decoder step: decode of N parallel traces through a LLaMA-style model.

The model is the reference's ``TinyLlamaModel`` architecture
(``antigravity-engine/src/transformer.py:161-225``: RMSNorm, RoPE, attention with a
KV cache, SwiGLU MLP, final RMSNorm, LM head) with every linear weight stored as the
reference's 144-byte INT4 super-block stream and run by ``mb_int4_gemm``, the
attention over the growing cache run by ``mb_decode_attn_cache`` with the exp-LUT
softmax the reference's decode path uses (``batch_generator.py:226,234``), and greedy
token choice by ``mb_argmax_f16`` (``batch_generator.py:203-206``).

Shapes default to BASELINE config 5 (Qwen-1.5B-like: 24 layers, hidden 2048, 16 heads
x 128, FFN 5504, vocab 151936, multi-head attention). Layout per layer, with
``out = x @ W`` for a row-major ``[K, M]`` weight:

* ``wqkv [D, 3D]`` (q | k | v), ``wo [D, D]``, ``wgu [D, 2F]`` (gate | up),
  ``wd [F, D]``; ``lm_head [D, V]``; RMSNorm weights fp32; embedding fp16 ``[V, D]``.
* KV caches ``[N, H, max_len, head_dim]`` fp16 per layer.

The residual stream stays fp32; each GEMM input is rounded to fp16 once.

Tensor parallelism (``rank``/``world``, one process per GPU): the Megatron split of
``tp_shards``. q/k/v columns, o_proj rows and the KV cache of a head range; gate/up
columns and down rows of an FFN range; lm_head columns of a vocabulary range. Every
rank draws the whole weights from the same random stream as one GPU and keeps its
slice, so the shards hold exactly the one-GPU model's codes and scales. The two
row-parallel partial products of a layer are joined by ``exchange="peer"`` (the
default: the o_proj and down GEMMs store their rows into every rank's exchange buffer
from their epilogue, ``mb_int4_gemm_peer``, and one kernel per join waits for the
other ranks' rows over NVLink, then does the residual add and RMSNorm;
``fused_join=False`` keeps the GEMM's partial in HBM and lets the join kernel store
it) or ``"nccl"`` (``all_reduce``, then ``mb_add_rmsnorm``); the greedy choice over
the split vocabulary is one 64-bit key per shard, maximised across ranks.

``temperature > 0`` replaces the greedy choice by ``mb_sample_tokens``: a draw from
the top-50 of the exp-LUT softmax of the scaled logits, as the reference's
``sample_tokens`` (``batch_generator.py:187-253``), with the random stream's counter
on the device so the captured step keeps drawing fresh values; ``logprobs`` holds
each trace's log-probability of its token. Tensor-parallel ranks all-gather their
vocabulary shards (NCCL) and draw with the same seed and counter, so every rank picks
the same token.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check, lib, stream_of


_STORED = object()  # a row-parallel partial that its GEMM stored into the exchange buffers


@dataclass
class DecoderConfig:
    layers: int = 24
    hidden: int = 2048
    heads: int = 16
    head_dim: int = 128
    ffn: int = 5504
    vocab: int = 151936
    eps: float = 1e-6
    theta: float = 10000.0
    lut_range: float = 16.0
    max_len: int = 768


def rope_table(head_dim: int, max_len: int, theta: float):
    """(cos, sin) pairs [max_len, head_dim/2, 2] fp32, computed the way
    ``precompute_freqs_cis`` does (``transformer.py:39-44``: fp32 frequencies,
    ``torch.polar`` in complex64)."""
    t = _lib.torch()
    freqs = 1.0 / (theta ** (t.arange(0, head_dim, 2, dtype=t.float32) / head_dim))
    pos = t.arange(max_len, dtype=t.float32)
    ang = t.outer(pos, freqs)
    cis = t.polar(t.ones_like(ang), ang)
    return t.view_as_real(cis).contiguous()


def tp_shards(cfg: DecoderConfig, world: int):
    """Megatron split of the decoder over ``world`` GPUs: per rank its head range
    (q/k/v columns, o_proj rows, KV cache), its FFN range (gate/up columns, down rows)
    and its vocabulary range (lm_head columns). FFN and vocabulary ranges are cut on
    128-column boundaries where the size allows (whole quantization groups, and widths
    the fast GEMM plan takes), else on 32-column group boundaries."""
    from .dist import column_bounds, head_bounds

    def cols(M):
        if world == 1:
            return [(0, M)]
        return column_bounds(M, world, group=128 if M % 128 == 0 and M // 128 >= world else 32)

    return {"heads": head_bounds(cfg.heads, world), "ffn": cols(cfg.ffn), "vocab": cols(cfg.vocab)}


def lm_head_cols(vocab_range: int) -> int:
    """Stored width of an LM-head vocabulary range: a range of an odd number of
    128-column blocks gets 128 zero-weight columns, so that its GEMM runs in 256-column
    strips (a 128-wide strip takes a wave as long as a 256-wide one, so the wider strip
    halves the waves); any other range is stored as it is."""
    return vocab_range + 128 if vocab_range % 256 == 128 else vocab_range


class Int4Decoder:
    """Random-init INT4 decoder for N traces decoding in lockstep, on one GPU or
    tensor-parallel over ``world`` GPUs (this process being ``rank``)."""

    def __init__(self, cfg: DecoderConfig, n_traces: int, device="cuda:0", seed: int = 0, std: float = 0.02,
                 keep_dense: bool = False, rank: int = 0, world: int = 1, group=None, exchange: str = "peer",
                 exchange_timeout_s: float = 10.0, temperature: float = 0.0, sample_seed: int = 0,
                 fused_join: bool = True):
        t = _lib.require_cuda()
        from .attention import ExponentialLUT
        from .dequant import quantize_to_superblocks
        self.cfg, self.N = cfg, n_traces
        self.dev = t.device(device)
        D, H, dh, F, V = cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.vocab
        if H * dh != D:
            raise ValueError("heads * head_dim must equal hidden")
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
        self.rank, self.world, self.group = rank, world, group
        self.exchange, self.peer, self.exchange_timeout_s = exchange, None, exchange_timeout_s
        self.fused_join = bool(fused_join) and world > 1 and exchange == "peer"
        self.temperature = float(temperature)
        self.shards = tp_shards(cfg, world)
        sh = {k: v[rank] for k, v in self.shards.items()}
        (h0, h1), (f0, f1), (v0, v1) = sh["heads"], sh["ffn"], sh["vocab"]
        self.Hl, self.Fl, self.Vl, self.v0 = h1 - h0, f1 - f0, v1 - v0, v0
        Hl, Fl, Vl = self.Hl, self.Fl, self.Vl
        Dl = Hl * dh
        self.head_range = (h0, h1)
        g = t.Generator(device=self.dev)
        g.manual_seed(seed)
        self.dense = [] if keep_dense else None

        def int4(K, M, cols=None, rows=None, pad=0):
            # the whole [K, M] weight is drawn on every rank (the same random stream as
            # one GPU), then this rank's columns / rows are quantized: whole 32-wide
            # groups, so its codes and scales equal the unsplit weight's; `pad` zero
            # columns appended after them leave those codes and scales unchanged too
            w = t.randn((K, M), generator=g, device=self.dev, dtype=t.float32) * std
            if self.dense is not None:
                self.dense.append(w.cpu())
            if cols is not None and world > 1:
                w = t.cat([w[:, c0:c1] for c0, c1 in cols], dim=1)
            if rows is not None and world > 1:
                w = w[rows[0]:rows[1]]
            if pad:
                w = t.cat([w, t.zeros((w.shape[0], pad), device=self.dev, dtype=w.dtype)], dim=1)
            sb = quantize_to_superblocks(w.contiguous().reshape(-1))
            del w
            return sb

        qkv_cols = [(j * D + h0 * dh, j * D + h1 * dh) for j in range(3)]
        gu_cols = [(f0, f1), (F + f0, F + f1)]
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "wqkv": int4(D, 3 * D, cols=qkv_cols), "wo": int4(D, D, rows=(h0 * dh, h1 * dh)),
                "wgu": int4(D, 2 * F, cols=gu_cols), "wd": int4(F, D, rows=(f0, f1)),
                "attn_norm": (1.0 + 0.02 * t.randn((D,), generator=g, device=self.dev)).float(),
                "ffn_norm": (1.0 + 0.02 * t.randn((D,), generator=g, device=self.dev)).float(),
            })
        self.final_norm = (1.0 + 0.02 * t.randn((D,), generator=g, device=self.dev)).float()
        # the LM head in 256-column strips (151,936 = 1187 x 128 -> 152,064 columns); its
        # logits are copied back to the range's own width
        self.lm_cols = lm_head_cols(Vl)
        self.lm_head = int4(D, V, cols=[(v0, v1)], pad=self.lm_cols - Vl)
        self.embed = (t.randn((V, D), generator=g, device=self.dev) * std).half()
        self.cs = rope_table(dh, cfg.max_len, cfg.theta).to(self.dev)
        self.lut = ExponentialLUT(range_max=cfg.lut_range)
        self.table = self.lut.device_table(self.dev)
        N, L = n_traces, cfg.max_len
        self.k_cache = [t.zeros((N, Hl, L, dh), dtype=t.float16, device=self.dev) for _ in range(cfg.layers)]
        self.v_cache = [t.zeros((N, Hl, L, dh), dtype=t.float16, device=self.dev) for _ in range(cfg.layers)]
        f16, f32 = t.float16, t.float32
        self.x = t.empty((N, D), dtype=f32, device=self.dev)
        self.h = t.empty((N, D), dtype=f16, device=self.dev)
        self.qkv = t.empty((N, 3 * Dl), dtype=f16, device=self.dev)
        self.q = t.empty((N, Hl, dh), dtype=f16, device=self.dev)
        self.att = t.empty((N, Hl, dh), dtype=f16, device=self.dev)
        self.o = t.empty((N, D), dtype=f16, device=self.dev)
        self.gu = t.empty((N, 2 * Fl), dtype=f16, device=self.dev)
        self.a = t.empty((N, Fl), dtype=f16, device=self.dev)
        self.logits = t.empty((N, Vl), dtype=f16, device=self.dev)
        self.logits_lm = (self.logits if self.lm_cols == Vl
                          else t.empty((N, self.lm_cols), dtype=f16, device=self.dev))
        self.keys = t.zeros((N,), dtype=t.int64, device=self.dev)
        self.ids = t.zeros((N,), dtype=t.int32, device=self.dev)
        self.logprobs = t.zeros((N,), dtype=t.float32, device=self.dev)
        self.pos = t.zeros((N,), dtype=t.int32, device=self.dev)
        self.err = t.zeros((1,), dtype=t.int32, device=self.dev)
        self.sampler = None
        if self.temperature > 0:  # top-50 draw from the LUT softmax (range 10), device random stream
            from .sampling import BatchSampler
            self.sampler = BatchSampler(n_traces, V, device=self.dev, seed=sample_seed)
            if world > 1:  # the vocabulary shards are gathered; every rank draws the same token
                vmax = max(c1 - c0 for c0, c1 in self.shards["vocab"])
                self.logits_pad = t.zeros((N, vmax), dtype=f16, device=self.dev)
                self.logits_all = t.empty((world * N, vmax), dtype=f16, device=self.dev)
                self.logits_full = t.empty((N, V), dtype=f16, device=self.dev)
        self.length = 0  # positions filled so far (the same for every trace)
        self.graph = None
        nb = int(lib().mb_decode_attn_workspace_size(N, Hl, L, dh))
        self.ws = t.zeros(nb, dtype=t.uint8, device=self.dev)
        self.scale = float(np.float32(1.0 / np.sqrt(dh)))

    # -------------------------------------------------------------------------
    def fill_prompt_cache(self, length: int, seed: int = 1):
        """Seeded N(0,1) keys and values for the first ``length`` positions of every
        layer (a stand-in for the prompt's prefill; decode speed does not depend on the
        cache contents), and sets the next position to ``length``. A tensor-parallel
        rank draws every head as one GPU does and keeps its own heads."""
        t = _lib.torch()
        if not 0 <= length < self.cfg.max_len:
            raise ValueError("prompt length must leave room to decode")
        g = t.Generator(device=self.dev)
        g.manual_seed(seed)
        h0, h1 = self.head_range
        full = None
        if self.world > 1:
            cfg = self.cfg
            full = t.zeros((self.N, cfg.heads, cfg.max_len, cfg.head_dim), dtype=t.float16, device=self.dev)
        for kc, vc in zip(self.k_cache, self.v_cache):
            for c in (kc, vc):
                if full is None:
                    c[:, :, :length].normal_(generator=g)
                else:
                    full[:, :, :length].normal_(generator=g)
                    c.copy_(full[:, h0:h1])
        self.length = length
        self.pos.fill_(length)

    def prefill(self, prompt_ids):
        """Run a prompt through the decoder one position at a time, as the reference's
        engine does (``transformer_engine.mm:846-881``: every prompt token goes through
        the decode step, its keys and values land in the cache, and the last position's
        logits give the first generated token). ``prompt_ids``: int32 ``[N, P]`` on the
        device. The first position runs eagerly (it caches GEMM plans and tensor maps),
        the rest replay the captured step with the prompt token copied into
        ``self.ids`` before each replay. Leaves the first generated ids in ``self.ids``
        and ``P`` positions in the cache."""
        t = _lib.torch()
        if prompt_ids.dim() != 2 or prompt_ids.shape[0] != self.N:
            raise ValueError(f"prompt ids must be [{self.N}, P]")
        P = int(prompt_ids.shape[1])
        if self.length + P >= self.cfg.max_len:
            raise ValueError("prompt does not fit the KV cache")
        ids = prompt_ids.to(device=self.dev, dtype=t.int32)
        for p in range(P):
            if p == 0:
                self.step(ids[:, 0].contiguous())
                self.capture()
                continue
            self.ids.copy_(ids[:, p])
            self.step_graphed()
        return self.ids

    def cache_snapshot(self, length=None):
        """Host copies of the first ``length`` cached positions of every layer (keys,
        values), to rewind the decoder with ``restore_cache``."""
        n = self.length if length is None else length
        return ([k[:, :, :n].cpu() for k in self.k_cache], [v[:, :, :n].cpu() for v in self.v_cache], n)

    def restore_cache(self, snap):
        """Rewind to a ``cache_snapshot``: its positions are written back, the next
        position is its length on the host and on the device."""
        ks, vs, n = snap
        for dst, src in zip(self.k_cache, ks):
            dst[:, :, :n].copy_(src)
        for dst, src in zip(self.v_cache, vs):
            dst[:, :, :n].copy_(src)
        self.length = n
        self.pos.fill_(n)

    def dense_weights(self):
        """The model with every INT4 stream dequantized (bit-exact fp16 values, as fp32
        CPU tensors ``[K, M]``) and the fp32 norms, embedding and RoPE factors on the
        host: the inputs of a reference-style CPU forward. One GPU only."""
        t = _lib.torch()
        from .dequant import unpack_superblock_weights
        if self.world != 1:
            raise ValueError("dense_weights needs the whole model (world = 1)")
        cfg = self.cfg
        D, F, V = cfg.hidden, cfg.ffn, cfg.vocab

        def deq(sb, K, M):
            return unpack_superblock_weights(sb, K * M // 256).reshape(K, M).float().cpu()

        layers = [{"wqkv": deq(lw["wqkv"], D, 3 * D), "wo": deq(lw["wo"], D, D), "wgu": deq(lw["wgu"], D, 2 * F),
                   "wd": deq(lw["wd"], F, D), "attn_norm": lw["attn_norm"].cpu(), "ffn_norm": lw["ffn_norm"].cpu()}
                  for lw in self.layers]
        return {"layers": layers, "final_norm": self.final_norm.cpu(),
                "lm_head": deq(self.lm_head, D, self.lm_cols)[:, :V].contiguous(),
                "embed": self.embed.float().cpu(), "cis": t.view_as_complex(self.cs.cpu().contiguous())}

    def step(self, ids):
        """One decode step for all traces: token ids [N] (int32, device) in, the next
        ids [N] out (a device tensor, also kept in ``self.ids``)."""
        if self.length >= self.cfg.max_len:
            raise ValueError("KV cache is full")
        self._enqueue(ids, device_lengths=False)
        self.length += 1
        return self.ids

    def capture(self):
        """Capture one decode step (reading ``self.ids``, writing the next ids back into
        it) as a CUDA graph; the attention reads its length from the device positions,
        so the graph replays unchanged while the cache grows. Run one eager step first
        (plans and tensor maps are cached on the first call of each shape)."""
        t = _lib.torch()
        self._ensure_exchange()
        g = t.cuda.CUDAGraph()
        side = t.cuda.Stream(device=self.dev)
        side.wait_stream(t.cuda.current_stream(self.dev))
        with t.cuda.stream(side):
            with t.cuda.graph(g, stream=side):
                self._enqueue(self.ids, device_lengths=True)
        t.cuda.current_stream(self.dev).wait_stream(side)
        self.graph = g
        return g

    def step_graphed(self):
        """Replay the captured step: consumes ``self.ids``, leaves the next ids there."""
        if self.length >= self.cfg.max_len:
            raise ValueError("KV cache is full")
        self.graph.replay()
        self.length += 1
        return self.ids

    def _ensure_exchange(self):
        """Map the other ranks' exchange buffers (a collective: every rank's first step
        or capture makes it)."""
        if self.world > 1 and self.exchange == "peer" and self.peer is None:
            from .peer import PeerExchange
            self.peer = PeerExchange(self.N, self.cfg.hidden, self.dev, group=self.group,
                                     timeout_s=self.exchange_timeout_s)

    def close(self):
        """Release the captured graph and the exchange buffers (before the process group
        is destroyed)."""
        t = _lib.torch()
        self.graph = None
        t.cuda.synchronize(self.dev)
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _row_parallel(self, act, w, K, st):
        """This rank's partial of a row-parallel projection (o_proj, down). With the
        fused join the GEMM's epilogue stores it into the exchange buffers and the
        marker ``_STORED`` is returned; otherwise it lands in ``self.o``."""
        if self.fused_join and self.peer.gemm(act, w, K, self.cfg.hidden, self.err, st):
            return _STORED
        check(lib().mb_int4_gemm(act.data_ptr(), w.data_ptr(), self.o.data_ptr(), self.N, K, self.cfg.hidden,
                                 self.err.data_ptr(), st), "row-parallel GEMM")
        return self.o

    def _residual_norm(self, y, w, st):
        """x += y (the sum over ranks of the row-parallel partials y), h = RMSNorm(x) * w."""
        cfg, N, L = self.cfg, self.N, lib()
        p = lambda x: x.data_ptr()  # noqa: E731
        if y is _STORED:  # every rank's rows are in the exchange buffers already
            self.peer.sum_rmsnorm(self.x, w, cfg.eps, self.h, self.err, st)
            return
        if y is not None and self.world > 1:
            if self.exchange == "peer":
                self.peer.add_rmsnorm(y, self.x, w, cfg.eps, self.h, self.err, st)
                return
            import torch.distributed as dist
            dist.all_reduce(y, group=self.group)
        check(L.mb_add_rmsnorm(p(self.x), None if y is None else p(y), p(w), N, cfg.hidden, cfg.eps, p(self.h), st),
              "mb_add_rmsnorm")

    def _enqueue(self, ids, device_lengths: bool):
        cfg, N, L = self.cfg, self.N, lib()
        D, dh = cfg.hidden, cfg.head_dim
        H, F, V = self.Hl, self.Fl, self.Vl  # this rank's heads, FFN columns, vocabulary columns
        Dl = H * dh
        self._ensure_exchange()
        st = stream_of(self.dev)
        p = lambda x: x.data_ptr()  # noqa: E731
        err = p(self.err)
        check(L.mb_embed(p(ids), N, p(self.embed), cfg.vocab, D, p(self.x), err, st), "mb_embed")
        y = None
        for li, lw in enumerate(self.layers):
            self._residual_norm(y, lw["attn_norm"], st)
            check(L.mb_int4_gemm(p(self.h), p(lw["wqkv"]), p(self.qkv), N, D, 3 * Dl, err, st), "qkv")
            check(L.mb_rope_append(p(self.qkv), N, H, dh, p(self.pos), p(self.cs), cfg.max_len, p(self.q),
                                   p(self.k_cache[li]), p(self.v_cache[li]), err, st), "mb_rope_append")
            if device_lengths:  # length = position + 1, read on the device
                check(L.mb_decode_attn_cache_lens(p(self.q), p(self.k_cache[li]), p(self.v_cache[li]), p(self.att),
                                                  N, H, cfg.max_len, dh, p(self.pos), 1, self.scale, p(self.table),
                                                  self.lut.size, float(self.lut.range_max), p(self.ws),
                                                  self.ws.numel(), st), "mb_decode_attn_cache_lens")
            else:
                check(L.mb_decode_attn_cache(p(self.q), p(self.k_cache[li]), p(self.v_cache[li]), p(self.att), N, H,
                                             self.length + 1, cfg.max_len, dh, self.scale, p(self.table),
                                             self.lut.size, float(self.lut.range_max), p(self.ws), self.ws.numel(),
                                             st), "mb_decode_attn_cache")
            y = self._row_parallel(self.att, lw["wo"], Dl, st)  # o_proj
            self._residual_norm(y, lw["ffn_norm"], st)  # row-parallel o_proj joined over ranks
            check(L.mb_int4_gemm(p(self.h), p(lw["wgu"]), p(self.gu), N, D, 2 * F, err, st), "gate_up")
            check(L.mb_swiglu(p(self.gu), N, F, p(self.a), st), "mb_swiglu")
            y = self._row_parallel(self.a, lw["wd"], F, st)  # down, joined by the next norm
        self._residual_norm(y, self.final_norm, st)
        check(L.mb_int4_gemm(p(self.h), p(self.lm_head), p(self.logits_lm), N, D, self.lm_cols, err, st), "lm_head")
        if self.logits_lm is not self.logits:  # the padded columns dropped
            self.logits.copy_(self.logits_lm[:, :V])
        if self.sampler is not None:
            src = self.logits
            if self.world > 1:  # all-gather the shards into the whole row on every rank
                import torch.distributed as dist
                vmax = self.logits_pad.shape[1]
                self.logits_pad[:, :V].copy_(self.logits)
                dist.all_gather_into_tensor(self.logits_all, self.logits_pad, group=self.group)
                allv = self.logits_all.view(self.world, N, vmax)
                for r, (c0, c1) in enumerate(self.shards["vocab"]):
                    self.logits_full[:, c0:c1].copy_(allv[r, :, :c1 - c0])
                src = self.logits_full
            self.sampler.sample(src, self.temperature, tokens=self.ids, logprobs=self.logprobs, err=self.err,
                                stream=st)
        elif self.world == 1:
            check(L.mb_argmax_f16(p(self.logits), N, V, p(self.ids), st), "mb_argmax_f16")
        elif self.exchange == "peer":  # per-shard keys exchanged over NVLink, max -> ids, one kernel
            self.peer.argmax(self.logits, self.v0, self.ids, self.err, st)
        else:  # per-shard keys, one int64 MAX all-reduce, keys -> ids
            import torch.distributed as dist
            check(L.mb_argmax_key_f16(p(self.logits), N, V, self.v0, p(self.keys), st), "mb_argmax_key_f16")
            dist.all_reduce(self.keys, op=dist.ReduceOp.MAX, group=self.group)
            check(L.mb_argmax_keys_to_ids(p(self.keys), N, p(self.ids), st), "mb_argmax_keys_to_ids")
        check(L.mb_advance_positions(p(self.pos), N, st), "mb_advance_positions")

    def generate(self, first_ids, steps: int):
        """Decode ``steps`` tokens from ``first_ids`` [N]; returns [steps, N] ids
        (device, int32)."""
        t = _lib.torch()
        out = t.empty((steps, self.N), dtype=t.int32, device=self.dev)
        ids = first_ids
        for s in range(steps):
            ids = self.step(ids)
            out[s].copy_(ids)
        return out


def timed_decode(dec: Int4Decoder, steps: int, warmup: int = 3, graph: bool = True) -> float:
    """Milliseconds per decode step, CUDA-event timed on this rank after ``warmup``
    steps (one eager step first, which caches the GEMM plans and tensor maps, then the
    step captured as a CUDA graph unless ``graph`` is False); the maximum over ranks
    when the decoder is tensor-parallel."""
    t = _lib.torch()
    dec.step(dec.ids)
    if dec.world > 1:  # every rank learns whether an exchange wait expired before timing
        import torch.distributed as dist
        e = dec.err.clone()
        dist.all_reduce(e, op=dist.ReduceOp.MAX, group=dec.group)
        if int(e.item()) & 1:
            raise RuntimeError("tensor-parallel exchange timed out on the first step (device error word %d)"
                               % int(e.item()))
    if graph:
        dec.capture()
    step = dec.step_graphed if graph else (lambda: dec.step(dec.ids))
    for _ in range(warmup):
        step()
    t.cuda.synchronize()
    if dec.world > 1:
        import torch.distributed as dist
        dist.barrier(group=dec.group)
        t.cuda.synchronize()
    e0, e1 = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    t.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if dec.world > 1:
        import torch.distributed as dist
        m = t.tensor([ms], dtype=t.float64, device=dec.dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=dec.group)
        ms = float(m.item())
    return ms


__all__ = ["DecoderConfig", "Int4Decoder", "rope_table", "timed_decode", "tp_shards"]
