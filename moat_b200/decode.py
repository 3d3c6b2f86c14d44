"""INT4 decoder step: greedy decode of N parallel traces through a LLaMA-style model.

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
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check, lib, stream_of


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


class Int4Decoder:
    """Random-init INT4 decoder on one GPU, for N traces decoding in lockstep."""

    def __init__(self, cfg: DecoderConfig, n_traces: int, device="cuda:0", seed: int = 0, std: float = 0.02,
                 keep_dense: bool = False):
        t = _lib.require_cuda()
        from .attention import ExponentialLUT
        from .dequant import quantize_to_superblocks
        self.cfg, self.N = cfg, n_traces
        self.dev = t.device(device)
        D, H, dh, F, V = cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.vocab
        if H * dh != D:
            raise ValueError("heads * head_dim must equal hidden")
        g = t.Generator(device=self.dev)
        g.manual_seed(seed)
        self.dense = [] if keep_dense else None

        def int4(K, M):
            w = t.randn((K, M), generator=g, device=self.dev, dtype=t.float32) * std
            if self.dense is not None:
                self.dense.append(w.cpu())
            sb = quantize_to_superblocks(w.reshape(-1))
            del w
            return sb

        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "wqkv": int4(D, 3 * D), "wo": int4(D, D), "wgu": int4(D, 2 * F), "wd": int4(F, D),
                "attn_norm": (1.0 + 0.02 * t.randn((D,), generator=g, device=self.dev)).float(),
                "ffn_norm": (1.0 + 0.02 * t.randn((D,), generator=g, device=self.dev)).float(),
            })
        self.final_norm = (1.0 + 0.02 * t.randn((D,), generator=g, device=self.dev)).float()
        self.lm_head = int4(D, V)
        self.embed = (t.randn((V, D), generator=g, device=self.dev) * std).half()
        self.cs = rope_table(dh, cfg.max_len, cfg.theta).to(self.dev)
        self.lut = ExponentialLUT(range_max=cfg.lut_range)
        self.table = self.lut.device_table(self.dev)
        N, L = n_traces, cfg.max_len
        self.k_cache = [t.zeros((N, H, L, dh), dtype=t.float16, device=self.dev) for _ in range(cfg.layers)]
        self.v_cache = [t.zeros((N, H, L, dh), dtype=t.float16, device=self.dev) for _ in range(cfg.layers)]
        f16, f32 = t.float16, t.float32
        self.x = t.empty((N, D), dtype=f32, device=self.dev)
        self.h = t.empty((N, D), dtype=f16, device=self.dev)
        self.qkv = t.empty((N, 3 * D), dtype=f16, device=self.dev)
        self.q = t.empty((N, H, dh), dtype=f16, device=self.dev)
        self.att = t.empty((N, H, dh), dtype=f16, device=self.dev)
        self.o = t.empty((N, D), dtype=f16, device=self.dev)
        self.gu = t.empty((N, 2 * F), dtype=f16, device=self.dev)
        self.a = t.empty((N, F), dtype=f16, device=self.dev)
        self.logits = t.empty((N, V), dtype=f16, device=self.dev)
        self.ids = t.zeros((N,), dtype=t.int32, device=self.dev)
        self.pos = t.zeros((N,), dtype=t.int32, device=self.dev)
        self.err = t.zeros((1,), dtype=t.int32, device=self.dev)
        self.length = 0  # positions filled so far (the same for every trace)
        self.graph = None
        nb = int(lib().mb_decode_attn_workspace_size(N, H, L, dh))
        self.ws = t.zeros(nb, dtype=t.uint8, device=self.dev)
        self.scale = float(np.float32(1.0 / np.sqrt(dh)))

    # -------------------------------------------------------------------------
    def fill_prompt_cache(self, length: int, seed: int = 1):
        """Seeded N(0,1) keys and values for the first ``length`` positions of every
        layer (a stand-in for the prompt's prefill; decode speed does not depend on the
        cache contents), and sets the next position to ``length``."""
        t = _lib.torch()
        if not 0 <= length < self.cfg.max_len:
            raise ValueError("prompt length must leave room to decode")
        g = t.Generator(device=self.dev)
        g.manual_seed(seed)
        for kc, vc in zip(self.k_cache, self.v_cache):
            kc[:, :, :length].normal_(generator=g)
            vc[:, :, :length].normal_(generator=g)
        self.length = length
        self.pos.fill_(length)

    def step(self, ids):
        """One decode step for all traces: token ids [N] (int32, device) in, the greedy
        next ids [N] out (a device tensor, also kept in ``self.ids``)."""
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

    def _enqueue(self, ids, device_lengths: bool):
        cfg, N, L = self.cfg, self.N, lib()
        D, H, dh, F, V = cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.vocab
        st = stream_of(self.dev)
        p = lambda x: x.data_ptr()  # noqa: E731
        err = p(self.err)
        check(L.mb_embed(p(ids), N, p(self.embed), V, D, p(self.x), err, st), "mb_embed")
        y = None
        for li, lw in enumerate(self.layers):
            check(L.mb_add_rmsnorm(p(self.x), y, p(lw["attn_norm"]), N, D, cfg.eps, p(self.h), st), "mb_add_rmsnorm")
            check(L.mb_int4_gemm(p(self.h), p(lw["wqkv"]), p(self.qkv), N, D, 3 * D, err, st), "qkv")
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
            check(L.mb_int4_gemm(p(self.att), p(lw["wo"]), p(self.o), N, D, D, err, st), "o_proj")
            check(L.mb_add_rmsnorm(p(self.x), p(self.o), p(lw["ffn_norm"]), N, D, cfg.eps, p(self.h), st),
                  "mb_add_rmsnorm")
            check(L.mb_int4_gemm(p(self.h), p(lw["wgu"]), p(self.gu), N, D, 2 * F, err, st), "gate_up")
            check(L.mb_swiglu(p(self.gu), N, F, p(self.a), st), "mb_swiglu")
            check(L.mb_int4_gemm(p(self.a), p(lw["wd"]), p(self.o), N, F, D, err, st), "down")
            y = p(self.o)
        check(L.mb_add_rmsnorm(p(self.x), y, p(self.final_norm), N, D, cfg.eps, p(self.h), st), "final norm")
        check(L.mb_int4_gemm(p(self.h), p(self.lm_head), p(self.logits), N, D, V, err, st), "lm_head")
        check(L.mb_argmax_f16(p(self.logits), N, V, p(self.ids), st), "mb_argmax_f16")
        check(L.mb_advance_positions(p(self.pos), N, st), "mb_advance_positions")

    def generate(self, first_ids, steps: int):
        """Greedy decode ``steps`` tokens from ``first_ids`` [N]; returns [steps, N] ids
        (device, int32)."""
        t = _lib.torch()
        out = t.empty((steps, self.N), dtype=t.int32, device=self.dev)
        ids = first_ids
        for s in range(steps):
            ids = self.step(ids)
            out[s].copy_(ids)
        return out


__all__ = ["DecoderConfig", "Int4Decoder", "rope_table"]


def main(argv=None) -> int:
    """``python -m moat_b200.decode``: build the config-5 decoder (random INT4 weights),
    seed a prompt-length KV cache and time greedy decode steps (CUDA graph replay by
    default, ``--eager`` for per-kernel launches)."""
    import argparse
    import json
    import time
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--traces", type=int, default=16)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--eager", action="store_true")
    args = ap.parse_args(argv)
    t = _lib.require_cuda()
    cfg = DecoderConfig(layers=args.layers, max_len=max(768, args.prompt + args.warmup + args.steps + 2))
    t0 = time.perf_counter()
    dec = Int4Decoder(cfg, args.traces, seed=0)
    dec.fill_prompt_cache(args.prompt, seed=1)
    dec.ids.copy_(t.arange(args.traces, dtype=t.int32, device=dec.dev) * 7919 % cfg.vocab)
    dec.step(dec.ids)
    if not args.eager:
        dec.capture()
    step = (lambda: dec.step(dec.ids)) if args.eager else dec.step_graphed
    for _ in range(args.warmup):
        step()
    t.cuda.synchronize()
    build = time.perf_counter() - t0
    e0, e1 = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    t.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"tok_per_s": args.traces / ms * 1e3, "ms_per_step": ms, "traces": args.traces,
                      "layers": cfg.layers, "prompt": args.prompt, "steps": args.steps,
                      "mode": "eager" if args.eager else "graph", "setup_s": build,
                      "device_error_bits": int(dec.err.item())}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
