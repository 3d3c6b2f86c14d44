"""Generate ``tests/golden/decoder_vectors.npz`` by running the REFERENCE's own decoder
blocks (``antigravity-engine/src/transformer.py``).

Run once, in a container where the reference tree is mounted read-only:

    python tests/golden/make_decoder_golden.py /path/to/reference

A small LLaMA-style model (2 blocks, hidden 64, 4 heads of 16, as many KV heads as
query heads, SwiGLU 96, vocabulary 101, RMSNorm eps 1e-6) is built from the
reference's ``RMSNorm``, ``TransformerBlock`` and ``precompute_freqs_cis`` with seeded
weights, and driven the way ``TinyLlamaModel.forward`` (:200-220) drives its blocks: the
whole prompt at once with the causal mask, then greedy single-token steps with the
returned KV caches. The weights (as ``[K, M]`` matrices for ``x @ W``), the prompt, the
last prompt position's logits and every step's logits and ids are saved; the CPU test
``tests/test_decoder_oracle_cpu.py`` replays them through ``oracle.decoder.CpuDecoder``
one position at a time. Nothing at test or bench time reads the reference tree.
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root: str) -> None:
    import torch
    T = _load("ref_transformer", os.path.join(ref_root, "antigravity-engine/src/transformer.py"))
    torch.manual_seed(1234)
    D, H, F, V, NL, N, P, STEPS, MAXLEN, EPS = 64, 4, 96, 101, 2, 3, 6, 4, 32, 1e-6
    embed = torch.nn.Embedding(V, D)
    blocks = [T.TransformerBlock(D, F, H, H, norm_eps=EPS) for _ in range(NL)]
    norm = T.RMSNorm(D, eps=EPS)
    lm_head = torch.nn.Linear(D, V, bias=False)
    with torch.no_grad():
        for b in blocks:  # non-trivial norm weights
            b.input_layernorm.weight.mul_(1.0 + 0.1 * torch.randn(D))
            b.post_attention_layernorm.weight.mul_(1.0 + 0.1 * torch.randn(D))
        norm.weight.mul_(1.0 + 0.1 * torch.randn(D))
    freqs = T.precompute_freqs_cis(D // H, MAXLEN)
    prompt = torch.randint(0, V, (N, P))

    def run(ids, start, caches):
        h = embed(ids)
        fc = freqs[start:start + ids.shape[1]]
        mask = None
        if ids.shape[1] > 1:
            mask = torch.triu(torch.full((ids.shape[1], ids.shape[1]), float("-inf")), diagonal=1)[None, None]
        new = []
        for i, b in enumerate(blocks):
            h, kv = b(h, fc, mask, kv_cache=None if caches is None else caches[i])
            new.append(kv)
        return lm_head(norm(h)), new

    arrays = {"prompt": prompt.numpy().astype(np.int32)}
    with torch.no_grad():
        logits, caches = run(prompt, 0, None)
        arrays["prompt_last_logits"] = logits[:, -1].numpy()
        ids = torch.argmax(logits[:, -1], dim=-1)
        step_ids, step_logits = [ids.numpy().astype(np.int32)], []
        for s in range(STEPS):
            logits, caches = run(ids[:, None], P + s, caches)
            step_logits.append(logits[:, 0].numpy())
            ids = torch.argmax(logits[:, 0], dim=-1)
            step_ids.append(ids.numpy().astype(np.int32))
    arrays["step_logits"] = np.stack(step_logits)
    arrays["step_ids"] = np.stack(step_ids)  # [STEPS + 1, N]: the input id of each step, then the last output
    with torch.no_grad():
        arrays["embed"] = embed.weight.numpy()
        arrays["final_norm"] = norm.weight.numpy()
        arrays["lm_head"] = lm_head.weight.t().contiguous().numpy()
        for i, b in enumerate(blocks):
            a, m = b.self_attn, b.mlp
            arrays[f"l{i}_wqkv"] = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).t().numpy()
            arrays[f"l{i}_wo"] = a.o_proj.weight.t().contiguous().numpy()
            arrays[f"l{i}_wgu"] = torch.cat([m.gate_proj.weight, m.up_proj.weight], 0).t().numpy()
            arrays[f"l{i}_wd"] = m.down_proj.weight.t().contiguous().numpy()
            arrays[f"l{i}_attn_norm"] = b.input_layernorm.weight.numpy()
            arrays[f"l{i}_ffn_norm"] = b.post_attention_layernorm.weight.numpy()
    arrays["dims"] = np.array([D, H, F, V, NL, N, P, STEPS, MAXLEN], dtype=np.int64)
    arrays["eps"] = np.array([EPS], dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "decoder_vectors.npz"), **{k: np.ascontiguousarray(v) for k, v in
                                                                       arrays.items()})
    print("wrote", os.path.join(HERE, "decoder_vectors.npz"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_decoder_golden.py /path/to/reference")
    main(sys.argv[1])
