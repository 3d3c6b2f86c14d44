"""The CPU decoder oracle (``oracle/decoder.py``) against golden vectors made by the
reference's own decoder blocks (``antigravity-engine/src/transformer.py``; generator
``tests/golden/make_decoder_golden.py``): the reference runs the whole prompt at once
with the causal mask and then single-token steps with its KV caches; the oracle runs
every position as a single-token step with its preallocated cache. Logits agree to fp32
summation-order noise and the greedy ids are identical."""

import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "decoder_vectors.npz"))


def _oracle(gold, softmax="exact"):
    import torch
    from oracle.decoder import CpuDecoder
    D, H, F, V, NL, N, P, STEPS, MAXLEN = (int(x) for x in gold["dims"])
    t = lambda k: torch.from_numpy(gold[k].astype(np.float32))  # noqa: E731
    layers = [{"wqkv": t(f"l{i}_wqkv"), "wo": t(f"l{i}_wo"), "wgu": t(f"l{i}_wgu"), "wd": t(f"l{i}_wd"),
               "attn_norm": t(f"l{i}_attn_norm"), "ffn_norm": t(f"l{i}_ffn_norm")} for i in range(NL)]
    dh = D // H
    freqs = 1.0 / (10000.0 ** (torch.arange(0, dh, 2, dtype=torch.float32) / dh))
    ang = torch.outer(torch.arange(MAXLEN, dtype=torch.float32), freqs)
    cis = torch.polar(torch.ones_like(ang), ang)
    from oracle import attention as OA
    return CpuDecoder(layers, t("final_norm"), t("lm_head"), t("embed"), cis, H, N, MAXLEN,
                      eps=float(gold["eps"][0]), softmax=softmax, lut=OA.exp_table(32768, 16.0), lut_range=16.0)


def test_decoder_oracle_matches_reference_blocks(gold):
    import torch
    dec = _oracle(gold)
    prompt = gold["prompt"]
    with torch.no_grad():
        for p in range(prompt.shape[1]):
            logits = dec.step(torch.from_numpy(prompt[:, p]))
        np.testing.assert_allclose(logits.numpy(), gold["prompt_last_logits"], rtol=1e-4, atol=1e-5)
        ids = gold["step_ids"]
        assert np.array_equal(torch.argmax(logits, -1).numpy(), ids[0])
        for s in range(gold["step_logits"].shape[0]):
            logits = dec.step(torch.from_numpy(ids[s]))
            np.testing.assert_allclose(logits.numpy(), gold["step_logits"][s], rtol=1e-4, atol=1e-5)
            assert np.array_equal(torch.argmax(logits, -1).numpy(), ids[s + 1])


def test_decoder_oracle_lut_softmax_stays_close(gold):
    """The exp-LUT softmax (the reference's batch decode path) changes the logits by far
    less than the 1e-2 bar on the same model."""
    import torch
    a, b = _oracle(gold, "exact"), _oracle(gold, "lut")
    prompt = gold["prompt"]
    with torch.no_grad():
        for p in range(prompt.shape[1]):
            la, lb = a.step(torch.from_numpy(prompt[:, p])), b.step(torch.from_numpy(prompt[:, p]))
    np.testing.assert_allclose(lb.numpy(), la.numpy(), rtol=1e-2, atol=1e-2)


def test_cache_load_and_full_cache_error(gold):
    import torch
    a, b = _oracle(gold), _oracle(gold)
    prompt = torch.from_numpy(gold["prompt"])
    with torch.no_grad():
        for p in range(3):
            a.step(prompt[:, p])
        b.load_cache(a.k_cache, a.v_cache, 3)
        np.testing.assert_array_equal(a.step(prompt[:, 3]).numpy(), b.step(prompt[:, 3]).numpy())
    b.length = b.max_len
    with pytest.raises(ValueError):
        b.step(prompt[:, 0])
