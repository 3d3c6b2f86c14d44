"""GPU parity of the batched sampler (``mb_sample_tokens``).

Against the oracle restatement (``oracle/sampling.py``, itself pinned to the
reference's sampler in ``tests/test_sampling_cpu.py``) on the same inputs and the same
uniform draws: tokens equal, log-probabilities within one fp16 step (greedy: the value
is fp16) or 1e-6 relative (temperature: fp32 log). And against the reference's golden
greedy outputs directly. Edge cases as in the reference's fuzz tests
(antigravity-engine/tests/test_fuzz_extreme_inputs.py:31-60): zero logits, huge
logits, extreme temperatures; and the device random stream's counter, graph replay and
its distribution.
"""

import json
import os

import numpy as np
import pytest

from oracle import attention as OA
from oracle import sampling as S

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TABLE = OA.exp_table(32768, 10.0)


def _ulps16(a, b):
    ai = np.asarray(a, np.float32).astype(np.float16).view(np.int16).astype(np.int64)
    bi = np.asarray(b, np.float32).astype(np.float16).view(np.int16).astype(np.int64)
    return np.abs(ai - bi)


def _dev(x, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def _run(x, T, cuda, uniforms=None, seed=0):
    import torch
    from moat_b200.sampling import BatchSampler
    N, V = x.shape
    s = BatchSampler(N, V, device=cuda, seed=seed)
    u = None if uniforms is None else _dev(np.asarray(uniforms, np.float32), cuda)
    tok, lp = s.sample(_dev(x, cuda), T, uniforms=u)
    torch.cuda.synchronize()
    return tok.cpu().numpy().copy(), lp.cpu().numpy().copy(), int(s.err.item())


def test_greedy_matches_reference_golden(cuda):
    g = np.load(os.path.join(GOLD, "sampling_vectors.npz"))
    with open(os.path.join(GOLD, "sampling_vectors.json")) as f:
        meta = json.load(f)
    for name, c in meta["cases"].items():
        dt = np.dtype(c["dtype"])
        x = (np.zeros((c["N"], c["V"]), dt) if c["seed"] is None
             else S.make_logits(c["N"], c["V"], c["seed"], c["scale"], dt))
        tok, lp, err = _run(x, 0.0, cuda)
        assert err == 0
        np.testing.assert_array_equal(tok, g[name + "_tok"], err_msg=name)
        assert _ulps16(lp, g[name + "_lp"]).max() <= 1, name
        otok, olp = S.sample_tokens(x, 0.0, TABLE, 10.0, np.zeros(c["N"], np.float32))
        np.testing.assert_array_equal(tok, otok)
        assert _ulps16(lp, olp).max() <= 1


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("T", [1e-10, 0.01, 0.7, 1.0, 10.0, 100.0])
def test_temperature_matches_oracle(cuda, dtype, T):
    x = S.make_logits(8, 1000, 10, 3.0, dtype)
    if not np.all(np.isfinite(S.scaled_logits(x, T))):
        pytest.skip("the reference raises here (covered by test_non_finite_rows)")
    u = S.uniforms(5, 0, 8)
    tok, lp, err = _run(x, T, cuda, uniforms=u)
    otok, olp = S.sample_tokens(x, T, TABLE, 10.0, u)
    assert err == 0
    np.testing.assert_array_equal(tok, otok)
    np.testing.assert_allclose(lp, olp, rtol=1e-6, atol=1e-6)


def test_big_vocabulary_and_ties(cuda):
    x = S.make_logits(4, 151936, 11, 3.0, np.float16)
    x[1] = 0.0                     # every column ties: the first 50 columns are the set
    x[2] = -5.0
    x[2, :64] = 5.0                # 64 ties at the top: the first 50 of them
    u = np.array([0.1, 0.999, 0.5, 0.0], np.float32)
    tok, lp, err = _run(x, 0.7, cuda, uniforms=u)
    otok, olp = S.sample_tokens(x, 0.7, TABLE, 10.0, u)
    assert err == 0
    np.testing.assert_array_equal(tok, otok)
    np.testing.assert_allclose(lp, olp, rtol=1e-6, atol=1e-6)
    assert 0 <= tok[1] < 50 and 0 <= tok[2] < 50


@pytest.mark.parametrize("T", [100.0, 0.05])
def test_big_vocabulary_plateaus_and_clipped_rows(cuda, T):
    """Full config-5 rows at the two ends of the temperature range. T = 100: every
    probability is about 1/V, in the fp16 subnormal range, where long runs of
    neighbouring table indices share one probability (the tie interval of the k-th
    largest spans many indices). T = 0.05: fewer than 50 columns lie within the table's
    range of the maximum, so the set is completed with the first columns at the clipped
    index."""
    x = S.make_logits(4, 151936, 12, 3.0, np.float16)
    u = np.array([0.1, 0.5, 0.9, 0.0], np.float32)
    tok, lp, err = _run(x, T, cuda, uniforms=u)
    otok, olp = S.sample_tokens(x, T, TABLE, 10.0, u)
    assert err == 0
    np.testing.assert_array_equal(tok, otok)
    np.testing.assert_allclose(lp, olp, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("V", [1, 7, 50, 63, 1000])
def test_small_vocabularies(cuda, V):
    x = S.make_logits(3, V, 4, 2.0, np.float32)
    u = np.array([0.0, 0.5, 0.99999], np.float32)
    tok, lp, _ = _run(x, 1.0, cuda, uniforms=u)
    otok, olp = S.sample_tokens(x, 1.0, TABLE, 10.0, u)
    np.testing.assert_array_equal(tok, otok)
    np.testing.assert_allclose(lp, olp, rtol=1e-6, atol=1e-6)


def test_extreme_logits_have_finite_logprobs(cuda):
    """The reference's fuzz cases: huge, huge negative and zero logits at T = 0.7."""
    rng = np.random.default_rng(1337)
    for x in (rng.standard_normal((8, 1000)) * 1e8, -np.abs(rng.standard_normal((8, 1000))) * 1e8,
              np.zeros((8, 1000))):
        x = x.astype(np.float32)
        u = S.uniforms(3, 1, 8)
        tok, lp, err = _run(x, 0.7, cuda, uniforms=u)
        assert err == 0 and np.all(np.isfinite(lp))
        otok, olp = S.sample_tokens(x, 0.7, TABLE, 10.0, u)
        np.testing.assert_array_equal(tok, otok)


def test_non_finite_rows(cuda):
    """fp16 logits over a tiny temperature overflow (the reference raises): error bit,
    the argmax as token, a NaN log-probability."""
    x = S.make_logits(2, 1000, 10, 3.0, np.float16)
    tok, lp, err = _run(x, 1e-5, cuda)
    assert err & 4
    assert tok.tolist() == np.argmax(x, axis=1).tolist()
    assert np.all(np.isnan(lp))
    from moat_b200.sampling import sample_tokens
    with pytest.raises(FloatingPointError):
        sample_tokens(x, temperature=1e-5)


def test_nan_rows_and_signed_zero_maxima(cuda):
    """T > 0 on fp16 rows (the kernel's packed path): rows holding a NaN of either sign
    err with the first NaN column as token (numpy.argmax's choice); rows whose maximum
    is zero, held as -0 in some columns and +0 in others (or -0 alone), sample exactly
    as the oracle does."""
    x = S.make_logits(5, 1000, 21, 3.0, np.float16)
    bits = x.view(np.uint16)
    bits[0, 700] = 0xFE00      # negative quiet NaN
    bits[0, 900] = 0x7E00
    bits[1, 333] = 0x7C01      # positive signalling NaN
    x[2] = -np.abs(x[2])
    x[2, [10, 500]] = 0.0
    bits[2, [20, 800]] = 0x8000  # -0
    x[3] = -np.abs(x[3])
    bits[3, [5, 6, 999]] = 0x8000
    x[4] = -np.abs(x[4]) - 1.0
    u = np.array([0.3, 0.3, 0.1, 0.7, 0.95], np.float32)
    tok, lp, err = _run(x, 0.7, cuda, uniforms=u)
    assert err & 4
    assert tok[0] == 700 and tok[1] == 333
    assert np.isnan(lp[0]) and np.isnan(lp[1])
    otok, olp = S.sample_tokens(x[2:], 0.7, TABLE, 10.0, u[2:])
    np.testing.assert_array_equal(tok[2:], otok)
    np.testing.assert_allclose(lp[2:], olp, rtol=1e-6, atol=1e-6)


def test_device_stream_counter_and_graph_replay(cuda):
    import torch
    from moat_b200.sampling import BatchSampler
    N, V = 16, 5000
    x = S.make_logits(N, V, 21, 2.0, np.float16)
    s = BatchSampler(N, V, device=cuda, seed=99)
    xd = _dev(x, cuda)
    for c in range(2):  # eager calls draw counter 0, 1
        tok, lp = s.sample(xd, 0.8)
        torch.cuda.synchronize()
        otok, _ = S.sample_tokens(x, 0.8, TABLE, 10.0, S.uniforms(99, c, N))
        np.testing.assert_array_equal(tok.cpu().numpy(), otok)
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            s.sample(xd, 0.8)
    torch.cuda.current_stream().wait_stream(side)
    for c in range(2, 5):  # replays draw counter 2, 3, 4
        g.replay()
        torch.cuda.synchronize()
        otok, olp = S.sample_tokens(x, 0.8, TABLE, 10.0, S.uniforms(99, c, N))
        np.testing.assert_array_equal(s.tokens.cpu().numpy(), otok)
        np.testing.assert_allclose(s.logprobs.cpu().numpy(), olp, rtol=1e-6, atol=1e-6)
    assert s.rng_state.cpu().tolist() == [5, 0]
    assert int(s.err.item()) == 0


def test_device_draws_follow_the_top50_distribution(cuda):
    row = S.make_logits(1, 60, 12, 1.0, np.float32)
    xs = np.repeat(row, 20000, axis=0)
    from moat_b200.sampling import sample_tokens
    tok, _ = sample_tokens(xs, temperature=1.0, seed=4)
    p16 = S.lut_probs16(S.scaled_logits(row, 1.0), TABLE, 10.0)[0]
    cand = S.top_candidates(p16, 50)
    probs = np.zeros(60)
    probs[cand] = p16[cand].astype(np.float64) / p16[cand].astype(np.float64).sum()
    counts = np.bincount(tok, minlength=60)
    assert counts[probs == 0].sum() == 0
    exp = probs * counts.sum()
    keep = exp > 0
    assert float(np.sum((counts[keep] - exp[keep]) ** 2 / exp[keep])) < 95.0
    np.testing.assert_array_equal(tok, S.sample_tokens(xs, 1.0, TABLE, 10.0, S.uniforms(4, 0, 20000))[0])
