"""GPU parity of the decoder-step glue and of one INT4 decode step.

Element-wise kernels are checked against NumPy restatements of the reference
semantics (antigravity-engine/src/transformer.py). The whole step is checked against
a torch fp32 CPU restatement of the same model: the reference's layer order
(transformer.py:148-158, 199-225) with the INT4 weights dequantized by the oracle and
the oracle's LUT softmax, rounding to fp16 where the GPU path does. Tolerance: logits
within 2e-2 (fp16 activations between fp32-accumulated GEMMs, summation order
differs) and the greedy tokens equal.
"""

import numpy as np
import pytest

from oracle import attention as OA
from oracle import int4 as O

pytestmark = pytest.mark.gpu


def _lib():
    from moat_b200 import _lib as lb
    return lb.lib()


def _st():
    import torch
    return torch.cuda.current_stream().cuda_stream


def test_embed_and_bad_ids(cuda):
    import torch
    L = _lib()
    V, D, N = 50, 96, 5
    tab = torch.randn((V, D), device=cuda).half()
    ids = torch.tensor([0, 7, 49, 3, 7], dtype=torch.int32, device=cuda)
    x = torch.empty((N, D), device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    assert L.mb_embed(ids.data_ptr(), N, tab.data_ptr(), V, D, x.data_ptr(), err.data_ptr(), _st()) == 0
    torch.cuda.synchronize()
    assert torch.equal(x, tab[ids.long()].float()) and int(err.item()) == 0
    bad = torch.tensor([1, 50, -1, 2, 3], dtype=torch.int32, device=cuda)
    assert L.mb_embed(bad.data_ptr(), N, tab.data_ptr(), V, D, x.data_ptr(), err.data_ptr(), _st()) == 0
    torch.cuda.synchronize()
    assert int(err.item()) & 2 and float(x[1].abs().sum()) == 0.0 and torch.equal(x[0], tab[1].float())


@pytest.mark.parametrize("with_residual", [False, True])
def test_add_rmsnorm(cuda, with_residual):
    import torch
    L = _lib()
    N, D, eps = 7, 2048, 1e-6
    x0 = torch.randn((N, D), device=cuda)
    y = torch.randn((N, D), device=cuda).half()
    w = (1 + 0.1 * torch.randn(D, device=cuda)).float()
    x = x0.clone()
    h = torch.empty((N, D), dtype=torch.float16, device=cuda)
    rc = L.mb_add_rmsnorm(x.data_ptr(), y.data_ptr() if with_residual else None, w.data_ptr(), N, D, eps,
                          h.data_ptr(), _st())
    assert rc == 0
    torch.cuda.synchronize()
    xr = (x0.double() + y.double()) if with_residual else x0.double()
    np.testing.assert_allclose(x.double().cpu().numpy(), xr.cpu().numpy(), rtol=1e-6, atol=1e-6)
    ref = (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + eps) * w.double()).float()
    got = h.float().cpu().numpy()
    np.testing.assert_allclose(got, ref.cpu().numpy(), rtol=2e-3, atol=2e-3)


def test_rope_append_matches_reference_rotation(cuda):
    import torch
    from moat_b200.decode import rope_table
    L = _lib()
    N, H, dh, Lmax = 3, 4, 64, 40
    pos = torch.tensor([0, 5, 39], dtype=torch.int32, device=cuda)
    qkv = torch.randn((N, 3 * H * dh), device=cuda).half()
    cs = rope_table(dh, Lmax, 10000.0).to(cuda)
    q = torch.empty((N, H, dh), dtype=torch.float16, device=cuda)
    kc = torch.zeros((N, H, Lmax, dh), dtype=torch.float16, device=cuda)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = L.mb_rope_append(qkv.data_ptr(), N, H, dh, pos.data_ptr(), cs.data_ptr(), Lmax, q.data_ptr(),
                          kc.data_ptr(), vc.data_ptr(), err.data_ptr(), _st())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # the reference's apply_rotary_emb: adjacent pairs as complex numbers times cis(pos * f)
    cis = torch.view_as_complex(cs.cpu())
    x = qkv.float().cpu().reshape(N, 3, H, dh // 2, 2)
    for n in range(N):
        p = int(pos[n])
        rq = torch.view_as_real(torch.view_as_complex(x[n, 0].contiguous()) * cis[p]).reshape(H, dh)
        rk = torch.view_as_real(torch.view_as_complex(x[n, 1].contiguous()) * cis[p]).reshape(H, dh)
        np.testing.assert_allclose(q[n].float().cpu().numpy(), rq.half().float().numpy(), rtol=0, atol=2e-3)
        np.testing.assert_allclose(kc[n, :, p].float().cpu().numpy(), rk.half().float().numpy(), rtol=0, atol=2e-3)
        assert torch.equal(vc[n, :, p].cpu(), qkv[n, 2 * H * dh:].reshape(H, dh).cpu())
    # only position pos[n] was written
    assert float(kc[0, :, 1:].abs().sum()) == 0.0


def test_swiglu(cuda):
    import torch
    L = _lib()
    N, F = 5, 5504
    gu = torch.randn((N, 2 * F), device=cuda).half()
    a = torch.empty((N, F), dtype=torch.float16, device=cuda)
    assert L.mb_swiglu(gu.data_ptr(), N, F, a.data_ptr(), _st()) == 0
    torch.cuda.synchronize()
    g, u = gu[:, :F].double(), gu[:, F:].double()
    ref = (torch.nn.functional.silu(g) * u).cpu().numpy()
    np.testing.assert_allclose(a.float().cpu().numpy(), ref, rtol=2e-3, atol=2e-3)


def test_argmax_ties_and_nan(cuda):
    import torch
    L = _lib()
    N, V = 4, 151936
    logits = torch.randn((N, V), device=cuda).half()
    logits[1, 100] = 8.0
    logits[1, 99999] = 8.0          # tie: the first index wins
    logits[2, 77] = float("nan")    # NaN counts as the largest (numpy.argmax)
    logits[3, :] = -3.0             # all equal: index 0
    ids = torch.empty(N, dtype=torch.int32, device=cuda)
    assert L.mb_argmax_f16(logits.data_ptr(), N, V, ids.data_ptr(), _st()) == 0
    torch.cuda.synchronize()
    ref = np.argmax(logits.float().cpu().numpy(), axis=-1)
    assert ids.cpu().numpy().tolist() == ref.tolist()
    assert ids.cpu().numpy().tolist()[1:] == [100, 77, 0]


def test_argmax_odd_width_unaligned_rows_and_tail(cuda):
    """V = 1001: rows after the first start off a 16-byte boundary (the scalar row
    scan) and the first row ends in a one-column tail after its 16-byte loads. A tie, a
    NaN, a -0 / +0 pair and the row maximum are placed in those tail columns and
    unaligned rows; mb_argmax_f16 equals numpy.argmax and mb_argmax_key_f16 the
    oracle's keys (column offset 4096)."""
    import torch
    from oracle import sampling as S
    L = _lib()
    N, V, col0 = 4, 1001, 4096
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn((N, V), generator=g, device=cuda).half()
    x[0, 1000] = 9.0                      # the maximum in the tail column of the aligned row
    x[1, 3] = x[1, 1000] = 7.5            # tie in an unaligned row: the first index wins
    x[2, 999] = float("nan")              # NaN near the end of an unaligned row
    x[3, :] = -1.0
    x[3, 997] = -0.0
    x[3, 1000] = 0.0                      # -0 == +0: the first of them wins
    ids = torch.empty(N, dtype=torch.int32, device=cuda)
    keys = torch.zeros(N, dtype=torch.int64, device=cuda)
    assert L.mb_argmax_f16(x.data_ptr(), N, V, ids.data_ptr(), _st()) == 0
    assert L.mb_argmax_key_f16(x.data_ptr(), N, V, col0, keys.data_ptr(), _st()) == 0
    torch.cuda.synchronize()
    xn = x.cpu().numpy()
    assert ids.cpu().numpy().tolist() == S.reference_argmax(xn).tolist() == [1000, 3, 999, 997]
    np.testing.assert_array_equal(keys.cpu().numpy(), S.argmax_keys(xn, col0))


@pytest.mark.parametrize("L_used,Lmax,d", [(1, 32, 128), (300, 768, 128), (513, 600, 64)])
def test_attention_over_cache(cuda, L_used, Lmax, d):
    import torch
    from moat_b200.attention import ExponentialLUT
    lb = _lib()
    T, H = 3, 2
    q, k, v = OA.make_attention_inputs(T, H, Lmax, d, L_used + d)
    e = ExponentialLUT(range_max=16.0)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty((T, H, d), dtype=torch.float16, device=cuda)
    nb = int(lb.mb_decode_attn_workspace_size(T, H, L_used, d))
    ws = torch.zeros(nb, dtype=torch.uint8, device=cuda)
    sc = float(np.float32(1.0 / np.sqrt(d)))
    rc = lb.mb_decode_attn_cache(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), T, H, L_used, Lmax, d,
                                 sc, e.device_table(cuda).data_ptr(), e.size, 16.0, ws.data_ptr(), nb, _st())
    assert rc == 0
    torch.cuda.synchronize()
    ref = OA.decode_attention(q, k[:, :, :L_used], v[:, :, :L_used], e.lut, 16.0).astype(np.float32)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=1e-2, atol=1e-2)


def _reference_step(dec, ids, caches, pos):
    """torch fp32 CPU restatement of one decode step of ``dec`` (see module docstring)."""
    import torch
    cfg, N = dec.cfg, dec.N
    D, H, dh, F, V = cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.vocab
    f16 = lambda t: t.half().float()  # noqa: E731

    def deq(sb, K, M):
        return torch.from_numpy(O.unpack_superblock_weights(sb.cpu().numpy()).reshape(K, M).astype(np.float32))

    def rms(x, w):
        return f16(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.eps) * w)

    cis = torch.view_as_complex(dec.cs.cpu())
    table = dec.lut.lut
    x = dec.embed.cpu().float()[ids.long().cpu()]
    for li, lw in enumerate(dec.layers):
        h = rms(x, lw["attn_norm"].cpu())
        qkv = f16(h @ deq(lw["wqkv"], D, 3 * D)).reshape(N, 3, H, dh // 2, 2)
        qr = f16(torch.view_as_real(torch.view_as_complex(qkv[:, 0].contiguous()) * cis[pos]).reshape(N, H, dh))
        kr = f16(torch.view_as_real(torch.view_as_complex(qkv[:, 1].contiguous()) * cis[pos]).reshape(N, H, dh))
        kc, vc = caches[li]
        kc[:, :, pos] = kr
        vc[:, :, pos] = qkv[:, 2].reshape(N, H, dh)
        s = torch.einsum("nhd,nhld->nhl", qr, kc[:, :, :pos + 1]) * float(np.float32(1.0 / np.sqrt(dh)))
        p = torch.from_numpy(OA.safe_softmax_lut(s.numpy(), table, cfg.lut_range).astype(np.float32))
        att = f16(torch.einsum("nhl,nhld->nhd", p, vc[:, :, :pos + 1])).reshape(N, D)
        x = x + f16(att @ deq(lw["wo"], D, D))
        h = rms(x, lw["ffn_norm"].cpu())
        gu = f16(h @ deq(lw["wgu"], D, 2 * F))
        a = f16(torch.nn.functional.silu(gu[:, :F]) * gu[:, F:])
        x = x + f16(a @ deq(lw["wd"], F, D))
    h = rms(x, dec.final_norm.cpu())
    return f16(h @ deq(dec.lm_head, D, dec.lm_cols)[:, :V])  # without the LM head's zero padding


@pytest.mark.parametrize("vocab", [1000, 1152])
def test_decoder_steps_match_fp32_reference(cuda, vocab):
    """vocab = 1152 (9 x 128 columns): the LM head runs padded to 1280 columns of
    256-wide strips and its logits are copied back to 1152."""
    import torch
    from moat_b200.decode import DecoderConfig, Int4Decoder
    cfg = DecoderConfig(layers=2, hidden=256, heads=2, head_dim=128, ffn=512, vocab=vocab, max_len=48)
    N = 4
    dec = Int4Decoder(cfg, N, device=cuda, seed=3)
    assert dec.lm_cols == (1280 if vocab == 1152 else vocab)
    dec.fill_prompt_cache(10, seed=4)
    caches = [(k.cpu().float().clone(), v.cpu().float().clone()) for k, v in zip(dec.k_cache, dec.v_cache)]
    ids = torch.tensor([1, 500, 999, 42], dtype=torch.int32, device=cuda)
    for step in range(3):
        pos = dec.length
        ref_logits = _reference_step(dec, ids, caches, pos)
        nxt = dec.step(ids)
        torch.cuda.synchronize()
        got = dec.logits.float().cpu()
        np.testing.assert_allclose(got.numpy(), ref_logits.numpy(), rtol=2e-2, atol=2e-2)
        assert nxt.cpu().tolist() == torch.argmax(got, dim=-1).tolist()
        assert int(dec.err.item()) == 0
        ids = nxt.clone()
    assert dec.pos.cpu().tolist() == [13] * N


def test_captured_step_matches_eager_steps(cuda):
    """The CUDA-graph step (attention length read on the device) gives the eager
    step's tokens and, within the attention's summation-order noise, its logits."""
    import torch
    from moat_b200.decode import DecoderConfig, Int4Decoder
    cfg = DecoderConfig(layers=2, hidden=256, heads=2, head_dim=128, ffn=512, vocab=1000, max_len=300)
    N = 3
    a = Int4Decoder(cfg, N, device=cuda, seed=9)
    b = Int4Decoder(cfg, N, device=cuda, seed=9)
    for dec in (a, b):
        dec.fill_prompt_cache(257, seed=2)
    ids = torch.tensor([5, 6, 7], dtype=torch.int32, device=cuda)
    b.ids.copy_(ids)
    b.step(b.ids)            # one eager step caches plans and tensor maps
    a.step(ids)
    b.capture()
    for _ in range(4):
        ea = a.step(a.ids.clone()).clone()
        eb = b.step_graphed().clone()
        torch.cuda.synchronize()
        np.testing.assert_allclose(b.logits.float().cpu().numpy(), a.logits.float().cpu().numpy(),
                                   rtol=1e-2, atol=1e-2)
        assert eb.cpu().tolist() == ea.cpu().tolist()
    assert a.pos.cpu().tolist() == b.pos.cpu().tolist() == [262] * N
    assert int(b.err.item()) == 0


def test_sampled_decode_step_matches_oracle_draw(cuda):
    """temperature > 0: the step's token is the oracle's draw from the step's own
    logits with the device stream's uniforms (counter = step), eager and replayed."""
    import torch
    from moat_b200.decode import DecoderConfig, Int4Decoder
    from oracle import sampling as S
    cfg = DecoderConfig(layers=2, hidden=256, heads=2, head_dim=128, ffn=512, vocab=1000, max_len=64)
    N = 4
    dec = Int4Decoder(cfg, N, device=cuda, seed=3, temperature=0.8, sample_seed=17)
    dec.fill_prompt_cache(10, seed=4)
    table = OA.exp_table(32768, 10.0)
    dec.ids.copy_(torch.tensor([1, 2, 3, 4], dtype=torch.int32, device=cuda))
    dec.step(dec.ids)
    for c in range(4):
        if c == 1:
            dec.capture()
        if c >= 1:
            dec.step_graphed()
        torch.cuda.synchronize()
        otok, olp = S.sample_tokens(dec.logits.cpu().numpy(), 0.8, table, 10.0, S.uniforms(17, c, N))
        assert dec.ids.cpu().numpy().tolist() == otok.tolist()
        np.testing.assert_allclose(dec.logprobs.cpu().numpy(), olp, rtol=1e-6, atol=1e-6)
    assert int(dec.err.item()) == 0


def test_config5_full_shape_greedy_agreement(cuda):
    """BASELINE config 5 at full shape (24 layers, hidden 2048, 16 x 128 heads, FFN 5504,
    vocabulary 151,936, N = 16): a 32-token random prompt runs through the step, then
    16 greedy steps; the reference-style CPU forward (``oracle/decoder.py``, fp32 torch,
    the same dequantized weights, the prompt's cache copied from the GPU) replays the
    GPU's inputs. The north-star bar is argmax agreement >= 99% over the 256 (trace,
    step) ids, against the reference's exp-LUT decode softmax (batch_generator.py:226)
    and against its exact-softmax TinyLlamaModel (transformer.py:117)."""
    import os
    import torch
    from moat_b200.decode import DecoderConfig, Int4Decoder
    from oracle.decoder import CpuDecoder, argmax_agreement
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = DecoderConfig(max_len=64)
    N, P, S = 16, 32, 16
    dec = Int4Decoder(cfg, N, device=cuda, seed=21)
    try:
        g = torch.Generator(device=cuda).manual_seed(22)
        dec.prefill(torch.randint(0, cfg.vocab, (N, P), generator=g, device=cuda, dtype=torch.int32))
        snap = dec.cache_snapshot()
        ids = dec.ids.clone()
        ins, outs = [], []
        for _ in range(S):
            ins.append(ids.cpu())
            ids = dec.step(ids).clone()
            outs.append(ids.cpu().numpy())
        assert int(dec.err.item()) == 0
        dense = dec.dense_weights()
    finally:
        dec.close()
    gpu = np.stack(outs)
    for mode in ("lut", "exact"):
        cpu = CpuDecoder(dense["layers"], dense["final_norm"], dense["lm_head"], dense["embed"], dense["cis"],
                         cfg.heads, N, P + S + 1, eps=cfg.eps, softmax=mode, lut=dec.lut.lut, lut_range=cfg.lut_range)
        cpu.load_cache(snap[0], snap[1], snap[2])
        with torch.no_grad():
            got = np.stack([torch.argmax(cpu.step(i), dim=-1).numpy() for i in ins])
        agree = argmax_agreement(got, gpu)
        assert agree >= 0.99, (mode, agree)
        del cpu
