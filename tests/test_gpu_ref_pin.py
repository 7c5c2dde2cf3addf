"""Pins the oracle restatement to outputs of the reference's own kernels.

The reference's device kernels (HIP C++ source strings in its
src/gpu/kernels.rs) are extracted and compiled for sm_100a by
oracle/build_ref.py into oracle/_ref/libqtts_ref.so, and run here on the
same inputs as the oracle (oracle/qtts_oracle.py):

* kernel by kernel: RMSNorm, RoPE, argmax (ties, NaN, infinities), codec
  suppression, per-occurrence repetition penalty, device top-k sampling;
* a whole decode step of a tiny talker (every layer of
  decode_step_layer_on_stream, src/model/decode.rs:1694-1894), composed from
  the reference kernels with an fp32 GEMM standing in for rocBLAS sgemm,
  against the oracle's DecoderStack at successive cache offsets;
* the talker head and token (talker.rs:431-496) on those hidden states.

Tolerances: fp32 against fp32, so 1e-5 relative for single kernels; the
GEMM's summation order differs from torch-CPU's, so 1e-4 on whole layers.
Tokens are identical except where the oracle's own margin is below 1e-5.
"""
import numpy as np
import pytest
import torch

from oracle import qtts_oracle as O
from oracle import ref_kernels as R

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not R.available(),
                                 reason="oracle/_ref/libqtts_ref.so not built (oracle/build_ref.py)")]


@pytest.fixture(scope="module")
def rk():
    return R.RefKernels()


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_rmsnorm_and_rope(rk):
    rng = np.random.default_rng(0)
    for rows, cols in [(1, 1024), (16, 128), (8, 128), (1, 2048)]:
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
        got = rk.rmsnorm(dev(x), dev(g), 1e-6, rows, cols).cpu().numpy()
        want = O.rmsnorm(torch.from_numpy(x), torch.from_numpy(g), 1e-6).numpy()
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    for heads, offset in [(16, 0), (8, 7), (16, 300), (8, 4095)]:
        x = rng.standard_normal((heads, 128)).astype(np.float32)
        got = rk.rope(dev(x), heads, 1, 128, offset, 1e6).cpu().numpy()
        cos, sin = O.rope_tables(1e6, 128, np.array([offset]))
        want = O.rope(torch.from_numpy(x)[None], cos, sin)[0].numpy()
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=2e-5)


def test_argmax_suppression_penalty(rk):
    rng = np.random.default_rng(1)
    cases = []
    for vocab in (2048, 3072):
        v = rng.standard_normal(vocab).astype(np.float32)
        cases.append(v)
        t = v.copy()
        t[[5, 700, 1500]] = 9.0  # exact ties: lowest index wins
        cases.append(t)
        n = v.copy()
        n[[3, 10]] = np.nan
        n[11] = np.inf
        cases.append(n)
        cases.append(np.full(vocab, -np.inf, np.float32))
    for v in cases:
        assert rk.argmax(dev(v)) == O.argmax_device(v)
    m = O.OracleModel.__new__(O.OracleModel)
    m.vocab, m.codec_eos = 3072, 2150
    for _ in range(4):
        v = rng.standard_normal(3072).astype(np.float32)
        hist = list(rng.integers(0, 3072, 40)) + [17, 17, 17, -1, 5000]
        got = rk.penalty(dev(v), hist, 1.05)
        got = rk.suppress(got, 2150).cpu().numpy()
        want = m.penalise_and_suppress(v, [h for h in hist], 1.05)
        np.testing.assert_array_equal(got, want)


def test_sample_topk(rk):
    rng = np.random.default_rng(2)
    draws = 0
    for vocab in (2048, 3072):
        for i in range(60):
            v = (rng.standard_normal(vocab) * 2).astype(np.float32)
            if vocab == 3072:
                v[-1024:] = -np.inf  # suppressed band
            u = np.float32(rng.random())
            k = [1, 50, 256][i % 3]
            got = rk.sample_topk(dev(v), k, 0.9, float(u))
            want, margin = O.sample_topk_device(v, k, 0.9, u, with_margin=True)
            if got != want:
                assert margin < 1e-5, (vocab, i, got, want, margin)
            draws += 1
    assert draws == 120


def test_decode_steps_and_head(rk, oracles):
    """A run of decode steps at offsets 0..N-1 through every talker layer."""
    m = oracles["tiny"]
    m.talker.reset()
    ref = R.RefDecodeStack(m.talker)
    rng = np.random.default_rng(3)
    norm_g, head = m.norm.cuda(), m.head.cuda().contiguous()
    hist = []
    for off in range(12):
        x = (rng.standard_normal(m.tdims.hidden) * 0.5).astype(np.float32)
        want = m.talker.forward(torch.from_numpy(x)[None], off)[0]
        got = ref.step(dev(x), off)
        np.testing.assert_allclose(got.cpu().numpy(), want.numpy(), rtol=1e-4, atol=1e-4)
        raw, sup, tok = R.ref_head_token(rk, got, norm_g, head, m.tdims.eps, hist, 1.05,
                                         m.codec_eos)
        _, lg = m.talker_logits(want)
        np.testing.assert_allclose(raw, lg.numpy(), rtol=1e-4, atol=1e-4)
        osup = m.penalise_and_suppress(lg.numpy(), hist, 1.05)
        want_tok = O.argmax_device(osup)
        if tok != want_tok:
            assert O.top2_gap(osup) < 1e-5
        hist.append(want_tok)
