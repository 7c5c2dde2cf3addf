"""The codec oracle's building blocks against direct loop transcriptions of the
reference kernels' formulas (src/gpu/kernels.rs:453-974), on small random
shapes (CPU only)."""
import numpy as np
import pytest
import torch

from oracle import codec as K


def _rng(seed=0):
    return np.random.default_rng(seed)


@pytest.fixture(scope="module")
def codec_weights():
    return K.generate(0)


def test_causal_conv_matches_kernel_loop():
    """codec_causal_conv1d_dilated_f32: source = t + k*dil - pad, pad = dil*(k-1)."""
    r = _rng(1)
    ci, co, T, k, d = 3, 4, 11, 3, 2
    x = r.standard_normal((ci, T)).astype(np.float32)
    w = r.standard_normal((co, ci, k)).astype(np.float32)
    b = r.standard_normal(co).astype(np.float32)
    pad = d * (k - 1)
    ref = np.zeros((co, T), np.float32)
    for oc in range(co):
        for t in range(T):
            s = b[oc]
            for ic in range(ci):
                for kk in range(k):
                    src = t + kk * d - pad
                    if 0 <= src < T:
                        s += x[ic, src] * w[oc, ic, kk]
            ref[oc, t] = s
    got = K.CodecOracle._causal_conv(torch.from_numpy(x), torch.from_numpy(w),
                                     torch.from_numpy(b), d).numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("kernel_mult", [1, 2])
def test_transconv_matches_kernel_loop(kernel_mult):
    """codec_transconv1d_channels_f32: out_t = in_t*stride + k, first in*stride kept."""
    r = _rng(2)
    ci, co, T, s = 3, 2, 5, 3
    k = kernel_mult * s
    x = r.standard_normal((ci, T)).astype(np.float32)
    w = r.standard_normal((ci, co, k)).astype(np.float32)
    b = r.standard_normal(co).astype(np.float32)
    out_T = T * s
    ref = np.zeros((co, out_T), np.float32)
    for oc in range(co):
        for ot in range(out_T):
            acc = b[oc]
            for kk in range(k):
                rem = ot - kk
                if rem >= 0 and rem % s == 0:
                    it = rem // s
                    if it < T:
                        acc += sum(x[ic, it] * w[ic, oc, kk] for ic in range(ci))
            ref[oc, ot] = acc
    got = K.CodecOracle._transconv(torch.from_numpy(x), torch.from_numpy(w),
                                   torch.from_numpy(b), s).numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


def test_snake_matches_kernel_formula():
    """codec_snake_beta_f32: x + sin(x * e^alpha)^2 / (e^beta + 1e-9)."""
    r = _rng(3)
    x = r.standard_normal((4, 7)).astype(np.float32)
    al = r.standard_normal(4).astype(np.float32) * 0.3
    be = r.standard_normal(4).astype(np.float32) * 0.3
    ref = x + np.sin(x * np.exp(al)[:, None]) ** 2 / (np.exp(be)[:, None] + 1e-9)
    got = K.CodecOracle._snake(torch.from_numpy(x), torch.from_numpy(al),
                               torch.from_numpy(be)).numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_rvq_matches_kernel_loop(codec_weights):
    """codec_rvq_project_f32 with normalised codebooks, codes taken modulo 2048."""
    w = codec_weights
    o = K.CodecOracle(w)
    codes = np.array([[5, 7, -1] + [2047] * 13, [4096 + 3] + list(range(15))], dtype=np.int64)
    got = o.rvq(codes.reshape(-1)).numpy()
    q = "decoder.quantizer"

    def book(name):
        e = w[f"{name}._codebook.embedding_sum"].astype(np.float64)
        u = np.maximum(w[f"{name}._codebook.cluster_usage"].astype(np.float64), 1e-7)
        return e / u[:, None]

    first = book(f"{q}.rvq_first.vq.layers.0")
    rest = [book(f"{q}.rvq_rest.vq.layers.{g}") for g in range(15)]
    wf = w[f"{q}.rvq_first.output_proj.weight"][:, :, 0].astype(np.float64)
    wr = w[f"{q}.rvq_rest.output_proj.weight"][:, :, 0].astype(np.float64)
    for t in range(codes.shape[0]):
        c = codes[t] % 2048
        fv = first[c[0]]
        rv = sum(rest[g - 1][c[g]] for g in range(1, 16))
        np.testing.assert_allclose(got[:, t], wf @ fv + wr @ rv, rtol=1e-4, atol=1e-4)


def test_decode_shapes_and_range(codec_weights):
    """decode_codes: 1920 samples per frame, clamped to [-1, 1]; empty in, empty out."""
    o = K.CodecOracle(codec_weights)
    wav = o.decode(np.random.default_rng(4).integers(0, 2048, (3, 16)))
    assert wav.shape == (3 * K.SAMPLES_PER_FRAME,)
    assert np.all(np.abs(wav) <= 1.0) and wav.std() > 0.05
    assert o.decode([]).size == 0


def test_golden_fixture_reproduces(codec_weights):
    """tests/golden/codec_seed0.json (made by tests/golden/make_codec_golden.py)
    pins the codec oracle's stage sums and waveform across changes."""
    import importlib.util
    import json
    from pathlib import Path

    gdir = Path(__file__).parent / "golden"
    spec = importlib.util.spec_from_file_location("make_codec_golden",
                                                  gdir / "make_codec_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    want = json.loads((gdir / "codec_seed0.json").read_text())
    got = mod.compute(codec_weights)
    assert got["codes"] == want["codes"]
    for stage in ("rvq", "pre_conv", "pre_transformer", "upsample", "waveform"):
        assert got[stage]["shape"] == want[stage]["shape"]
        tol = 1e-5 * want[stage]["abs_sum"]
        assert abs(got[stage]["sum"] - want[stage]["sum"]) <= tol, stage
        assert abs(got[stage]["abs_sum"] - want[stage]["abs_sum"]) <= tol, stage
    np.testing.assert_allclose(got["waveform_samples"], want["waveform_samples"], atol=1e-5)
