"""CPU checks of the parity oracle: golden fixture, known answers of the
reference's formulas, and sampler semantics (no GPU needed)."""
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qtts_oracle as O, synth

GOLDEN = json.loads((Path(__file__).parent / "golden" / "tiny_seed0.json").read_text())


def test_golden_fixture_reproduces(model_dirs):
    from tests.golden.make_golden import compute

    got = compute(model_dirs["tiny"])
    for k in ("ids", "prefill_steps", "prefill_token", "greedy_codes", "sampled_lcg_codes",
              "sampled_philox_codes", "cp_tokens"):
        assert got[k] == GOLDEN[k], k
    for k in ("prefill_sum", "trailing_sum"):
        assert got[k] == pytest.approx(GOLDEN[k], rel=1e-5, abs=1e-5), k
    for k in ("prefill_row0_head", "tts_pad_head", "prefill_logits_head", "cp_embedding_sum_head"):
        np.testing.assert_allclose(got[k], GOLDEN[k], rtol=1e-5, atol=1e-6, err_msg=k)


def test_lcg_known_answer():
    # next_f32 (sampling.rs:120-126) evaluated independently with Python ints.
    state = (0 ^ 0x9E3779B97F4A7C15) & ((1 << 64) - 1)
    expect = []
    for _ in range(5):
        state = (state * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        expect.append((state >> 40) / float(1 << 24))
    r = O.Lcg(0)
    got = [float(r.next_f32()) for _ in range(5)]
    assert got == expect
    assert all(0.0 <= u < 1.0 for u in got)


def test_philox_known_answer():
    # Philox-4x32-10 test vector (Random123 kat_vectors): ctr=0, key=0 ->
    # 6627e8d5 e169c58d bc57ac4c 9b00dbd8; the uniform uses word 0 >> 8.
    assert O.philox_uniform(0, 0) == np.float32(0x6627E8D5 >> 8) / np.float32(1 << 24)


def test_rmsnorm_and_rope_formulas():
    x = torch.tensor([[1.0, -2.0, 3.0, 0.5]])
    g = torch.tensor([1.0, 2.0, 0.5, 1.0])
    ref = x / math.sqrt((1 + 4 + 9 + 0.25) / 4 + 1e-6) * g
    torch.testing.assert_close(O.rmsnorm(x, g, 1e-6), ref)
    cos, sin = O.rope_tables(1_000_000.0, 128, np.array([0, 5]))
    assert torch.all(cos[0] == 1) and torch.all(sin[0] == 0)
    # angle for pair i at position 5: 5 / theta^(2i/128)
    i = 10
    assert cos[1, i].item() == pytest.approx(math.cos(5 / 1_000_000.0 ** (2 * i / 128)), abs=1e-6)
    v = torch.randn(2, 3, 128)
    r = O.rope(v, cos, sin)
    torch.testing.assert_close(r[0], v[0])  # position 0 is identity
    torch.testing.assert_close(r.norm(dim=-1), v.norm(dim=-1))


def test_argmax_device_ties_and_nonfinite():
    v = np.array([0.5, 2.0, -np.inf, 2.0, np.nan], dtype=np.float32)
    assert O.argmax_device(v) == 1  # lowest index wins (kernels.rs:203-205)
    assert O.argmax_device(np.full(4, -np.inf, np.float32)) == 0


def test_device_topk_sampler_cdf():
    logits = np.array([0.0, 3.0, 1.0, 2.0], dtype=np.float32)
    # top-2 at T=1: tokens 1 (e^0) and 3 (e^-1)
    p1 = 1.0 / (1.0 + math.exp(-1.0))
    assert O.sample_topk_device(logits, 2, 1.0, np.float32(p1 - 1e-4)) == 1
    assert O.sample_topk_device(logits, 2, 1.0, np.float32(p1 + 1e-4)) == 3
    assert O.sample_topk_device(logits, 2, 1.0, np.float32(0.999999)) == 3


def test_cpu_sampler_top_p_and_finite_filter():
    logits = np.array([np.inf * -1, 1.0, 5.0, np.nan, 4.0], dtype=np.float32)

    class U:
        def __init__(self, u):
            self.u = u

        def next_f32(self):
            return np.float32(self.u)

    cfg = O.SamplingConfig(True, 0, 0.5, 1.0)  # top_p=0.5 keeps only the max token
    assert O.sample_cpu(logits, cfg, U(0.99)) == 2
    cfg = O.SamplingConfig(True, 300, 1.0, 1.0)  # top_k > 256 -> CPU path, all finite
    assert O.select(logits, cfg, U(0.9999)) in (1, 4)


def test_penalty_per_occurrence_and_suppression(oracles):
    m = oracles["tiny"]
    logits = np.zeros(m.vocab, np.float32)
    logits[5], logits[6] = 2.0, -2.0
    out = m.penalise_and_suppress(logits, [5, 5, 6], 2.0)
    assert out[5] == pytest.approx(0.5)  # divided twice
    assert out[6] == pytest.approx(-4.0)
    assert np.all(np.isneginf(np.delete(out[m.vocab - 1024:], m.codec_eos - (m.vocab - 1024))))
    assert np.isfinite(out[m.codec_eos])


def test_bf16_rounding_matches_torch():
    x = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    b = synth.f32_to_bf16_bits(x)
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(b, t)


def test_prefill_layout(oracles):
    m = oracles["tiny"]
    ids = [11, 12, 13]
    pre, tr, pad = m.prepare(ids)
    assert pre.shape[0] == 9 + 3 and tr.shape[0] == 1
    pre2, tr2, _ = m.prepare(ids, lookahead=1)
    assert pre2.shape[0] == 10 and tr2.shape[0] == 3
    # last text row carries codec_bos, earlier ones codec_pad (text.rs:563-568)
    t = m.projected_text(ids)
    cfg = m.cfg["talker_config"]
    torch.testing.assert_close(pre[-1], t[-1] + m.codec_emb[cfg["codec_bos_id"]])
    torch.testing.assert_close(pre[-2], t[-2] + m.codec_emb[cfg["codec_pad_id"]])


def test_reference_kernel_extraction():
    """oracle/build_ref.py finds every reference kernel that oracle/ref_launch.cu
    launches (needs the reference tree, present where the library is built)."""
    import re
    from pathlib import Path

    from oracle import build_ref

    if not (build_ref.DEFAULT_REFERENCE / "src" / "gpu" / "kernels.rs").exists():
        pytest.skip("reference tree not on this machine")
    names = set(build_ref.kernel_names(build_ref.extract(build_ref.DEFAULT_REFERENCE)))
    launched = set(re.findall(r"(\w+_f32)<<<", (Path(build_ref.HERE) / "ref_launch.cu").read_text()))
    assert launched and launched <= names, launched - names


def test_reference_kernel_library_exports():
    """The built checker library exports one wrapper per launched kernel."""
    import ctypes

    from oracle import ref_kernels

    if not ref_kernels.available():
        pytest.skip("oracle/_ref/libqtts_ref.so not built")
    try:
        lib = ctypes.CDLL(str(ref_kernels.LIB))
    except OSError as e:  # no CUDA driver on this machine
        pytest.skip(str(e))
    for fn in ("ref_rmsnorm", "ref_rope", "ref_write_kv", "ref_attention_scores_cache",
               "ref_softmax", "ref_apply_value_cache", "ref_residual_add", "ref_swiglu",
               "ref_argmax", "ref_suppress", "ref_penalty", "ref_sample_topk"):
        assert hasattr(lib, fn), fn
