"""Parity of the sm_100a path (through the C ABI) against the CPU oracle.

Bar: tokens identical wherever the oracle's top-2 logit
gap exceeds 1e-2; logits within 2e-2 max-abs; sampled runs (in the
reference's LCG draw order, and Philox) reproduce the oracle's tokens wherever
the draw is robust to a 5e-3 logit error (tests/parity.py). Rollouts are
checked with the oracle teacher-forced along the GPU's own codes, so a
near-tie does not make later frames incomparable.
"""
import json
import shutil
import struct

import numpy as np
import pytest
import torch

from oracle import qtts_oracle as O, synth
from parity import check_codes, check_end

pytestmark = pytest.mark.gpu

GAP = 1e-2
LOGIT_TOL = 2e-2
GREEDY = O.SamplingConfig(False, 0, 1.0, 1.0)
SAMPLED = O.SamplingConfig(True, 50, 1.0, 0.9)
SHAPES = ["tiny", "tiny_proj"]


@pytest.fixture(scope="module")
def engines(pkg, model_dirs):
    out = {s: pkg.HipTtsEngine.load_with_options(model_dirs[s], pkg.EngineOptions(0, 128))
           for s in SHAPES}
    yield out
    for e in out.values():
        e.close()


def ids_for(seed, n=10, vocab=4000):
    return np.random.default_rng(seed).integers(0, vocab, n)


def gaps_per_code(records):
    return [g for r in records for g in [r.talker_gap] + r.cp_gaps]


def assert_tokens_match(gpu_codes, ref_codes, gaps):
    """Greedy codes against the oracle's own choices along the same path:
    identical wherever the oracle's top-2 gap exceeds GAP."""
    gpu, ref = np.asarray(gpu_codes), np.asarray(ref_codes[: len(gpu_codes)])
    assert len(gpu) == len(ref)
    mism = np.flatnonzero(gpu != ref)
    hard = [int(i) for i in mism if gaps[i] > GAP]
    assert not hard, f"token mismatch above the gap threshold at {hard[:10]}"


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("lookahead", [None, 1, 3])
def test_text_prep(engines, oracles, shape, lookahead):
    e, m = engines[shape], oracles[shape]
    ids = ids_for(1, 7)
    got = e.prepare_inputs_from_ids(ids, lookahead)
    pre, tr, pad = m.prepare(list(ids), lookahead)
    np.testing.assert_allclose(got.prefill, pre.numpy(), atol=1e-4, rtol=1e-4)
    np.testing.assert_allclose(got.trailing_text, tr.numpy(), atol=1e-4, rtol=1e-4)
    np.testing.assert_allclose(got.tts_pad_embed, pad.numpy(), atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("shape", SHAPES)
def test_talker_prefill_and_step(engines, oracles, shape):
    e, m = engines[shape], oracles[shape]
    pre, _, _ = m.prepare(list(ids_for(2, 12)))
    hidden, logits, tok = e.talker_prefill(pre.numpy())
    _, rh, rl = m.talker_prefill(pre)
    assert np.abs(hidden - rh.numpy()).max() <= LOGIT_TOL
    assert np.abs(logits - rl).max() <= LOGIT_TOL
    sup = m.penalise_and_suppress(rl, None, 1.0)
    if O.top2_gap(sup) > GAP:
        assert tok == O.argmax_device(sup)
    x = np.random.default_rng(5).standard_normal(e.hidden).astype(np.float32) * 0.05
    for off in (pre.shape[0], pre.shape[0] + 1):
        h2, l2, t2 = e.talker_decode_step(x, off)
        _, rh2, rl2 = m.talker_step(torch.from_numpy(x), off)
        print(f"[logits] {shape} talker step at {off}: max abs error {np.abs(l2 - rl2).max():.2e}")
        assert np.abs(l2 - rl2).max() <= LOGIT_TOL
        assert np.abs(h2 - rh2.numpy()).max() <= LOGIT_TOL


@pytest.mark.parametrize("shape", SHAPES)
def test_code_predictor_reference_inputs(engines, oracles, shape):
    """code-predictor-parity's deterministic inputs (qwen3_tts_reference.py:620-660)."""
    e, m = engines[shape], oracles[shape]
    th = O.deterministic_hidden(e.hidden, 17, 15.0)
    se = O.deterministic_hidden(e.hidden, 23, 11.0)
    toks, esum, logits = e.code_predictor(th, se)
    rt, resum, gaps, rlg = m.code_predictor(torch.from_numpy(th), torch.from_numpy(se), GREEDY,
                                            O.Lcg(0), forced=toks)
    print(f"[logits] {shape} CodePredictor heads: max abs error "
          f"{max(float(np.abs(logits[g] - rlg[g]).max()) for g in range(len(toks))):.2e}")
    for g in range(len(toks)):
        assert np.abs(logits[g] - rlg[g]).max() <= LOGIT_TOL
        if gaps[g] > GAP:
            assert toks[g] == O.argmax_device(rlg[g]), g
    np.testing.assert_allclose(esum, resum.numpy(), atol=2e-3)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("rng", ["lcg", "philox"])
def test_code_predictor_sampler_exact(engines, oracles, pkg, shape, rng):
    """The device top-k sampler against the reference's sampling semantics on
    the GPU's own logits: the CodePredictor pass (the same kernel the frame
    graph runs) returns every head's logits and token; the oracle's
    sample_topk_device on those logits with the same draws must pick the same
    tokens (sample_topk_f32, kernels.rs:265-336), exempt only where the
    draw sits within 1e-5 (logit units) of a bucket edge."""
    e = engines[shape]
    th = O.deterministic_hidden(e.hidden, 17, 15.0)
    se = O.deterministic_hidden(e.hidden, 23, 11.0)
    seed = 5
    opts = pkg.GenerateOptions(decode_audio=False, subtalker_dosample=True, subtalker_top_k=50,
                               subtalker_temperature=0.9, seed=seed, rng=rng)
    toks, _, logits = e.code_predictor(th, se, opts)
    draws = O.Lcg(seed) if rng == "lcg" else O.PhiloxStream(seed)
    for g in range(len(toks)):
        u = draws.next_f32()
        want, margin = O.sample_topk_device(logits[g], 50, 0.9, u, with_margin=True)
        assert toks[g] == want or margin < 1e-5, (g, toks[g], want, margin)


@pytest.mark.parametrize("shape", SHAPES)
def test_greedy_rollout(engines, oracles, pkg, shape):
    e, m = engines[shape], oracles[shape]
    ids = ids_for(3, 10)
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=24)
    out = e.generate_codes_from_ids(ids, opts)
    assert out.frames == 24 and len(out.codes) == 24 * 16 and not out.ended_by_eos
    pre, tr, pad = m.prepare(list(ids))
    codes, ended, recs = m.rollout(pre, tr, pad, 24, GREEDY, GREEDY, forced_codes=out.codes)
    assert_tokens_match(out.codes, codes, gaps_per_code(recs))


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("rng", ["lcg", "philox"])
def test_sampled_rollout(engines, oracles, pkg, shape, rng):
    e, m = engines[shape], oracles[shape]
    ids = ids_for(4, 9)
    opts = pkg.GenerateOptions(decode_audio=False, max_frames=16, seed=11, rng=rng)
    out = e.generate_codes_from_ids(ids, opts)
    pre, tr, pad = m.prepare(list(ids))
    codes, _, recs = m.rollout(pre, tr, pad, 16, SAMPLED, SAMPLED, penalty=1.05, seed=11,
                               rng_kind=rng, forced_codes=out.codes)
    check_codes(out.codes, codes, recs, f"sampled {shape} {rng}", sampled=True)


def test_cpu_sampler_path(engines, oracles, pkg):
    """top_k > 256 and top_p < 1 route to the reference's CPU sampler semantics."""
    e, m = engines["tiny"], oracles["tiny"]
    ids = ids_for(5, 6)
    opts = pkg.GenerateOptions(decode_audio=False, max_frames=6, top_k=300, top_p=0.8,
                               subtalker_top_k=0, subtalker_top_p=0.9, seed=3)
    out = e.generate_codes_from_ids(ids, opts)
    t = O.SamplingConfig(True, 300, 0.8, 0.9)
    s = O.SamplingConfig(True, 0, 0.9, 0.9)
    pre, tr, pad = m.prepare(list(ids))
    codes, _, recs = m.rollout(pre, tr, pad, 6, t, s, penalty=1.05, seed=3,
                               forced_codes=out.codes)
    check_codes(out.codes, codes, recs, "cpu sampler path", sampled=True)


def test_graph_equals_eager(engines, oracles, pkg):
    """The frame graph's CodePredictor tokens equal the eager pass on the same
    prefix (decode-step-graph-bench.rs:71-97 checks graph == eager)."""
    e, m = engines["tiny"], oracles["tiny"]
    ids = ids_for(6, 8)
    inp = e.prepare_inputs_from_ids(ids)
    hidden, _, tok = e.talker_prefill(inp.prefill)
    sem = m.codec_emb[tok].numpy()
    toks, _, _ = e.code_predictor(hidden, sem)
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=2)
    out = e.generate_codes_from_ids(ids, opts)
    assert out.codes[0] == tok
    # the graph replays the same per-op kernels the eager seam launches
    assert list(out.codes[1:16]) == list(toks)


def test_stream_chunks(engines, oracles, pkg):
    e, m = engines["tiny"], oracles["tiny"]
    ids = ids_for(7, 20)
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=15)
    st = e.start_stream_from_ids(ids, opts, pkg.StreamOptions(text_lookahead_tokens=8))
    chunks = []
    while (c := st.next_codes_chunk(6)) is not None:
        chunks.append(c)
    assert [c.frames for c in chunks] == [6, 6, 3]
    assert [c.total_frames for c in chunks] == [6, 12, 15]
    codes = [x for c in chunks for x in c.codes]
    assert st.next_codes_chunk(6) is None
    with pytest.raises(pkg.InvalidInput):
        st.next_codes_chunk(0)
    pre, tr, pad = m.prepare(list(ids), lookahead=8)
    ref, _, recs = m.rollout(pre, tr, pad, 15, GREEDY, GREEDY, forced_codes=codes)
    assert_tokens_match(codes, ref, gaps_per_code(recs))


def test_text_stream_equals_stream(engines, pkg):
    e = engines["tiny"]
    ids = ids_for(8, 24)
    opts = pkg.GenerateOptions(decode_audio=False, max_frames=30, seed=5)
    st = e.start_stream_from_ids(ids, opts, pkg.StreamOptions(text_lookahead_tokens=8))
    whole = []
    while (c := st.next_codes_chunk(7)) is not None:
        whole.extend(c.codes)
    ts = e.start_text_stream_polling(opts, pkg.TextStreamOptions(min_start_tokens=8))
    assert isinstance(ts.next_codes_chunk(4), pkg.NeedMoreText)
    got = []
    fed = 0
    while True:
        r = ts.next_codes_chunk(4)
        if isinstance(r, pkg.NeedMoreText):
            if fed < len(ids):
                ts.push_ids(ids[fed: fed + 8])
                fed += 8
            else:
                ts.finish_text()
            continue
        if isinstance(r, pkg.Finished):
            break
        got.extend(r.codes)
    assert got == whole
    assert ts.finish_codes().codes == whole


def test_text_stream_channel(engines, pkg):
    """start_text_stream's (TextStreamInput, HipTextStream) pair."""
    e = engines["tiny"]
    opts = pkg.GenerateOptions(decode_audio=False, max_frames=5, seed=1)
    inp, stream = pkg.start_text_stream(e, opts, pkg.TextStreamOptions(min_start_tokens=2))
    inp.push_ids([5, 6, 7])
    inp.finish()
    frames = 0
    while (c := stream.next_codes_chunk(2)) is not None:
        frames += c.frames
    assert stream.finished_codes() is not None
    assert frames == stream.finished_codes().frames <= 5


def test_voice_clone_xvector(engines, oracles, pkg):
    e, m = engines["tiny"], oracles["tiny"]
    ids = ids_for(9, 6)
    spk = np.random.default_rng(1).standard_normal(e.hidden).astype(np.float32) * 0.02
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=8)
    out = e.generate_voice_clone_codes_from_ids(ids, spk, opts)
    pre, tr, pad = m.prepare(list(ids))
    cfg = m.cfg["talker_config"]
    pre = pre.clone()  # x-vector replaces the speaker codec row (prefill row 3 + 4)
    pre[7] = pre[7] - m.codec_emb[cfg["spk_id"]["ryan"]] + torch.from_numpy(spk)
    ref, _, recs = m.rollout(pre, tr, pad, 8, GREEDY, GREEDY, forced_codes=out.codes)
    assert_tokens_match(out.codes, ref, gaps_per_code(recs))


def test_generate_from_rows_matches_ids(engines, pkg):
    e = engines["tiny_proj"]
    ids = ids_for(10, 5)
    opts = pkg.GenerateOptions(decode_audio=False, max_frames=6, seed=2)
    a = e.generate_codes_from_ids(ids, opts)
    b = e.generate_codes_from_inputs(e.prepare_inputs_from_ids(ids), opts)
    assert a.codes == b.codes


def test_errors(engines, pkg):
    e = engines["tiny"]
    ids = ids_for(11, 5)
    with pytest.raises(pkg.InvalidInput, match="cache steps"):
        e.generate_codes_from_ids(ids, pkg.GenerateOptions(decode_audio=False, max_frames=200))
    with pytest.raises(pkg.InvalidInput, match="top_p"):
        e.generate_codes_from_ids(ids, pkg.GenerateOptions(decode_audio=False, top_p=0.0))
    with pytest.raises(pkg.InvalidInput, match="temperature"):
        e.generate_codes_from_ids(ids, pkg.GenerateOptions(decode_audio=False,
                                                           subtalker_temperature=0.0))
    with pytest.raises(pkg.InvalidInput, match="repetition_penalty"):
        e.generate_codes_from_ids(ids, pkg.GenerateOptions(decode_audio=False,
                                                           repetition_penalty=0.0))
    with pytest.raises(pkg.InvalidInput, match="out of range"):
        e.generate_codes_from_ids([10**6], pkg.GenerateOptions(decode_audio=False))
    with pytest.raises(pkg.Error, match="codec"):  # no speech_tokenizer/ here
        e.decode_codes([0] * 16)
    out = e.generate_codes_from_ids(ids, pkg.GenerateOptions(decode_audio=False, max_frames=2))
    assert out.frames == 2


def test_bounded_device_wait_reports_expiry(engines, pkg):
    """A device wait on a counter nothing increments runs out after its bound
    (0.2 s here) and the host gets the device-state error; the engine keeps
    working afterwards."""
    import time

    e = engines["tiny"]
    t0 = time.perf_counter()
    with pytest.raises(pkg.CudaError, match="bounded device wait ran out") as info:
        e.selftest_device_wait(200_000)
    assert info.value.code == pkg.engine.ERR_DEVICE_STATE
    assert 0.15 < time.perf_counter() - t0 < 5.0
    out = e.generate_codes_from_ids(ids_for(15, 5), pkg.GenerateOptions(decode_audio=False,
                                                                       max_frames=2))
    assert out.frames == 2


def _scale_codec_head_row(src, dst, row, scale):
    """Copies a synthetic checkpoint with one codec_head row scaled."""
    shutil.copytree(src, dst)
    p = dst / "model.safetensors"
    raw = bytearray(p.read_bytes())
    (n,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8: 8 + n])
    meta = hdr["talker.codec_head.weight"]
    H = meta["shape"][1]
    off = 8 + n + meta["data_offsets"][0] + row * H * 2
    vals = synth.bf16_bits_to_f32(np.frombuffer(bytes(raw[off: off + 2 * H]), np.uint16))
    raw[off: off + 2 * H] = synth.f32_to_bf16_bits(vals * scale).tobytes()
    p.write_bytes(bytes(raw))
    return dst


def test_eos_stops_generation(pkg, model_dirs, oracles, tmp_path):
    """EOS selected on the device halts the queued frames (generation.rs:698-701).
    The EOS row of codec_head is aligned with the hidden state of a later frame
    so that EOS wins there."""
    m0 = oracles["tiny"]
    eos = m0.codec_eos
    ids = ids_for(12, 4)
    pre, tr, pad = m0.prepare(list(ids))
    # talker hidden after a few decode steps (greedy): build EOS row = c * h_k
    m0.talker.reset()
    _, h, lg = m0.talker_prefill(pre)
    d = tmp_path / "eos"
    shutil.copytree(model_dirs["tiny"], d)
    p = d / "model.safetensors"
    raw = bytearray(p.read_bytes())
    (n,) = struct.unpack("<Q", raw[:8])
    meta = json.loads(raw[8: 8 + n])["talker.codec_head.weight"]
    H = meta["shape"][1]
    off = 8 + n + meta["data_offsets"][0] + eos * H * 2
    row = (h / h.norm() * 0.14).numpy().astype(np.float32)
    raw[off: off + 2 * H] = synth.f32_to_bf16_bits(row).tobytes()
    p.write_bytes(bytes(raw))
    m = O.OracleModel(d, 64)
    e = pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 64))
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=20)
    out = e.generate_codes_from_ids(ids, opts)
    print("eos test: frames", out.frames, "ended", out.ended_by_eos)
    codes, ended, recs = m.rollout(pre, tr, pad, 20, GREEDY, GREEDY, forced_codes=out.codes)
    assert out.ended_by_eos == ended
    check_end(m, out.ended_by_eos, "eos test")
    assert out.frames == len(codes) // 16
    assert_tokens_match(out.codes, codes, gaps_per_code(recs))
    if out.ended_by_eos:
        st = e.start_stream_from_ids(ids, opts, pkg.StreamOptions(text_lookahead_tokens=100))
        n = 0
        while (c := st.next_codes_chunk(3)) is not None:
            n += c.frames
        assert n == out.frames and st.finish_codes().ended_by_eos
    # the same model served as a batch: each request halts on its own EOS
    # while the others keep stepping (halted rows are skipped on the device)
    reqs = [ids, ids_for(13, 9), ids_for(14, 6)]
    outs = e.generate_codes_batch_from_ids(reqs, [opts] * len(reqs))
    for r, o in zip(reqs, outs):
        p2, t2, q2 = m.prepare(list(r))
        c2, ended2, rec2 = m.rollout(p2, t2, q2, 20, GREEDY, GREEDY, forced_codes=o.codes)
        assert o.ended_by_eos == ended2
        check_end(m, o.ended_by_eos, "eos batch")
        assert o.frames == len(c2) // 16
        assert_tokens_match(o.codes, c2, gaps_per_code(rec2))
    e.close()


def test_full_size_0p6b(pkg, tmp_path_factory):
    """BASELINE shapes: 0.6B talker + CodePredictor, a few frames, greedy."""
    d = synth.write_model(tmp_path_factory.mktemp("m06"), "0.6b", 0)
    m = O.OracleModel(d, 128)
    e = pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 128))
    ids = np.random.default_rng(0).integers(0, 150000, 32)
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=4)
    out = e.generate_codes_from_ids(ids, opts)
    pre, tr, pad = m.prepare(list(ids))
    assert pre.shape[0] == 41
    _, _, rl = m.talker_prefill(pre)
    _, lg, _ = e.talker_prefill(pre.numpy())
    assert np.abs(lg - rl).max() <= LOGIT_TOL
    codes, _, recs = m.rollout(pre, tr, pad, 4, GREEDY, GREEDY, forced_codes=out.codes)
    assert_tokens_match(out.codes, codes, gaps_per_code(recs))
    # Cross-CTA reductions sum in a fixed order: a sampled run repeats bit for bit.
    s = pkg.GenerateOptions(decode_audio=False, max_frames=8, seed=7)
    a, b = e.generate_codes_from_ids(ids, s), e.generate_codes_from_ids(ids, s)
    assert a.frames == b.frames and list(a.codes) == list(b.codes)
    e.close()


def test_full_size_1p7b(pkg, tmp_path_factory):
    """BASELINE config 3 shapes (1.7B talker, CodePredictor behind the 2048->1024
    projection): prefill logits, two greedy frames teacher-forced against the
    oracle, and a two-request batch through the tensor-core path."""
    d = synth.write_model(tmp_path_factory.mktemp("m17"), "1.7b", 0)
    m = O.OracleModel(d, 128)
    e = pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 128))
    ids = np.random.default_rng(2).integers(0, 150000, 24)
    pre, tr, pad = m.prepare(list(ids))
    _, _, rl = m.talker_prefill(pre)
    _, lg, _ = e.talker_prefill(pre.numpy())
    assert np.abs(lg - rl).max() <= LOGIT_TOL
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=2)
    out = e.generate_codes_from_ids(ids, opts)
    codes, _, recs = m.rollout(pre, tr, pad, 2, GREEDY, GREEDY, forced_codes=out.codes)
    assert_tokens_match(out.codes, codes, gaps_per_code(recs))
    reqs = [ids, np.random.default_rng(3).integers(0, 150000, 40)]
    outs = e.generate_codes_batch_from_ids(reqs, [opts, opts])
    for r, o in zip(reqs, outs):
        p2, t2, q2 = m.prepare(list(r))
        c2, _, rec2 = m.rollout(p2, t2, q2, 2, GREEDY, GREEDY, forced_codes=o.codes)
        assert_tokens_match(o.codes, c2, gaps_per_code(rec2))
    e.close()


@pytest.mark.parametrize("env", [{"QTTS_FUSE_ATTN_O": "0"},
                                 {"QTTS_TC_CP": "1"},
                                 {"QTTS_TC": "0"}],
                         ids=["unfused-cp-attn", "cp-tc-prefill", "cuda-core-prefill"])
def test_alternate_path_parity(model_dirs, tmp_path, env):
    """The alternate paths against the oracle: the CodePredictor attention as
    a separate kernel (QTTS_FUSE_ATTN_O=0), its 2-row prefill on the tcgen05
    GEMM (QTTS_TC_CP=1), and the talker prefill on CUDA cores only
    (QTTS_TC=0). Run in a child process so the engine reads the setting at
    load."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = f"""
import sys, numpy as np
sys.path.insert(0, {str(root)!r})
import __graft_entry__ as G
from oracle import qtts_oracle as O
pkg = G.load_package()
for shape, d in [('tiny', {str(model_dirs['tiny'])!r}), ('tiny_proj', {str(model_dirs['tiny_proj'])!r})]:
    e = pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 128))
    m = O.OracleModel(d, 128)
    ids = np.random.default_rng(3).integers(0, 4000, 10)
    g = O.SamplingConfig(False, 0, 1.0, 1.0)
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=12)
    out = e.generate_codes_from_ids(ids, opts)
    pre, tr, pad = m.prepare(list(ids))
    codes, _, recs = m.rollout(pre, tr, pad, 12, g, g, forced_codes=out.codes)
    gaps = [x for r in recs for x in [r.talker_gap] + r.cp_gaps]
    bad = [i for i, (a, b) in enumerate(zip(out.codes, codes)) if a != b and gaps[i] > 1e-2]
    assert out.frames == 12 and not bad, (shape, bad)
    s = pkg.GenerateOptions(decode_audio=False, max_frames=12, seed=4)
    out2 = e.generate_codes_from_ids(ids, s)
    assert list(e.generate_codes_from_ids(ids, s).codes) == list(out2.codes), shape  # repeatable
    sc = O.SamplingConfig(True, 50, 1.0, 0.9)
    codes2, _, recs2 = m.rollout(pre, tr, pad, 12, sc, sc, penalty=1.05, seed=4, forced_codes=out2.codes)
    ms = [x for r in recs2 for x in [r.talker_margin] + r.cp_margins]
    bad2 = [i for i, (a, b) in enumerate(zip(out2.codes, codes2)) if a != b and ms[i] > 5e-3]
    assert not bad2, (shape, bad2)
print("alternate path ok")
"""
    env = dict(os.environ, **env)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "alternate path ok" in r.stdout, r.stdout + r.stderr
