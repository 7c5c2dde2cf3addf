"""Codec decoder (HipCodecInitial, src/audio/codec_hip.rs) on the B200 against
the fp32 CPU restatement in oracle/codec.py, through the C ABI
(qtts_decode_codes). Both sides compute in fp32; the tolerance covers
summation-order differences through the ~60-layer stack."""
import numpy as np
import pytest

from oracle import codec as K
from oracle import synth

pytestmark = pytest.mark.gpu

WAVE_TOL = 2e-3  # max abs difference of the waveform (values in [-1, 1], std ~0.25)


@pytest.fixture(scope="module")
def codec_model(tmp_path_factory):
    d = tmp_path_factory.mktemp("codec_model") / "tiny_codec"
    synth.write_model(d, "tiny", 0)
    tensors = K.write_codec(d, 0)
    return d, K.CodecOracle(tensors)


@pytest.fixture(scope="module")
def codec_engine(pkg, codec_model):
    d, _ = codec_model
    e = pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 128))
    yield e
    e.close()


@pytest.mark.parametrize("frames,seed", [(1, 0), (6, 1), (40, 2)])
def test_decode_matches_oracle(codec_engine, codec_model, frames, seed):
    _, oracle = codec_model
    assert codec_engine.has_codec and codec_engine.samples_per_code_frame == 1920
    codes = np.random.default_rng(seed).integers(0, 2048, (frames, 16)).astype(np.int32)
    got = codec_engine.decode_codes(codes.reshape(-1))
    ref = oracle.decode(codes.reshape(-1))
    assert got.shape == ref.shape == (frames * 1920,)
    err = float(np.max(np.abs(got - ref)))
    assert err <= WAVE_TOL, err


def test_codes_taken_modulo_codebook(codec_engine, codec_model):
    """codec_rvq_project_f32 reduces every code modulo 2048 (negative codes too)."""
    _, oracle = codec_model
    codes = np.random.default_rng(5).integers(-4096, 8192, (3, 16)).astype(np.int32)
    got = codec_engine.decode_codes(codes.reshape(-1))
    np.testing.assert_allclose(got, codec_engine.decode_codes((codes % 2048).reshape(-1)),
                               atol=0, rtol=0)
    assert np.max(np.abs(got - oracle.decode(codes.reshape(-1)))) <= WAVE_TOL


def test_decode_is_deterministic(codec_engine):
    codes = np.random.default_rng(6).integers(0, 2048, 16 * 8).astype(np.int32)
    a = codec_engine.decode_codes(codes)
    b = codec_engine.decode_codes(codes)
    assert np.array_equal(a, b)


def test_generate_and_stream_audio(pkg, codec_engine):
    """generate with decode_audio = decode_codes(codes); stream audio chunks are
    the chunk's window decoded with up to left_context_frames of context, the
    context samples dropped (generation.rs:965-989)."""
    ids = np.random.default_rng(7).integers(0, 4000, 12)
    opts = pkg.GenerateOptions(decode_audio=True, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=9)
    sp = codec_engine.generate_from_ids(ids, opts)
    assert sp.frames > 0 and sp.sample_rate == 24000
    assert np.array_equal(sp.samples, codec_engine.decode_codes(sp.codes))

    st = codec_engine.start_stream_from_ids(
        ids, opts, pkg.StreamOptions(text_lookahead_tokens=8, left_context_frames=2))
    chunks = []
    while True:
        ch = st.next_audio_chunk(3)
        if ch is None:
            break
        chunks.append(ch)
    codes = st.finish_codes().codes
    st.close()
    assert chunks and sum(c.frames for c in chunks) * 16 == len(codes)
    for c in chunks:
        start = c.total_frames - c.frames
        ctx = min(2, start)
        window = codec_engine.decode_codes(codes[(start - ctx) * 16: c.total_frames * 16])
        assert c.samples.shape == (c.frames * 1920,)
        assert np.array_equal(c.samples, window[ctx * 1920:])


def test_decode_errors(pkg, codec_engine, model_dirs):
    with pytest.raises(pkg.InvalidInput, match="divisible"):
        codec_engine.decode_codes(np.zeros(17, np.int32))
    assert codec_engine.decode_codes([]).size == 0
    # no speech_tokenizer/ in this model directory: codes still generate, audio does not
    tiny = pkg.HipTtsEngine.load_with_options(model_dirs["tiny"], pkg.EngineOptions(0, 128))
    try:
        assert not tiny.has_codec
        with pytest.raises(pkg.Error, match="codec"):
            tiny.decode_codes(np.zeros(16, np.int32))
        with pytest.raises(pkg.Error, match="codec"):
            tiny.generate_from_ids([1, 2, 3], pkg.GenerateOptions(decode_audio=True, max_frames=2))
        out = tiny.generate_from_ids([1, 2, 3], pkg.GenerateOptions(decode_audio=False, max_frames=2))
        assert out.frames == 2 and out.samples.size == 0
    finally:
        tiny.close()


def test_server_shell_streams_the_engine(pkg, codec_engine):
    """The HTTP shell over the real engine: /api/stream sends one s16le chunk
    per audio chunk, equal to the Python stream's chunks for the same request;
    /api/generate's WAV holds decode_codes of the generated codes."""
    import threading

    from qwen3_tts_hip_b200 import server as S
    from test_server import _raw_chunks, _post

    srv = S.TtsServer(codec_engine, "127.0.0.1:0", max_cache_frames=64, log=lambda *_: None)
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    try:
        ids = np.random.default_rng(8).integers(0, 4000, 10)
        form = ("ids=" + ",".join(str(i) for i in ids) +
                "&max_frames=7&stream_chunk_frames=3&left_context_frames=2&seed=3&"
                "text_lookahead_tokens=4")
        _, chunks = _raw_chunks(srv, form)
        opts = pkg.GenerateOptions(decode_audio=False, max_frames=7, seed=3)
        st = codec_engine.start_stream_from_ids(
            ids, opts, pkg.StreamOptions(text_lookahead_tokens=4, left_context_frames=2))
        want = []
        while (ch := st.next_audio_chunk(3)) is not None:
            want.append(S.pcm16(ch.samples, 1.0))
        st.close()
        assert chunks == want and len(chunks) >= 1
        wav = _post(srv, "/api/generate", "ids=" + ",".join(str(i) for i in ids) +
                    "&max_frames=5&seed=3").read()
        gen = codec_engine.generate_codes_from_ids(
            ids, pkg.GenerateOptions(decode_audio=False, max_frames=5, seed=3))
        assert wav[44:] == S.pcm16(codec_engine.decode_codes(gen.codes), 1.0)
    finally:
        srv.shutdown()
        srv.server_close()


STREAM_TOL = 2e-3  # chunked vs one-shot: same arithmetic per output, summation order may differ


@pytest.mark.parametrize("chunks", [[1, 1, 1, 1, 1, 1, 1, 1], [6, 6, 6, 6, 6], [3, 7, 1, 12, 2]])
def test_codec_stream_equals_one_shot(codec_engine, codec_model, chunks):
    """A codec stream with carried state (every causal convolution's history,
    the pre-transformer's keys / values) decodes chunk by chunk to the samples
    of one decode of all the frames, and so to the oracle's."""
    _, oracle = codec_model
    total = sum(chunks)
    codes = np.random.default_rng(11 + total).integers(0, 2048, (total, 16)).astype(np.int32)
    whole = codec_engine.decode_codes(codes.reshape(-1))
    cs = codec_engine.open_codec_stream(total)
    try:
        parts, at = [], 0
        for n in chunks:
            out = cs.decode(codes[at: at + n].reshape(-1))
            assert out.shape == (n * 1920,)
            parts.append(out)
            at += n
    finally:
        cs.close()
    got = np.concatenate(parts)
    err = float(np.max(np.abs(got - whole)))
    assert err <= STREAM_TOL, err
    assert float(np.max(np.abs(got - oracle.decode(codes.reshape(-1))))) <= WAVE_TOL


def test_codec_stream_capacity_and_errors(pkg, codec_engine):
    cs = codec_engine.open_codec_stream(4)
    try:
        assert cs.decode(np.zeros(3 * 16, np.int32)).size == 3 * 1920
        with pytest.raises(pkg.InvalidInput, match="holds 4 frames"):
            cs.decode(np.zeros(2 * 16, np.int32))
        with pytest.raises(pkg.InvalidInput, match="divisible"):
            cs.decode(np.zeros(17, np.int32))
        assert cs.decode([]).size == 0
        assert cs.decode(np.zeros(16, np.int32)).size == 1920  # the last frame still fits
    finally:
        cs.close()
    with pytest.raises(pkg.InvalidInput, match="max_frames"):
        codec_engine.open_codec_stream(0)


def test_stream_audio_with_carried_state(pkg, codec_engine):
    """StreamOptions(carry_codec_state=True): each audio chunk decodes only its
    own frames on the stream's codec state; the chunks join to decode_codes of
    all the stream's codes."""
    ids = np.random.default_rng(9).integers(0, 4000, 12)
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=11)
    st = codec_engine.start_stream_from_ids(
        ids, opts, pkg.StreamOptions(text_lookahead_tokens=8, carry_codec_state=True))
    chunks = []
    while (ch := st.next_audio_chunk(4)) is not None:
        assert ch.samples.shape == (ch.frames * 1920,)
        chunks.append(ch.samples)
    codes = st.finish_codes().codes
    st.close()
    whole = codec_engine.decode_codes(codes)
    assert float(np.max(np.abs(np.concatenate(chunks) - whole))) <= STREAM_TOL
