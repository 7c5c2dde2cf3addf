"""The C-ABI library loads and exports every symbol include/qtts_b200.h declares
(no compute calls: runs without a GPU)."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "qtts_b200.h").read_text()
    return sorted(set(re.findall(r"\b(qtts_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree(pkg):
    names = declared_symbols()
    assert len(names) >= 25
    assert sorted(pkg.SIGNATURES) == names


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(str(pkg.library_path()))
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_defaults_match_reference(pkg):
    L = pkg.lib()
    from qwen3_tts_hip_b200.engine import _Options, _StreamOptions, _TextStreamOptions

    o = _Options()
    L.qtts_generate_options_default(ctypes.byref(o))
    assert (o.max_frames, o.do_sample, o.top_k, o.top_p) == (240, 1, 50, 1.0)
    assert o.temperature == pytest.approx(0.9) and o.repetition_penalty == pytest.approx(1.05)
    assert (o.subtalker_dosample, o.subtalker_top_k) == (1, 50)
    assert o.speaker == b"ryan" and o.language == b"english"
    s = _StreamOptions()
    L.qtts_stream_options_default(ctypes.byref(s))
    assert (s.text_lookahead_tokens, s.left_context_frames) == (8, 25)
    t = _TextStreamOptions()
    L.qtts_text_stream_options_default(ctypes.byref(t))
    assert (t.min_start_tokens, t.min_resume_tokens, t.flush_on_punctuation) == (8, 1, 1)
    py = pkg.GenerateOptions()
    assert (py.max_frames, py.top_k, py.temperature, py.seed) == (240, 50, 0.9, 0)


def test_load_errors_are_invalid_input(pkg, tmp_path):
    with pytest.raises(pkg.InvalidInput, match="failed to read"):
        pkg.HipTtsEngine.load(tmp_path / "missing", 0)
    (tmp_path / "config.json").write_text("{not json")
    with pytest.raises(pkg.InvalidInput, match="failed to parse"):
        pkg.HipTtsEngine.load(tmp_path, 0)
    with pytest.raises(pkg.InvalidInput, match="max_frames must be non-zero"):
        pkg.HipTtsEngine.load_with_max_frames(tmp_path, 0, 0)


def test_text_stream_input_semantics(pkg):
    # generation.rs:1453-1492: pushes then finish; push after finish fails.
    sink = []
    inp = pkg.TextStreamInput(sink)
    inp.push_ids([1, 2])
    inp.finish()
    assert sink == [("ids", [1, 2]), ("finish", None)]
    with pytest.raises(pkg.InvalidInput):
        inp.push_ids([3])


def test_audio_chunk_window(pkg):
    """next_audio_chunk's window (generation.rs:965-989) on the host: the chunk's
    frames plus min(left_context, start) earlier frames are decoded and the
    context's samples dropped. A stub decoder stands in for the codec."""
    spf = 4

    class Stub:
        code_groups = 2
        samples_per_code_frame = spf
        calls = []

        def decode_codes(self, codes):
            self.calls.append(list(codes))
            frames = len(codes) // self.code_groups
            # sample k of frame f encodes (first code of the frame, k)
            return np.array([codes[f * 2] * 10 + k for f in range(frames) for k in range(spf)],
                            dtype=np.float32)

    stub = Stub()
    all_codes = [f for f in range(7) for _ in range(2)]  # frame f's codes are (f, f)
    for start, n, ctx in [(0, 3, 2), (3, 2, 2), (5, 2, 25), (1, 1, 0)]:
        chunk = pkg.GeneratedCodesChunk(all_codes[start * 2:(start + n) * 2], n, start + n, False)
        out = pkg.HipTtsEngine._audio_chunk(stub, all_codes, chunk, ctx)
        used = min(ctx, start)
        assert stub.calls[-1] == all_codes[(start - used) * 2:(start + n) * 2]
        want = [f * 10 + k for f in range(start, start + n) for k in range(spf)]
        assert out.samples.tolist() == want
        assert (out.frames, out.total_frames, out.sample_rate) == (n, start + n, 24000)
