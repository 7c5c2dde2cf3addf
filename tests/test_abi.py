"""The C-ABI library loads and exports every symbol include/qtts_b200.h declares
(no compute calls: runs without a GPU)."""
import ctypes
import re
from pathlib import Path

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
