"""Python mirror of the reference's public API over the qtts_b200 C ABI.

Names, fields, defaults and error behaviour follow piedshag/qwen3-tts-hip's
``src/generation.rs`` (``HipTtsEngine``, ``GenerateOptions``, ``StreamOptions``,
``TextStreamOptions``, ``GeneratedCodes``, ``GeneratedCodesChunk``) and
``src/error.rs`` (``InvalidInput``).  Text arrives as content token ids
(the caller tokenises): ``generate_codes_from_ids`` / ``push_ids`` are the
id-based forms of ``generate_codes`` / ``push_text``.  The codec decoder
(``decode_codes``, ``generate_from_ids`` with ``decode_audio``,
``next_audio_chunk``) runs when the model directory holds
``speech_tokenizer/model.safetensors``.

All compute runs in ``libqtts_b200.so`` (sm_100a); loading fails loudly when the
library is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import List, Optional, Sequence

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "libqtts_b200.so"
_lib = None

# qtts_status values (include/qtts_b200.h)
OK, ERR_INVALID_INPUT, ERR_CUDA, ERR_CACHE_FULL, ERR_IO, ERR_UNSUPPORTED, ERR_DEVICE_STATE = range(7)
CHUNK, CHUNK_NONE, NEED_MORE_TEXT, FINISHED = range(4)

SAMPLE_RATE = 24_000
DEFAULT_MAX_CACHE_STEPS = 512
DEFAULT_PREFILL_HEADROOM = 256
DEFAULT_STREAM_LEFT_CONTEXT_FRAMES = 25
DEFAULT_TEXT_LOOKAHEAD_TOKENS = 8


class Error(RuntimeError):
    """Error of the reference (src/error.rs)."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class InvalidInput(Error, ValueError):
    pass


class CudaError(Error):
    pass


class _Options(C.Structure):
    _fields_ = [
        ("speaker", C.c_char_p), ("language", C.c_char_p), ("max_frames", C.c_uint32),
        ("decode_audio", C.c_int32), ("do_sample", C.c_int32), ("top_k", C.c_uint32),
        ("top_p", C.c_float), ("temperature", C.c_float), ("repetition_penalty", C.c_float),
        ("subtalker_dosample", C.c_int32), ("subtalker_top_k", C.c_uint32),
        ("subtalker_top_p", C.c_float), ("subtalker_temperature", C.c_float),
        ("seed", C.c_uint64), ("rng", C.c_int32),
    ]


class _StreamOptions(C.Structure):
    _fields_ = [("text_lookahead_tokens", C.c_uint32), ("left_context_frames", C.c_uint32)]


class _TextStreamOptions(C.Structure):
    _fields_ = [("min_start_tokens", C.c_uint32), ("min_resume_tokens", C.c_uint32),
                ("flush_on_punctuation", C.c_int32), ("left_context_frames", C.c_uint32)]


class _Chunk(C.Structure):
    _fields_ = [("frames", C.c_size_t), ("total_frames", C.c_size_t),
                ("ended_by_eos", C.c_int32), ("status", C.c_int32)]


class _TraceLaunch(C.Structure):
    _fields_ = [("name", C.c_char * 48), ("entry_ns", C.c_int64), ("wait_ns", C.c_int64),
                ("exit_ns", C.c_int64), ("last_wait_ns", C.c_int64), ("mark4_ns", C.c_int64),
                ("mark5_ns", C.c_int64), ("dur6_ns", C.c_uint64), ("dur7_ns", C.c_uint64)]


class _Info(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("vocab", C.c_uint32), ("cp_hidden", C.c_uint32),
                ("cp_vocab", C.c_uint32), ("num_code_groups", C.c_uint32),
                ("talker_layers", C.c_uint32), ("cp_layers", C.c_uint32),
                ("codec_eos", C.c_uint32), ("max_cache_steps", C.c_size_t),
                ("device_bytes", C.c_size_t), ("reserved", C.c_int32 * 2),
                ("has_codec", C.c_int32), ("samples_per_frame", C.c_uint32)]


# Exported symbols and their signatures (mirrors include/qtts_b200.h).
_P = C.c_void_p
_F = C.POINTER(C.c_float)
_I32 = C.POINTER(C.c_int32)
_U32 = C.POINTER(C.c_uint32)
_SZ = C.POINTER(C.c_size_t)
SIGNATURES = {
    "qtts_last_error": (C.c_char_p, []),
    "qtts_abi_version": (C.c_int32, []),
    "qtts_generate_options_default": (None, [C.POINTER(_Options)]),
    "qtts_stream_options_default": (None, [C.POINTER(_StreamOptions)]),
    "qtts_text_stream_options_default": (None, [C.POINTER(_TextStreamOptions)]),
    "qtts_engine_load": (C.c_int32, [C.c_char_p, C.c_int32, C.POINTER(_P)]),
    "qtts_engine_load_with_max_frames": (C.c_int32, [C.c_char_p, C.c_int32, C.c_size_t, C.POINTER(_P)]),
    "qtts_engine_load_with_options": (C.c_int32, [C.c_char_p, C.c_int32, C.c_size_t, C.POINTER(_P)]),
    "qtts_engine_destroy": (None, [_P]),
    "qtts_engine_get_info": (C.c_int32, [_P, C.POINTER(_Info)]),
    "qtts_decode_codes": (C.c_int32, [_P, _I32, C.c_size_t, _F, C.c_size_t, _SZ]),
    "qtts_last_decode_timing": (C.c_int32, [_P, _F, _SZ]),
    "qtts_codec_stream_open": (C.c_int32, [_P, C.c_size_t, C.POINTER(_P)]),
    "qtts_codec_stream_decode": (C.c_int32, [_P, _I32, C.c_size_t, _F, C.c_size_t, _SZ]),
    "qtts_codec_stream_destroy": (None, [_P]),
    "qtts_generate_codes_from_ids": (C.c_int32, [_P, _U32, C.c_size_t, C.POINTER(_Options), _I32, C.c_size_t, _SZ, _I32]),
    "qtts_generate_codes_batch_from_ids": (C.c_int32, [_P, _U32, _SZ, C.c_size_t, C.POINTER(_Options), _I32, C.c_size_t, _SZ, _I32]),
    "qtts_generate_voice_clone_codes_from_ids": (C.c_int32, [_P, _U32, C.c_size_t, _F, C.POINTER(_Options), _I32, C.c_size_t, _SZ, _I32]),
    "qtts_generate_codes_from_rows": (C.c_int32, [_P, _F, C.c_size_t, _F, C.c_size_t, _F, C.POINTER(_Options), _I32, C.c_size_t, _SZ, _I32]),
    "qtts_prepare_inputs_from_ids": (C.c_int32, [_P, _U32, C.c_size_t, C.c_size_t, C.c_char_p, C.c_char_p, _F, _SZ, _F, _SZ, _F]),
    "qtts_stream_start_from_ids": (C.c_int32, [_P, _U32, C.c_size_t, C.POINTER(_Options), C.POINTER(_StreamOptions), C.POINTER(_P)]),
    "qtts_stream_next_codes_chunk": (C.c_int32, [_P, C.c_size_t, _I32, C.c_size_t, C.POINTER(_Chunk)]),
    "qtts_stream_destroy": (None, [_P]),
    "qtts_text_stream_start": (C.c_int32, [_P, C.POINTER(_Options), C.POINTER(_TextStreamOptions), C.POINTER(_P)]),
    "qtts_text_stream_push_ids": (C.c_int32, [_P, _U32, C.c_size_t]),
    "qtts_text_stream_finish": (C.c_int32, [_P]),
    "qtts_text_stream_next_codes_chunk": (C.c_int32, [_P, C.c_size_t, _I32, C.c_size_t, C.POINTER(_Chunk)]),
    "qtts_text_stream_codes": (C.c_int32, [_P, _I32, C.c_size_t, _SZ, _I32]),
    "qtts_text_stream_destroy": (None, [_P]),
    "qtts_talker_prefill": (C.c_int32, [_P, _F, C.c_size_t, _F, _F, _I32]),
    "qtts_talker_decode_step": (C.c_int32, [_P, _F, C.c_size_t, _F, _F, _I32]),
    "qtts_talker_decode_step_static": (C.c_int32, [_P, _F, C.c_size_t, _F, _F, _I32]),
    "qtts_code_predictor": (C.c_int32, [_P, _F, _F, C.POINTER(_Options), _I32, _F, _F]),
    "qtts_selftest_device_wait": (C.c_int32, [_P, C.c_uint32]),
    "qtts_step_trace_enable": (C.c_int32, [_P, C.c_int32]),
    "qtts_step_trace_read": (C.c_int32, [_P, C.POINTER(_TraceLaunch), C.c_size_t, _SZ]),
    "qtts_last_timings": (C.c_int32, [_P, _F, _F, _SZ]),
    "qtts_last_launch_count": (C.c_int32, [_P, _SZ]),
    "qtts_profile_projection": (C.c_int32, [_P, C.c_int32, C.c_int32, _F, C.POINTER(C.c_double)]),
}


def library_path() -> Path:
    return _LIB_PATH


def lib():
    """Loads libqtts_b200.so (built in-tree by ``build()``); raises if absent."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise ImportError(f"{_LIB_PATH} is missing: run __graft_entry__.build() first")
        L = C.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status == OK:
        return
    msg = lib().qtts_last_error().decode(errors="replace")
    if status in (ERR_INVALID_INPUT, ERR_CACHE_FULL):
        raise InvalidInput(status, msg)
    if status in (ERR_CUDA, ERR_DEVICE_STATE):
        raise CudaError(status, msg)
    raise Error(status, msg)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _ids(ids) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(ids, dtype=np.uint32).reshape(-1))


# ---------------------------------------------------------------------------
@dataclass
class EngineOptions:
    """EngineOptions (generation.rs:25-38)."""
    device: int = 0
    max_cache_steps: int = DEFAULT_MAX_CACHE_STEPS


@dataclass
class GenerateOptions:
    """GenerateOptions (generation.rs:40-77); ``rng`` selects the reference's
    LCG draw order ("lcg", default) or Philox-4x32-10 ("philox")."""
    speaker: str = "ryan"
    language: str = "english"
    max_frames: int = 240
    decode_audio: bool = True
    do_sample: bool = True
    top_k: int = 50
    top_p: float = 1.0
    temperature: float = 0.9
    repetition_penalty: float = 1.05
    subtalker_dosample: bool = True
    subtalker_top_k: int = 50
    subtalker_top_p: float = 1.0
    subtalker_temperature: float = 0.9
    seed: int = 0
    rng: str = "lcg"

    def _c(self) -> _Options:
        if self.rng not in ("lcg", "philox"):
            raise InvalidInput(ERR_INVALID_INPUT, f"unknown rng {self.rng}")
        self._keep = (self.speaker.encode(), self.language.encode())
        return _Options(self._keep[0], self._keep[1], int(self.max_frames), int(bool(self.decode_audio)),
                        int(bool(self.do_sample)), int(self.top_k), float(self.top_p),
                        float(self.temperature), float(self.repetition_penalty),
                        int(bool(self.subtalker_dosample)), int(self.subtalker_top_k),
                        float(self.subtalker_top_p), float(self.subtalker_temperature),
                        int(self.seed) & ((1 << 64) - 1), 0 if self.rng == "lcg" else 1)


@dataclass
class StreamOptions:
    """StreamOptions (generation.rs:79-92)."""
    text_lookahead_tokens: int = DEFAULT_TEXT_LOOKAHEAD_TOKENS
    left_context_frames: int = DEFAULT_STREAM_LEFT_CONTEXT_FRAMES
    # False: audio chunks re-decode left_context_frames earlier frames, as the
    # reference does. True: a CodecStream carries the decoder state, so a
    # chunk decodes only its own frames (samples equal a one-shot decode).
    carry_codec_state: bool = False


@dataclass
class TextStreamOptions:
    """TextStreamOptions (generation.rs:211-228)."""
    min_start_tokens: int = DEFAULT_TEXT_LOOKAHEAD_TOKENS
    min_resume_tokens: int = 1
    flush_on_punctuation: bool = True
    left_context_frames: int = DEFAULT_STREAM_LEFT_CONTEXT_FRAMES
    carry_codec_state: bool = False  # as StreamOptions.carry_codec_state


@dataclass
class GeneratedCodes:
    """GeneratedCodes (generation.rs:1519-1523): codes frame-major [frames*16]."""
    codes: list
    frames: int
    ended_by_eos: bool


@dataclass
class GeneratedSpeech:
    """GeneratedSpeech (generation.rs:1494-1530) without the text field:
    codes plus the decoded waveform (empty unless decode_audio)."""
    codes: list
    frames: int
    ended_by_eos: bool
    samples: np.ndarray
    sample_rate: int = SAMPLE_RATE


@dataclass
class GeneratedAudioChunk:
    """GeneratedAudioChunk (generation.rs:246-252)."""
    samples: np.ndarray
    sample_rate: int
    frames: int
    total_frames: int
    ended_by_eos: bool


@dataclass
class GeneratedCodesChunk:
    """GeneratedCodesChunk (generation.rs:238-244)."""
    codes: list
    frames: int
    total_frames: int
    ended_by_eos: bool


@dataclass
class TtsPreparedInputs:
    """TtsPreparedInputs (text.rs:17-26), rows as float32 arrays."""
    prefill: np.ndarray
    prefill_steps: int
    trailing_text: np.ndarray
    trailing_steps: int
    tts_pad_embed: np.ndarray


class NeedMoreText:
    """IncrementalAudio::NeedMoreText (generation.rs:230-236)."""


@dataclass
class Finished:
    """IncrementalAudio::Finished."""
    codes: GeneratedCodes


class HipTtsEngine:
    """HipTtsEngine (generation.rs:133-143, 254-651) on one B200."""

    def __init__(self, handle, model_dir):
        self._h = handle
        self._model_dir = Path(model_dir)
        info = _Info()
        _check(lib().qtts_engine_get_info(self._h, C.byref(info)))
        self.info = info
        self.code_groups = info.num_code_groups
        self.hidden = info.hidden

    # ---- loading (generation.rs:254-315)
    @classmethod
    def load(cls, model_dir, device: int = 0) -> "HipTtsEngine":
        h = C.c_void_p()
        _check(lib().qtts_engine_load(str(model_dir).encode(), int(device), C.byref(h)))
        return cls(h, model_dir)

    @classmethod
    def load_with_max_frames(cls, model_dir, device: int, max_frames: int) -> "HipTtsEngine":
        h = C.c_void_p()
        _check(lib().qtts_engine_load_with_max_frames(str(model_dir).encode(), int(device),
                                                      int(max_frames), C.byref(h)))
        return cls(h, model_dir)

    @classmethod
    def load_with_options(cls, model_dir, options: EngineOptions) -> "HipTtsEngine":
        h = C.c_void_p()
        _check(lib().qtts_engine_load_with_options(str(model_dir).encode(), int(options.device),
                                                   int(options.max_cache_steps), C.byref(h)))
        return cls(h, model_dir)

    def close(self) -> None:
        if self._h:
            lib().qtts_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def model_dir(self) -> Path:
        return self._model_dir

    @property
    def max_cache_steps(self) -> int:
        return self.info.max_cache_steps

    # ---- generation
    def _codes_buf(self, options: GenerateOptions) -> np.ndarray:
        return np.zeros(max(1, options.max_frames) * self.code_groups, dtype=np.int32)

    def generate_codes_from_ids(self, content_ids: Sequence[int],
                                options: Optional[GenerateOptions] = None) -> GeneratedCodes:
        """generate_codes (generation.rs:356-371) for already-tokenised content."""
        options = options or GenerateOptions(decode_audio=False)
        ids = _ids(content_ids)
        out = self._codes_buf(options)
        frames, ended = C.c_size_t(), C.c_int32()
        _check(lib().qtts_generate_codes_from_ids(
            self._h, ids.ctypes.data_as(_U32), ids.size, C.byref(options._c()),
            out.ctypes.data_as(_I32), out.size, C.byref(frames), C.byref(ended)))
        n = frames.value * self.code_groups
        return GeneratedCodes(out[:n].tolist(), frames.value, bool(ended.value))

    def generate_codes_batch_from_ids(self, requests: Sequence[Sequence[int]],
                                      options: Sequence[GenerateOptions]) -> List[GeneratedCodes]:
        """Batched serving (no reference counterpart): up to 16 requests
        generated together; options may differ only in seed, speaker and
        language. Returns one GeneratedCodes per request."""
        reqs = [_ids(r) for r in requests]
        if len(options) != len(reqs):
            raise InvalidInput(ERR_INVALID_INPUT, "one GenerateOptions per request")
        ids = np.concatenate(reqs) if reqs else np.zeros(0, np.uint32)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        lens = np.array([r.size for r in reqs], dtype=np.uintp)
        opts = (_Options * len(reqs))(*[o._c() for o in options])
        cap = max(1, max((o.max_frames for o in options), default=1)) * self.code_groups
        out = np.zeros(len(reqs) * cap, dtype=np.int32)
        frames = np.zeros(len(reqs), dtype=np.uintp)
        ended = np.zeros(len(reqs), dtype=np.int32)
        _check(lib().qtts_generate_codes_batch_from_ids(
            self._h, ids.ctypes.data_as(_U32), lens.ctypes.data_as(_SZ), len(reqs), opts,
            out.ctypes.data_as(_I32), cap, frames.ctypes.data_as(_SZ), ended.ctypes.data_as(_I32)))
        res = []
        for b in range(len(reqs)):
            n = int(frames[b]) * self.code_groups
            res.append(GeneratedCodes(out[b * cap: b * cap + n].tolist(), int(frames[b]),
                                      bool(ended[b])))
        return res

    def generate_voice_clone_codes_from_ids(self, content_ids, speaker_embedding,
                                            options: Optional[GenerateOptions] = None) -> GeneratedCodes:
        """generate_voice_clone_codes (generation.rs:373-395), x-vector prompts."""
        options = options or GenerateOptions(decode_audio=False)
        ids = _ids(content_ids)
        spk = np.ascontiguousarray(speaker_embedding, dtype=np.float32)
        if spk.size != self.hidden:
            raise InvalidInput(ERR_INVALID_INPUT,
                               f"speaker embedding length {spk.size} does not match hidden {self.hidden}")
        out = self._codes_buf(options)
        frames, ended = C.c_size_t(), C.c_int32()
        _check(lib().qtts_generate_voice_clone_codes_from_ids(
            self._h, ids.ctypes.data_as(_U32), ids.size, _fptr(spk), C.byref(options._c()),
            out.ctypes.data_as(_I32), out.size, C.byref(frames), C.byref(ended)))
        n = frames.value * self.code_groups
        return GeneratedCodes(out[:n].tolist(), frames.value, bool(ended.value))

    def generate_codes_from_inputs(self, inputs: TtsPreparedInputs,
                                   options: Optional[GenerateOptions] = None) -> GeneratedCodes:
        """rollout (generation.rs:657-749) on prepared rows."""
        options = options or GenerateOptions(decode_audio=False)
        pre = np.ascontiguousarray(inputs.prefill, dtype=np.float32)
        tr = np.ascontiguousarray(inputs.trailing_text, dtype=np.float32)
        pad = np.ascontiguousarray(inputs.tts_pad_embed, dtype=np.float32)
        out = self._codes_buf(options)
        frames, ended = C.c_size_t(), C.c_int32()
        _check(lib().qtts_generate_codes_from_rows(
            self._h, _fptr(pre), int(inputs.prefill_steps), _fptr(tr), int(inputs.trailing_steps),
            _fptr(pad), C.byref(options._c()), out.ctypes.data_as(_I32), out.size,
            C.byref(frames), C.byref(ended)))
        n = frames.value * self.code_groups
        return GeneratedCodes(out[:n].tolist(), frames.value, bool(ended.value))

    def generate(self, text, options=None):
        raise Error(ERR_UNSUPPORTED, "text tokenisation is outside this library; "
                                     "use generate_from_ids")

    def generate_from_ids(self, content_ids, options: Optional[GenerateOptions] = None
                          ) -> GeneratedSpeech:
        """generate (generation.rs:317-334) from content ids: codes, then the
        waveform when options.decode_audio and any frames were produced."""
        options = options or GenerateOptions()
        c = self.generate_codes_from_ids(content_ids, options)
        samples = (self.decode_codes(c.codes) if options.decode_audio and c.codes
                   else np.zeros(0, np.float32))
        return GeneratedSpeech(c.codes, c.frames, c.ended_by_eos, samples)

    @property
    def has_codec(self) -> bool:
        return bool(self.info.has_codec)

    @property
    def samples_per_code_frame(self) -> int:
        """HipCodecInitial::samples_per_code_frame (codec_hip.rs:203-212)."""
        return int(self.info.samples_per_frame)

    def decode_codes(self, codes) -> np.ndarray:
        """decode_codes (generation.rs:619-646): codes [frames*16] -> 24 kHz samples."""
        a = np.ascontiguousarray(np.asarray(codes, dtype=np.int32).reshape(-1))
        n = a.size // self.code_groups * self.samples_per_code_frame if a.size % self.code_groups == 0 else 0
        out = np.zeros(max(1, n), dtype=np.float32)
        got = C.c_size_t()
        _check(lib().qtts_decode_codes(self._h, a.ctypes.data_as(_I32), a.size,
                                       out.ctypes.data_as(_F), n, C.byref(got)))
        return out[: got.value]

    def last_decode_timing(self):
        """(device ms, kernel launches) of the last decode_codes call."""
        ms, n = C.c_float(), C.c_size_t()
        _check(lib().qtts_last_decode_timing(self._h, C.byref(ms), C.byref(n)))
        return float(ms.value), int(n.value)

    def open_codec_stream(self, max_frames: int) -> "CodecStream":
        """A streaming codec decode of up to max_frames frames with carried state."""
        h = C.c_void_p()
        _check(lib().qtts_codec_stream_open(self._h, int(max_frames), C.byref(h)))
        return CodecStream(self, h)

    def _audio_chunk(self, all_codes: list, chunk: "GeneratedCodesChunk", left_context: int,
                     codec_stream: Optional["CodecStream"] = None) -> GeneratedAudioChunk:
        """next_audio_chunk's window (generation.rs:965-989): decode the chunk
        with up to left_context earlier frames and drop their samples; with a
        codec stream, decode only the chunk's frames on its carried state."""
        if codec_stream is not None:
            return GeneratedAudioChunk(codec_stream.decode(chunk.codes), SAMPLE_RATE, chunk.frames,
                                       chunk.total_frames, chunk.ended_by_eos)
        start = chunk.total_frames - chunk.frames
        ctx = min(left_context, start)
        g = self.code_groups
        decoded = self.decode_codes(all_codes[(start - ctx) * g: chunk.total_frames * g])
        skip = min(ctx * self.samples_per_code_frame, decoded.size)
        return GeneratedAudioChunk(decoded[skip:].copy(), SAMPLE_RATE, chunk.frames,
                                   chunk.total_frames, chunk.ended_by_eos)

    def prepare_inputs_from_ids(self, content_ids, lookahead: Optional[int] = None,
                                speaker: str = "ryan", language: str = "english") -> TtsPreparedInputs:
        """prepare_custom_voice_with_lookahead (text.rs:348-382) on the device."""
        ids = _ids(content_ids)
        H = self.hidden
        pre = np.zeros(((9 + ids.size) * H,), dtype=np.float32)
        tr = np.zeros(((ids.size + 1) * H,), dtype=np.float32)
        pad = np.zeros((H,), dtype=np.float32)
        P, T = C.c_size_t(), C.c_size_t()
        _check(lib().qtts_prepare_inputs_from_ids(
            self._h, ids.ctypes.data_as(_U32), ids.size, 0 if lookahead is None else int(lookahead),
            speaker.encode(), language.encode(), _fptr(pre), C.byref(P), _fptr(tr), C.byref(T),
            _fptr(pad)))
        return TtsPreparedInputs(pre[: P.value * H].reshape(P.value, H), P.value,
                                 tr[: T.value * H].reshape(T.value, H), T.value, pad)

    # ---- streams
    def start_stream_from_ids(self, content_ids, options: Optional[GenerateOptions] = None,
                              stream_options: Optional[StreamOptions] = None) -> "HipTtsStream":
        """start_stream (generation.rs:421-440)."""
        options = options or GenerateOptions(decode_audio=False)
        so = stream_options or StreamOptions()
        ids = _ids(content_ids)
        h = C.c_void_p()
        cso = _StreamOptions(int(so.text_lookahead_tokens), int(so.left_context_frames))
        _check(lib().qtts_stream_start_from_ids(self._h, ids.ctypes.data_as(_U32), ids.size,
                                                C.byref(options._c()), C.byref(cso), C.byref(h)))
        return HipTtsStream(self, h, options.max_frames, int(so.left_context_frames),
                            bool(so.carry_codec_state))

    def start_text_stream_polling(self, options: Optional[GenerateOptions] = None,
                                  stream_options: Optional[TextStreamOptions] = None) -> "PollingTextStream":
        """start_text_stream_polling (generation.rs:474-485)."""
        options = options or GenerateOptions(decode_audio=False)
        so = stream_options or TextStreamOptions()
        cso = _TextStreamOptions(int(so.min_start_tokens), int(so.min_resume_tokens),
                                 int(bool(so.flush_on_punctuation)), int(so.left_context_frames))
        h = C.c_void_p()
        _check(lib().qtts_text_stream_start(self._h, C.byref(options._c()), C.byref(cso), C.byref(h)))
        return PollingTextStream(self, h, options.max_frames, int(so.left_context_frames),
                                 bool(so.carry_codec_state))

    # ---- parity seams (talker-prefill-parity / code-predictor-parity)
    def talker_prefill(self, rows: np.ndarray):
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        hidden = np.zeros(self.hidden, np.float32)
        logits = np.zeros(self.info.vocab, np.float32)
        tok = C.c_int32()
        _check(lib().qtts_talker_prefill(self._h, _fptr(rows), rows.shape[0], _fptr(hidden),
                                         _fptr(logits), C.byref(tok)))
        return hidden, logits, tok.value

    def talker_decode_step(self, step_input: np.ndarray, offset: int):
        x = np.ascontiguousarray(step_input, dtype=np.float32)
        hidden = np.zeros(self.hidden, np.float32)
        logits = np.zeros(self.info.vocab, np.float32)
        tok = C.c_int32()
        _check(lib().qtts_talker_decode_step(self._h, _fptr(x), int(offset), _fptr(hidden),
                                             _fptr(logits), C.byref(tok)))
        return hidden, logits, tok.value

    def talker_decode_step_static(self, step_input: np.ndarray, offset: int):
        """talker_decode_step for hosts that may not allocate device memory
        while running: the call allocates nothing. All of its per-call
        activations (input row, QKV, attention output, post-attention row and
        MLP row of every layer) live in the library's 264 KiB static device
        array, which every call shares; overlapping calls race."""
        x = np.ascontiguousarray(step_input, dtype=np.float32)
        hidden = np.zeros(self.hidden, np.float32)
        logits = np.zeros(self.info.vocab, np.float32)
        tok = C.c_int32()
        _check(lib().qtts_talker_decode_step_static(self._h, _fptr(x), int(offset), _fptr(hidden),
                                                    _fptr(logits), C.byref(tok)))
        return hidden, logits, tok.value

    def code_predictor(self, talker_hidden, semantic_embed, options: Optional[GenerateOptions] = None):
        options = options or GenerateOptions(decode_audio=False, subtalker_dosample=False)
        th = np.ascontiguousarray(talker_hidden, dtype=np.float32)
        se = np.ascontiguousarray(semantic_embed, dtype=np.float32)
        na = self.code_groups - 1
        toks = np.zeros(na, np.int32)
        esum = np.zeros(self.hidden, np.float32)
        logits = np.zeros((na, self.info.cp_vocab), np.float32)
        _check(lib().qtts_code_predictor(self._h, _fptr(th), _fptr(se), C.byref(options._c()),
                                         toks.ctypes.data_as(_I32), _fptr(esum), _fptr(logits)))
        return toks.tolist(), esum, logits

    def step_trace_enable(self, on: bool) -> None:
        """Step trace of frame 6 of every generation (recaptures the graphs)."""
        _check(lib().qtts_step_trace_enable(self._h, int(bool(on))))

    def step_trace(self) -> list:
        """The last traced frame's launches in order: dicts of name and the
        globaltimer stamps (ns after the frame's first entry; -1 = none)."""
        n = C.c_size_t()
        _check(lib().qtts_step_trace_read(self._h, None, 0, C.byref(n)))
        rows = (_TraceLaunch * max(1, n.value))()
        _check(lib().qtts_step_trace_read(self._h, rows, n.value, C.byref(n)))
        keys = [f for f, _ in _TraceLaunch._fields_[1:]]
        return [dict(name=r.name.decode(), **{k: int(getattr(r, k)) for k in keys})
                for r in rows[: n.value]]

    def selftest_device_wait(self, limit_us: int) -> None:
        """Runs a bounded device wait that nothing satisfies; raises the
        library's device-state error once the bound expires."""
        _check(lib().qtts_selftest_device_wait(self._h, int(limit_us)))

    def last_timings(self):
        p, f, n = C.c_float(), C.c_float(), C.c_size_t()
        _check(lib().qtts_last_timings(self._h, C.byref(p), C.byref(f), C.byref(n)))
        k = C.c_size_t()
        _check(lib().qtts_last_launch_count(self._h, C.byref(k)))
        return {"prefill_ms": p.value, "frames_ms": f.value, "frames": n.value,
                "kernels": k.value}

    def profile_projection(self, which: int = 0, launches: int = 280):
        """Average device time (ms) and algorithmic bytes of one talker
        projection launch (0 gate|up, 1 QKV, 2 down, 3 O), weights from HBM."""
        ms, b = C.c_float(), C.c_double()
        _check(lib().qtts_profile_projection(self._h, int(which), int(launches), C.byref(ms),
                                             C.byref(b)))
        return ms.value, b.value


class CodecStream:
    """Streaming codec decode with carried state (qtts_codec_stream_*): each
    decode() takes the next frames' codes and returns exactly their samples,
    equal to those of one decode_codes call over the whole stream."""

    def __init__(self, engine: HipTtsEngine, handle):
        self._e, self._h = engine, handle

    def decode(self, codes) -> np.ndarray:
        a = np.ascontiguousarray(np.asarray(codes, dtype=np.int32).reshape(-1))
        g = self._e.code_groups
        n = a.size // g * self._e.samples_per_code_frame if a.size % g == 0 else 0
        out = np.zeros(max(1, n), dtype=np.float32)
        got = C.c_size_t()
        _check(lib().qtts_codec_stream_decode(self._h, a.ctypes.data_as(_I32), a.size,
                                              out.ctypes.data_as(_F), n, C.byref(got)))
        return out[: got.value]

    def close(self):
        if self._h:
            lib().qtts_codec_stream_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class HipTtsStream:
    """HipTtsStream (generation.rs:145-163, 876-997)."""

    def __init__(self, engine: HipTtsEngine, handle, max_frames: int,
                 left_context_frames: int = DEFAULT_STREAM_LEFT_CONTEXT_FRAMES,
                 carry_codec_state: bool = False):
        self._e, self._h = engine, handle
        self._codes: list = []
        self._ended = False
        self._max = max_frames
        self._ctx = left_context_frames
        self._carry = carry_codec_state
        self._codec: Optional[CodecStream] = None

    def _codec_stream(self) -> Optional[CodecStream]:
        if self._carry and self._codec is None:
            self._codec = self._e.open_codec_stream(self._max)
        return self._codec

    def next_audio_chunk(self, max_chunk_frames: int) -> Optional[GeneratedAudioChunk]:
        """next_audio_chunk (generation.rs:965-989)."""
        ch = self.next_codes_chunk(max_chunk_frames)
        return None if ch is None else self._e._audio_chunk(self._codes, ch, self._ctx,
                                                            self._codec_stream())

    def next_codes_chunk(self, max_chunk_frames: int) -> Optional[GeneratedCodesChunk]:
        out = np.zeros(max(1, int(max_chunk_frames)) * self._e.code_groups, dtype=np.int32)
        ch = _Chunk()
        _check(lib().qtts_stream_next_codes_chunk(self._h, int(max_chunk_frames),
                                                  out.ctypes.data_as(_I32), out.size, C.byref(ch)))
        self._ended = bool(ch.ended_by_eos)
        if ch.status != CHUNK:
            return None
        codes = out[: ch.frames * self._e.code_groups].tolist()
        self._codes.extend(codes)
        return GeneratedCodesChunk(codes, ch.frames, ch.total_frames, bool(ch.ended_by_eos))

    def finish_codes(self) -> GeneratedCodes:
        return GeneratedCodes(list(self._codes), len(self._codes) // self._e.code_groups, self._ended)

    def close(self):
        if self._codec is not None:
            self._codec.close()
            self._codec = None
        if self._h:
            lib().qtts_stream_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PollingTextStream:
    """PollingTextStream (generation.rs:1086-1451) fed with token ids."""

    def __init__(self, engine: HipTtsEngine, handle, max_frames: int,
                 left_context_frames: int = DEFAULT_STREAM_LEFT_CONTEXT_FRAMES,
                 carry_codec_state: bool = False):
        self._e, self._h, self._max = engine, handle, max_frames
        self._ctx = left_context_frames
        self._codes: list = []
        self._carry = carry_codec_state
        self._codec: Optional[CodecStream] = None

    def next_audio_chunk(self, max_chunk_frames: int):
        """IncrementalAudio from next_audio_chunk (generation.rs:1121-1181):
        GeneratedAudioChunk (window decoded with left context), NeedMoreText
        or Finished."""
        r = self.next_codes_chunk(max_chunk_frames)
        if not isinstance(r, GeneratedCodesChunk):
            return r
        if self._carry and self._codec is None:
            self._codec = self._e.open_codec_stream(self._max)
        return self._e._audio_chunk(self._codes, r, self._ctx, self._codec)

    def push_ids(self, ids) -> None:
        a = _ids(ids)
        _check(lib().qtts_text_stream_push_ids(self._h, a.ctypes.data_as(_U32), a.size))

    def finish_text(self) -> None:
        _check(lib().qtts_text_stream_finish(self._h))

    def next_codes_chunk(self, max_chunk_frames: int):
        """Returns GeneratedCodesChunk, NeedMoreText or Finished (the codes half
        of next_audio_chunk, generation.rs:1121-1181)."""
        out = np.zeros(max(1, int(max_chunk_frames)) * self._e.code_groups, dtype=np.int32)
        ch = _Chunk()
        _check(lib().qtts_text_stream_next_codes_chunk(self._h, int(max_chunk_frames),
                                                       out.ctypes.data_as(_I32), out.size,
                                                       C.byref(ch)))
        if ch.status == NEED_MORE_TEXT:
            return NeedMoreText()
        if ch.status == FINISHED:
            return Finished(self.finish_codes())
        codes = out[: ch.frames * self._e.code_groups].tolist()
        self._codes.extend(codes)
        return GeneratedCodesChunk(codes, ch.frames, ch.total_frames, bool(ch.ended_by_eos))

    def finish_codes(self) -> GeneratedCodes:
        n, ended = C.c_size_t(), C.c_int32()
        _check(lib().qtts_text_stream_codes(self._h, None, 0, C.byref(n), C.byref(ended)))
        out = np.zeros(max(1, n.value * self._e.code_groups), dtype=np.int32)
        _check(lib().qtts_text_stream_codes(self._h, out.ctypes.data_as(_I32), out.size,
                                            C.byref(n), C.byref(ended)))
        return GeneratedCodes(out[: n.value * self._e.code_groups].tolist(), n.value, bool(ended.value))

    def close(self):
        if self._codec is not None:
            self._codec.close()
            self._codec = None
        if self._h:
            lib().qtts_text_stream_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TextStreamInput:
    """TextStreamInput (generation.rs:1004-1041): host-side channel of id pushes."""

    def __init__(self, sink):
        self._sink = sink
        self.finished = False

    def push_ids(self, ids) -> None:
        if self.finished:
            raise InvalidInput(ERR_INVALID_INPUT, "cannot push text after finish")
        self._sink.append(("ids", list(ids)))

    def finish(self) -> None:
        if self.finished:
            return
        self.finished = True
        self._sink.append(("finish", None))


class HipTextStream:
    """HipTextStream (generation.rs:1059-1084): pulls input messages whenever the
    poller needs more text."""

    def __init__(self, poller: PollingTextStream):
        self._poller = poller
        self._queue: list = []
        self.input = TextStreamInput(self._queue)
        self._finished: Optional[GeneratedCodes] = None

    def next_codes_chunk(self, max_chunk_frames: int) -> Optional[GeneratedCodesChunk]:
        if self._finished is not None:
            return None
        while True:
            r = self._poller.next_codes_chunk(max_chunk_frames)
            if isinstance(r, GeneratedCodesChunk):
                return r
            if isinstance(r, Finished):
                self._finished = r.codes
                return None
            if not self._queue:
                self._poller.finish_text()  # sender dropped: finish (generation.rs:1075)
                continue
            kind, val = self._queue.pop(0)
            if kind == "ids":
                self._poller.push_ids(val)
            else:
                self._poller.finish_text()

    def finished_codes(self) -> Optional[GeneratedCodes]:
        return self._finished


def start_text_stream(engine: HipTtsEngine, options=None, stream_options=None):
    """start_text_stream (generation.rs:464-472): (TextStreamInput, HipTextStream)."""
    s = HipTextStream(engine.start_text_stream_polling(options, stream_options))
    return s.input, s
