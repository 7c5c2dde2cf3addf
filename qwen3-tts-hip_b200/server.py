"""HTTP shell over the engine: the reference's tts-server on this library.

Endpoints and behaviour follow piedshag/qwen3-tts-hip ``src/bin/tts-server.rs``:

* ``GET /`` a small page, ``GET /health`` -> ``ok``;
* ``POST /api/generate`` (application/x-www-form-urlencoded) -> one WAV file
  (``audio/wav``, 16-bit mono 24 kHz) with ``X-TTS-*`` timing headers
  (tts-server.rs:117-260);
* ``POST /api/stream`` -> chunked ``application/octet-stream`` s16le PCM, one
  HTTP chunk per audio chunk of ``stream_chunk_frames`` code frames, each
  decoded with ``left_context_frames`` of context (tts-server.rs:262-322,
  generation.rs:965-989).

Form fields and defaults are the reference's (tts-server.rs:324-470):
max_frames 120 (at most the server's max_cache_frames), speaker ryan,
language english, wav_gain 1.0, repetition_penalty 1.05, do_sample true,
top_k 50, top_p 1.0, temperature 0.9, subtalker_* the same, seed 0,
text_lookahead_tokens 8, stream_chunk_frames 6, left_context_frames 25.
This library does not tokenise: the text arrives as ``ids`` (comma- or
space-separated content token ids); a request with only ``text`` is answered
400. The optional ``rng`` field picks ``lcg`` (the reference's) or ``philox``.
Samples become PCM as the reference does: clamp(sample * gain, -1, 1) *
32767, truncated toward zero.

Like the reference, one request is served at a time (the engine is not
thread-safe). Run from the repository root:

    python -c "import sys, __graft_entry__ as G; G.load_package();
               from qwen3_tts_hip_b200 import server; server.main(sys.argv[1:])" \
        <model_dir> [bind_addr] [max_cache_frames]
"""
from __future__ import annotations

import struct
import sys
import time
import urllib.parse
from http.server import BaseHTTPRequestHandler, HTTPServer

import numpy as np

from .engine import (SAMPLE_RATE, Error, GenerateOptions, HipTtsEngine, InvalidInput,
                     StreamOptions, DEFAULT_STREAM_LEFT_CONTEXT_FRAMES,
                     DEFAULT_TEXT_LOOKAHEAD_TOKENS)

DEFAULT_BIND = "127.0.0.1:8080"
DEFAULT_MAX_CACHE_FRAMES = 240
DEFAULT_STREAM_CHUNK_FRAMES = 6
MAX_REQUEST_BYTES = 64 * 1024


def pcm16(samples: np.ndarray, gain: float) -> bytes:
    """samples_to_pcm16_bytes (tts-server.rs:527-534)."""
    v = np.clip(np.asarray(samples, dtype=np.float32) * np.float32(gain), -1.0, 1.0)
    return (v * np.float32(32767)).astype(np.int16).astype("<i2").tobytes()


def wav_bytes(samples: np.ndarray, gain: float, sample_rate: int = SAMPLE_RATE) -> bytes:
    """GeneratedSpeech::to_wav_bytes (generation.rs:1530-1553): 44-byte RIFF
    header, PCM 16-bit mono."""
    data = pcm16(samples, gain)
    if len(data) > 0xFFFFFFFF - 36:
        raise InvalidInput(1, "wav is too large")
    head = b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVEfmt " + struct.pack(
        "<IHHIIHH", 16, 1, 1, sample_rate, sample_rate * 2, 2, 16) + b"data" + struct.pack(
        "<I", len(data))
    return head + data


def _bool(v: str, name: str) -> bool:
    s = v.strip().lower()
    if s in ("1", "true", "on", "yes"):
        return True
    if s in ("0", "false", "off", "no"):
        return False
    raise InvalidInput(1, f"invalid {name}: {v}")


def _num(v: str, name: str, kind):
    try:
        return kind(v.strip())
    except ValueError:
        raise InvalidInput(1, f"invalid {name}: {v}") from None


class GenerationRequest:
    """parse_generation_request (tts-server.rs:324-470) with ids in place of text."""

    def __init__(self, body: bytes, max_cache_frames: int):
        form = {k: v[-1] for k, v in urllib.parse.parse_qs(body.decode("utf-8", "replace"),
                                                          keep_blank_values=True).items()}
        raw_ids = form.get("ids", "").replace(",", " ").split()
        if not raw_ids:
            if form.get("text", "").strip():
                raise InvalidInput(1, "this server takes content token ids ('ids'); "
                                      "text tokenisation is outside the library")
            raise InvalidInput(1, "ids must not be empty")
        self.ids = [_num(x, "ids", int) for x in raw_ids]
        if any(i < 0 for i in self.ids):
            raise InvalidInput(1, "ids must be non-negative")
        g = lambda k, d, kind: _num(form[k], k, kind) if k in form else d  # noqa: E731
        b = lambda k, d: _bool(form[k], k) if k in form else d  # noqa: E731
        max_frames = g("max_frames", 120, int)
        if max_frames == 0 or max_frames > max_cache_frames:
            raise InvalidInput(1, f"max_frames must be in 1..={max_cache_frames} for this server")
        self.wav_gain = g("wav_gain", 1.0, float)
        penalty = g("repetition_penalty", 1.05, float)
        if penalty <= 0:
            raise InvalidInput(1, "repetition_penalty must be positive")
        lookahead = g("text_lookahead_tokens", DEFAULT_TEXT_LOOKAHEAD_TOKENS, int)
        if lookahead == 0:
            raise InvalidInput(1, "text_lookahead_tokens must be non-zero")
        self.stream_chunk_frames = g("stream_chunk_frames", DEFAULT_STREAM_CHUNK_FRAMES, int)
        if self.stream_chunk_frames == 0:
            raise InvalidInput(1, "stream_chunk_frames must be non-zero")
        rng = form.get("rng", "lcg").strip().lower()
        if rng not in ("lcg", "philox"):
            raise InvalidInput(1, "rng must be lcg or philox")
        self.options = GenerateOptions(
            speaker=form.get("speaker", "ryan"), language=form.get("language", "english"),
            max_frames=max_frames, decode_audio=False, do_sample=b("do_sample", True),
            top_k=g("top_k", 50, int), top_p=g("top_p", 1.0, float),
            temperature=g("temperature", 0.9, float), repetition_penalty=penalty,
            subtalker_dosample=b("subtalker_dosample", True),
            subtalker_top_k=g("subtalker_top_k", 50, int),
            subtalker_top_p=g("subtalker_top_p", 1.0, float),
            subtalker_temperature=g("subtalker_temperature", 0.9, float),
            seed=g("seed", 0, int), rng=rng)
        self.stream_options = StreamOptions(
            text_lookahead_tokens=lookahead,
            left_context_frames=g("left_context_frames", DEFAULT_STREAM_LEFT_CONTEXT_FRAMES, int))


class TtsServer(HTTPServer):
    """One engine, requests served one at a time."""

    def __init__(self, engine, bind=DEFAULT_BIND, max_cache_frames=DEFAULT_MAX_CACHE_FRAMES,
                 load_seconds=0.0, log=print):
        host, port = bind.rsplit(":", 1)
        self.engine = engine
        self.max_cache_frames = max_cache_frames
        self.load_seconds = load_seconds
        self.log = log
        super().__init__((host, int(port)), _Handler)


def _fmt(x: float) -> str:
    return f"{x:.6f}"


def _rtf(seconds: float, audio_seconds: float) -> float:
    return seconds / audio_seconds if audio_seconds > 0 else 0.0


class _Handler(BaseHTTPRequestHandler):
    protocol_version = "HTTP/1.1"
    server: TtsServer

    def log_message(self, fmt, *args):  # the server logs one line per generation instead
        pass

    def _send(self, code: int, reason: str, body: bytes, headers=()):
        self.send_response(code, reason)
        for k, v in headers:
            self.send_header(k, v)
        self.send_header("Content-Length", str(len(body)))
        self.send_header("Connection", "close")
        self.end_headers()
        self.wfile.write(body)

    def _text(self, code: int, reason: str, text: str):
        self._send(code, reason, text.encode(), [("Content-Type", "text/plain; charset=utf-8")])

    def do_GET(self):
        if self.path == "/":
            html = ("<!doctype html><title>qtts_b200</title><p>POST ids to /api/generate "
                    "(WAV) or /api/stream (s16le PCM, chunked).</p>")
            self._send(200, "OK", html.encode(), [("Content-Type", "text/html; charset=utf-8")])
        elif self.path == "/health":
            self._text(200, "OK", "ok\n")
        elif self.path == "/favicon.ico":
            self._send(204, "No Content", b"")
        else:
            self._text(404, "Not Found", "not found\n")

    def _read_request(self):
        n = int(self.headers.get("Content-Length", "0") or 0)
        if n > MAX_REQUEST_BYTES:
            raise InvalidInput(1, "request is too large")
        if not self.headers.get("Content-Type", "").startswith(
                "application/x-www-form-urlencoded"):
            self._text(415, "Unsupported Media Type",
                       "expected application/x-www-form-urlencoded\n")
            return None
        body = self.rfile.read(n)
        try:
            return GenerationRequest(body, self.server.max_cache_frames)
        except InvalidInput as e:
            self._text(400, "Bad Request", f"{e}\n")
            return None

    def do_POST(self):
        try:
            if self.path == "/api/generate":
                self._generate()
            elif self.path == "/api/stream":
                self._stream()
            else:
                self._text(404, "Not Found", "not found\n")
        except InvalidInput as e:
            self._text(400, "Bad Request", f"{e}\n")
        except Error as e:
            self._text(500, "Internal Server Error", f"{e}\n")

    def _generate(self):
        """handle_generate (tts-server.rs:117-260)."""
        req = self._read_request()
        if req is None:
            return
        eng = self.server.engine
        t0 = time.perf_counter()
        gen = eng.generate_codes_from_ids(req.ids, req.options)
        gen_s = time.perf_counter() - t0
        t1 = time.perf_counter()
        samples = eng.decode_codes(gen.codes) if gen.codes else np.zeros(0, np.float32)
        dec_s = time.perf_counter() - t1
        t2 = time.perf_counter()
        wav = wav_bytes(samples, req.wav_gain)
        wav_s = time.perf_counter() - t2
        ttfa = time.perf_counter() - t0
        audio_s = samples.size / SAMPLE_RATE
        o = req.options
        headers = [
            ("Content-Type", "audio/wav"), ("Cache-Control", "no-store"),
            ("X-TTS-Load-Seconds", _fmt(self.server.load_seconds)),
            ("X-TTS-Generation-Seconds", _fmt(gen_s)), ("X-TTS-Decode-Seconds", _fmt(dec_s)),
            ("X-TTS-Wav-Seconds", _fmt(wav_s)), ("X-TTS-Time-To-First-Audio-Seconds", _fmt(ttfa)),
            ("X-TTS-Inference-Seconds", _fmt(gen_s + dec_s)),
            ("X-TTS-Audio-Seconds", _fmt(audio_s)),
            ("X-TTS-Generation-RTF", _fmt(_rtf(gen_s, audio_s))),
            ("X-TTS-Decode-RTF", _fmt(_rtf(dec_s, audio_s))),
            ("X-TTS-Inference-RTF", _fmt(_rtf(gen_s + dec_s, audio_s))),
            ("X-TTS-Frames", str(gen.frames)), ("X-TTS-Samples", str(samples.size)),
            ("X-TTS-Ended-By-EOS", str(gen.ended_by_eos).lower()),
            ("X-TTS-Repetition-Penalty", _fmt(o.repetition_penalty)),
            ("X-TTS-Do-Sample", str(o.do_sample).lower()), ("X-TTS-Top-K", str(o.top_k)),
            ("X-TTS-Top-P", _fmt(o.top_p)), ("X-TTS-Temperature", _fmt(o.temperature)),
            ("X-TTS-Subtalker-Do-Sample", str(o.subtalker_dosample).lower()),
            ("X-TTS-Subtalker-Top-K", str(o.subtalker_top_k)),
            ("X-TTS-Subtalker-Top-P", _fmt(o.subtalker_top_p)),
            ("X-TTS-Subtalker-Temperature", _fmt(o.subtalker_temperature)),
            ("X-TTS-Seed", str(o.seed)),
        ]
        self.server.log(f"generated: frames={gen.frames}, samples={samples.size}, "
                        f"ended_by_eos={gen.ended_by_eos}, generation_seconds={gen_s:.6f}, "
                        f"decode_seconds={dec_s:.6f}, audio_seconds={audio_s:.6f}")
        self._send(200, "OK", wav, headers)

    def _chunk(self, data: bytes):
        self.wfile.write(f"{len(data):x}\r\n".encode() + data + b"\r\n")

    def _stream(self):
        """handle_stream (tts-server.rs:262-322): chunked s16le PCM."""
        req = self._read_request()
        if req is None:
            return
        eng = self.server.engine
        t0 = time.perf_counter()
        st = eng.start_stream_from_ids(req.ids, req.options, req.stream_options)
        self.send_response(200, "OK")
        for k, v in [("Content-Type", "application/octet-stream"), ("Cache-Control", "no-store"),
                     ("X-TTS-Sample-Rate", str(SAMPLE_RATE)), ("X-TTS-Sample-Format", "s16le"),
                     ("X-TTS-Chunk-Frames", str(req.stream_chunk_frames)),
                     ("X-TTS-Text-Lookahead-Tokens",
                      str(req.stream_options.text_lookahead_tokens)),
                     ("X-TTS-Left-Context-Frames", str(req.stream_options.left_context_frames)),
                     ("Transfer-Encoding", "chunked"), ("Connection", "close")]:
            self.send_header(k, v)
        self.end_headers()
        total_samples = total_frames = 0
        ended = False
        ttfa = None
        try:
            while (ch := st.next_audio_chunk(req.stream_chunk_frames)) is not None:
                if ttfa is None and ch.samples.size:
                    ttfa = time.perf_counter() - t0
                total_samples += ch.samples.size
                total_frames, ended = ch.total_frames, ch.ended_by_eos
                self._chunk(pcm16(ch.samples, req.wav_gain))
        finally:
            st.close()
        self.wfile.write(b"0\r\n\r\n")
        secs = time.perf_counter() - t0
        self.server.log(f"streamed: frames={total_frames}, samples={total_samples}, "
                        f"ended_by_eos={ended}, time_to_first_audio_seconds="
                        f"{'n/a' if ttfa is None else f'{ttfa:.6f}'}, seconds={secs:.6f}")


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        print("usage: server.main([model_dir, bind_addr?, max_cache_frames?])", file=sys.stderr)
        return 2
    model_dir = argv[0]
    bind = argv[1] if len(argv) > 1 else DEFAULT_BIND
    max_cache_frames = int(argv[2]) if len(argv) > 2 else DEFAULT_MAX_CACHE_FRAMES
    if max_cache_frames == 0:
        raise InvalidInput(1, "max_cache_frames must be non-zero")
    t0 = time.perf_counter()
    engine = HipTtsEngine.load_with_max_frames(model_dir, 0, max_cache_frames)
    srv = TtsServer(engine, bind, max_cache_frames, time.perf_counter() - t0)
    print(f"TTS server listening on http://{bind}/, model_dir={model_dir}, "
          f"load_seconds={srv.load_seconds:.6f}, max_cache_frames={max_cache_frames}")
    srv.serve_forever()
    return 0


if __name__ == "__main__":
    sys.exit(main())
