"""The HTTP shell (qwen3-tts-hip_b200/server.py) against a stand-in engine on
the CPU: form parsing and defaults of the reference's tts-server
(tts-server.rs:324-470), the WAV layout (generation.rs:1530-1553), chunked
s16le streaming with one HTTP chunk per audio chunk (tts-server.rs:262-322)
and the error statuses. The GPU test in test_gpu_codec.py drives the same
server with the real engine."""
import socket
import struct
import threading
import urllib.error
import urllib.request

import numpy as np
import pytest


class FakeStream:
    def __init__(self, frames, chunk_total):
        self.frames, self.done = frames, 0

    def next_audio_chunk(self, n):
        from types import SimpleNamespace

        if self.done >= self.frames:
            return None
        k = min(n, self.frames - self.done)
        self.done += k
        samples = np.linspace(-1.5, 1.5, k * 100, dtype=np.float32) * (self.done / self.frames)
        return SimpleNamespace(samples=samples, frames=k, total_frames=self.done,
                               ended_by_eos=False)

    def close(self):
        pass


class FakeEngine:
    """Just enough of HipTtsEngine for the shell: 100 samples per frame."""

    def __init__(self):
        self.calls = []

    def generate_codes_from_ids(self, ids, options):
        from types import SimpleNamespace

        self.calls.append(("generate", list(ids), options))
        n = options.max_frames
        return SimpleNamespace(codes=list(range(16 * n)), frames=n, ended_by_eos=False)

    def decode_codes(self, codes):
        return np.sin(np.arange(len(codes) // 16 * 100, dtype=np.float32)) * 1.2

    def start_stream_from_ids(self, ids, options, stream_options):
        self.calls.append(("stream", list(ids), options, stream_options))
        return FakeStream(options.max_frames, 0)


@pytest.fixture()
def server(pkg):
    from qwen3_tts_hip_b200 import server as S

    eng = FakeEngine()
    srv = S.TtsServer(eng, "127.0.0.1:0", max_cache_frames=40, log=lambda *_: None)
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    yield srv, eng, S
    srv.shutdown()
    srv.server_close()


def _url(srv, path):
    return f"http://127.0.0.1:{srv.server_address[1]}{path}"


def _post(srv, path, body, ctype="application/x-www-form-urlencoded"):
    req = urllib.request.Request(_url(srv, path), data=body.encode(), method="POST",
                                 headers={"Content-Type": ctype})
    return urllib.request.urlopen(req, timeout=10)


def test_health_and_index(server):
    srv, _, _ = server
    assert urllib.request.urlopen(_url(srv, "/health"), timeout=10).read() == b"ok\n"
    assert b"/api/stream" in urllib.request.urlopen(_url(srv, "/"), timeout=10).read()
    with pytest.raises(urllib.error.HTTPError) as e:
        urllib.request.urlopen(_url(srv, "/nope"), timeout=10)
    assert e.value.code == 404


def test_generate_wav(server):
    srv, eng, S = server
    r = _post(srv, "/api/generate", "ids=5,6,7&max_frames=3&wav_gain=0.5&seed=9&do_sample=false")
    body = r.read()
    assert r.headers["Content-Type"] == "audio/wav"
    assert r.headers["X-TTS-Frames"] == "3" and r.headers["X-TTS-Seed"] == "9"
    assert r.headers["X-TTS-Do-Sample"] == "false"
    riff, size, wave, fmt = struct.unpack("<4sI4s4s", body[:16])
    assert (riff, wave, fmt) == (b"RIFF", b"WAVE", b"fmt ") and size == len(body) - 8
    _, pcm_fmt, ch, rate, byte_rate, align, bits = struct.unpack("<IHHIIHH", body[16:36])
    assert (pcm_fmt, ch, rate, byte_rate, align, bits) == (1, 1, 24000, 48000, 2, 16)
    assert body[36:40] == b"data"
    want = eng.decode_codes(list(range(48)))
    got = np.frombuffer(body[44:], "<i2")
    np.testing.assert_array_equal(got, (np.clip(want * 0.5, -1, 1) * 32767).astype(np.int16))
    _, ids, opts = eng.calls[-1]
    assert ids == [5, 6, 7]
    # the reference's defaults for the fields not sent
    assert (opts.top_k, opts.top_p, opts.temperature, opts.repetition_penalty) == (50, 1.0, 0.9, 1.05)
    assert opts.subtalker_dosample and opts.subtalker_top_k == 50 and opts.speaker == "ryan"


def _raw_chunks(srv, body):
    """The HTTP chunks of a chunked response, as sent."""
    s = socket.create_connection(("127.0.0.1", srv.server_address[1]), timeout=10)
    s.sendall(f"POST /api/stream HTTP/1.1\r\nHost: x\r\nContent-Type: "
              f"application/x-www-form-urlencoded\r\nContent-Length: {len(body)}\r\n\r\n{body}"
              .encode())
    data = b""
    while True:
        b = s.recv(65536)
        if not b:
            break
        data += b
    s.close()
    head, rest = data.split(b"\r\n\r\n", 1)
    chunks = []
    while True:
        line, rest = rest.split(b"\r\n", 1)
        n = int(line, 16)
        if n == 0:
            break
        chunks.append(rest[:n])
        rest = rest[n + 2:]
    return head.decode(), chunks


def test_stream_chunks(server):
    srv, eng, S = server
    head, chunks = _raw_chunks(srv, "ids=1 2 3&max_frames=14&stream_chunk_frames=4&"
                                    "left_context_frames=3&text_lookahead_tokens=2")
    assert "Transfer-Encoding: chunked" in head and "X-TTS-Sample-Format: s16le" in head
    assert [len(c) // 2 for c in chunks] == [400, 400, 400, 200]  # 4+4+4+2 frames of 100
    _, _, opts, so = eng.calls[-1]
    assert so.text_lookahead_tokens == 2 and so.left_context_frames == 3
    ref = FakeStream(14, 0)
    for c in chunks:
        a = ref.next_audio_chunk(4)
        np.testing.assert_array_equal(np.frombuffer(c, "<i2"), (np.clip(a.samples, -1, 1) * 32767).astype(np.int16))


@pytest.mark.parametrize("body,ctype,code", [
    ("text=hello", "application/x-www-form-urlencoded", 400),
    ("ids=", "application/x-www-form-urlencoded", 400),
    ("ids=1&max_frames=41", "application/x-www-form-urlencoded", 400),
    ("ids=1&max_frames=0", "application/x-www-form-urlencoded", 400),
    ("ids=1&repetition_penalty=0", "application/x-www-form-urlencoded", 400),
    ("ids=1&stream_chunk_frames=0", "application/x-www-form-urlencoded", 400),
    ("ids=1&do_sample=maybe", "application/x-www-form-urlencoded", 400),
    ("ids=1", "application/json", 415),
])
def test_errors(server, body, ctype, code):
    srv, _, _ = server
    with pytest.raises(urllib.error.HTTPError) as e:
        _post(srv, "/api/generate", body, ctype)
    assert e.value.code == code
