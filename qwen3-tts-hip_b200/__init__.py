"""B200-native Qwen3-TTS token loop (talker decode step + CodePredictor pass) and
codec decoder (codes to 24 kHz audio).

Import name ``qwen3_tts_hip_b200`` (the directory is ``qwen3-tts-hip_b200/``;
``__graft_entry__.load_package()`` registers it). Compute lives in
``libqtts_b200.so`` built from ``csrc/`` for sm_100a; this package is the
host-side mirror of the reference's ``HipTtsEngine`` API over its C ABI.
"""
from . import engine  # noqa: F401
from .engine import (  # noqa: F401
    SAMPLE_RATE, CudaError, EngineOptions, Error, Finished, GenerateOptions, GeneratedAudioChunk,
    CodecStream, GeneratedCodes, GeneratedCodesChunk, GeneratedSpeech, HipTextStream, HipTtsEngine,
    HipTtsStream, InvalidInput,
    NeedMoreText, PollingTextStream, StreamOptions, TextStreamInput, TextStreamOptions,
    TtsPreparedInputs, lib, library_path, start_text_stream, SIGNATURES,
)
