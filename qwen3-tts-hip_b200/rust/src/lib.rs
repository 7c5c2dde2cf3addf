//! Rust binding of `libqtts_b200.so`, the B200 (sm_100a) Qwen3-TTS token loop.
//!
//! `ffi` declares every entry point of `include/qtts_b200.h` one for one.
//! The safe layer above it keeps the surface of the reference crate's
//! `HipTtsEngine` (piedshag/qwen3-tts-hip `src/generation.rs:254-651`):
//! `load`, `load_with_max_frames`, `load_with_options`, code generation,
//! voice-clone codes, streams, polling text streams and `decode_codes`,
//! with `GenerateOptions` / `StreamOptions` / `TextStreamOptions` defaults of
//! `src/generation.rs:40-92,211-228`. Text enters as token ids: the caller
//! keeps tokenising with its own `TtsTextPrep` and passes the content ids.
//!
//! To use it inside the reference crate, add this file as `src/b200.rs`,
//! add the `Cuda`, `Io` and `Unsupported` variants below to
//! `src/error.rs`, and route `HipTtsEngine`'s methods to these calls.
//! Errors map as the reference keeps them apart (`src/error.rs:22-41`): only
//! invalid input and the cache-capacity rule are `InvalidInput`; device
//! failures are `Cuda { call, status, message }`.

use std::ffi::{CStr, CString};
use std::marker::PhantomData;
use std::path::Path;

#[allow(non_camel_case_types)]
pub mod ffi {
    use std::ffi::c_char;

    pub const QTTS_OK: i32 = 0;
    pub const QTTS_ERR_INVALID_INPUT: i32 = 1;
    pub const QTTS_ERR_CUDA: i32 = 2;
    pub const QTTS_ERR_CACHE_FULL: i32 = 3;
    pub const QTTS_ERR_IO: i32 = 4;
    pub const QTTS_ERR_UNSUPPORTED: i32 = 5;
    pub const QTTS_ERR_DEVICE_STATE: i32 = 6;

    pub const QTTS_CHUNK: i32 = 0;
    pub const QTTS_CHUNK_NONE: i32 = 1;
    pub const QTTS_NEED_MORE_TEXT: i32 = 2;
    pub const QTTS_FINISHED: i32 = 3;

    #[repr(C)]
    pub struct qtts_engine {
        _private: [u8; 0],
    }
    #[repr(C)]
    pub struct qtts_stream {
        _private: [u8; 0],
    }
    #[repr(C)]
    pub struct qtts_text_stream {
        _private: [u8; 0],
    }
    #[repr(C)]
    pub struct qtts_codec_stream {
        _private: [u8; 0],
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug)]
    pub struct qtts_trace_launch {
        pub name: [c_char; 48],
        pub entry_ns: i64,
        pub wait_ns: i64,
        pub exit_ns: i64,
        pub last_wait_ns: i64,
        pub mark4_ns: i64,
        pub mark5_ns: i64,
        pub dur6_ns: u64,
        pub dur7_ns: u64,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug)]
    pub struct qtts_generate_options {
        pub speaker: *const c_char,
        pub language: *const c_char,
        pub max_frames: u32,
        pub decode_audio: i32,
        pub do_sample: i32,
        pub top_k: u32,
        pub top_p: f32,
        pub temperature: f32,
        pub repetition_penalty: f32,
        pub subtalker_dosample: i32,
        pub subtalker_top_k: u32,
        pub subtalker_top_p: f32,
        pub subtalker_temperature: f32,
        pub seed: u64,
        pub rng: i32,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct qtts_stream_options {
        pub text_lookahead_tokens: u32,
        pub left_context_frames: u32,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct qtts_text_stream_options {
        pub min_start_tokens: u32,
        pub min_resume_tokens: u32,
        pub flush_on_punctuation: i32,
        pub left_context_frames: u32,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct qtts_codes_chunk {
        pub frames: usize,
        pub total_frames: usize,
        pub ended_by_eos: i32,
        pub status: i32,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct qtts_engine_info {
        pub hidden: u32,
        pub vocab: u32,
        pub cp_hidden: u32,
        pub cp_vocab: u32,
        pub num_code_groups: u32,
        pub talker_layers: u32,
        pub cp_layers: u32,
        pub codec_eos: u32,
        pub max_cache_steps: usize,
        pub device_bytes: usize,
        pub reserved: [i32; 2],
        pub has_codec: i32,
        pub samples_per_frame: u32,
    }

    #[link(name = "qtts_b200")]
    extern "C" {
        pub fn qtts_last_error() -> *const c_char;
        pub fn qtts_abi_version() -> i32;
        pub fn qtts_generate_options_default(out: *mut qtts_generate_options);
        pub fn qtts_stream_options_default(out: *mut qtts_stream_options);
        pub fn qtts_text_stream_options_default(out: *mut qtts_text_stream_options);
        pub fn qtts_engine_load(model_dir: *const c_char, device: i32,
                                out: *mut *mut qtts_engine) -> i32;
        pub fn qtts_engine_load_with_max_frames(model_dir: *const c_char, device: i32,
                                                max_frames: usize,
                                                out: *mut *mut qtts_engine) -> i32;
        pub fn qtts_engine_load_with_options(model_dir: *const c_char, device: i32,
                                             max_cache_steps: usize,
                                             out: *mut *mut qtts_engine) -> i32;
        pub fn qtts_engine_destroy(engine: *mut qtts_engine);
        pub fn qtts_engine_get_info(engine: *const qtts_engine, out: *mut qtts_engine_info) -> i32;
        pub fn qtts_decode_codes(engine: *mut qtts_engine, codes: *const i32, n_codes: usize,
                                 samples: *mut f32, samples_capacity: usize,
                                 n_samples: *mut usize) -> i32;
        pub fn qtts_last_decode_timing(engine: *const qtts_engine, ms: *mut f32,
                                       launches: *mut usize) -> i32;
        pub fn qtts_codec_stream_open(engine: *mut qtts_engine, max_frames: usize,
                                      out: *mut *mut qtts_codec_stream) -> i32;
        pub fn qtts_codec_stream_decode(stream: *mut qtts_codec_stream, codes: *const i32,
                                        n_codes: usize, samples: *mut f32,
                                        samples_capacity: usize, n_samples: *mut usize) -> i32;
        pub fn qtts_codec_stream_destroy(stream: *mut qtts_codec_stream);
        pub fn qtts_generate_codes_from_ids(engine: *mut qtts_engine, content_ids: *const u32,
                                            n_ids: usize, options: *const qtts_generate_options,
                                            codes_out: *mut i32, codes_capacity: usize,
                                            frames_out: *mut usize, ended_by_eos: *mut i32) -> i32;
        pub fn qtts_generate_codes_batch_from_ids(engine: *mut qtts_engine, ids: *const u32,
                                                  lengths: *const usize, batch: usize,
                                                  opts: *const qtts_generate_options,
                                                  codes_out: *mut i32, cap_per_request: usize,
                                                  frames_out: *mut usize,
                                                  ended_out: *mut i32) -> i32;
        pub fn qtts_generate_voice_clone_codes_from_ids(engine: *mut qtts_engine,
                                                        content_ids: *const u32, n_ids: usize,
                                                        speaker_embedding: *const f32,
                                                        options: *const qtts_generate_options,
                                                        codes_out: *mut i32,
                                                        codes_capacity: usize,
                                                        frames_out: *mut usize,
                                                        ended_by_eos: *mut i32) -> i32;
        pub fn qtts_generate_codes_from_rows(engine: *mut qtts_engine, prefill: *const f32,
                                             prefill_steps: usize, trailing: *const f32,
                                             trailing_steps: usize, tts_pad: *const f32,
                                             options: *const qtts_generate_options,
                                             codes_out: *mut i32, codes_capacity: usize,
                                             frames_out: *mut usize,
                                             ended_by_eos: *mut i32) -> i32;
        pub fn qtts_prepare_inputs_from_ids(engine: *mut qtts_engine, content_ids: *const u32,
                                            n_ids: usize, lookahead: usize,
                                            speaker: *const c_char, language: *const c_char,
                                            prefill_out: *mut f32, prefill_steps: *mut usize,
                                            trailing_out: *mut f32, trailing_steps: *mut usize,
                                            tts_pad_out: *mut f32) -> i32;
        pub fn qtts_stream_start_from_ids(engine: *mut qtts_engine, content_ids: *const u32,
                                          n_ids: usize, options: *const qtts_generate_options,
                                          stream_options: *const qtts_stream_options,
                                          out: *mut *mut qtts_stream) -> i32;
        pub fn qtts_stream_next_codes_chunk(stream: *mut qtts_stream, max_chunk_frames: usize,
                                            codes_out: *mut i32, codes_capacity: usize,
                                            chunk: *mut qtts_codes_chunk) -> i32;
        pub fn qtts_stream_destroy(stream: *mut qtts_stream);
        pub fn qtts_text_stream_start(engine: *mut qtts_engine,
                                      options: *const qtts_generate_options,
                                      text_options: *const qtts_text_stream_options,
                                      out: *mut *mut qtts_text_stream) -> i32;
        pub fn qtts_text_stream_push_ids(stream: *mut qtts_text_stream, ids: *const u32,
                                         n: usize) -> i32;
        pub fn qtts_text_stream_finish(stream: *mut qtts_text_stream) -> i32;
        pub fn qtts_text_stream_next_codes_chunk(stream: *mut qtts_text_stream,
                                                 max_chunk_frames: usize, codes_out: *mut i32,
                                                 codes_capacity: usize,
                                                 chunk: *mut qtts_codes_chunk) -> i32;
        pub fn qtts_text_stream_codes(stream: *mut qtts_text_stream, codes_out: *mut i32,
                                      codes_capacity: usize, frames_out: *mut usize,
                                      ended_by_eos: *mut i32) -> i32;
        pub fn qtts_text_stream_destroy(stream: *mut qtts_text_stream);
        pub fn qtts_talker_prefill(engine: *mut qtts_engine, rows: *const f32, steps: usize,
                                   hidden_out: *mut f32, logits_out: *mut f32,
                                   token_out: *mut i32) -> i32;
        pub fn qtts_talker_decode_step(engine: *mut qtts_engine, input: *const f32, offset: usize,
                                       hidden_out: *mut f32, logits_out: *mut f32,
                                       token_out: *mut i32) -> i32;
        pub fn qtts_talker_decode_step_static(engine: *mut qtts_engine, input: *const f32,
                                              offset: usize, hidden_out: *mut f32,
                                              logits_out: *mut f32, token_out: *mut i32) -> i32;
        pub fn qtts_code_predictor(engine: *mut qtts_engine, talker_hidden: *const f32,
                                   semantic_embed: *const f32,
                                   options: *const qtts_generate_options, tokens_out: *mut i32,
                                   embedding_sum_out: *mut f32, logits_out: *mut f32) -> i32;
        pub fn qtts_step_trace_enable(engine: *mut qtts_engine, on: i32) -> i32;
        pub fn qtts_step_trace_read(engine: *const qtts_engine, out: *mut qtts_trace_launch,
                                    cap: usize, n: *mut usize) -> i32;
        pub fn qtts_selftest_device_wait(engine: *mut qtts_engine, limit_us: u32) -> i32;
        pub fn qtts_last_timings(engine: *const qtts_engine, prefill_ms: *mut f32,
                                 frames_ms: *mut f32, frames: *mut usize) -> i32;
        pub fn qtts_last_launch_count(engine: *const qtts_engine, kernels: *mut usize) -> i32;
        pub fn qtts_profile_projection(engine: *mut qtts_engine, which: i32, launches: i32,
                                       ms_per_launch: *mut f32,
                                       bytes_per_launch: *mut f64) -> i32;
    }
}

/// The reference's error type (`src/error.rs:3-44`) with the CUDA-side
/// variants this library reports.
#[derive(Debug)]
pub enum Error {
    /// `Error::InvalidInput`: bad arguments or options, and the cache rule
    /// `P + max_frames <= max_cache_steps` (generation.rs:608-617).
    InvalidInput(String),
    /// A CUDA call failed, or the device reported an invalid state (a bounded
    /// device wait ran out, no finite logits to sample from). Takes the place
    /// of `Error::Hip { call, status, message }`.
    Cuda { call: &'static str, status: i32, message: String },
    /// Model directory or safetensors problems.
    Io(String),
    /// A feature this build does not provide (e.g. the codec without its
    /// checkpoint, text tokenisation).
    Unsupported(String),
}

impl std::fmt::Display for Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        match self {
            Error::InvalidInput(m) => write!(f, "invalid input: {m}"),
            Error::Cuda { call, status, message } => {
                write!(f, "CUDA call {call} failed with status {status}: {message}")
            }
            Error::Io(m) => write!(f, "i/o: {m}"),
            Error::Unsupported(m) => write!(f, "unsupported: {m}"),
        }
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn last_error() -> String {
    // SAFETY: the library returns a NUL-terminated thread-local string.
    unsafe {
        let p = ffi::qtts_last_error();
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

/// Maps a `qtts_status` to the reference's error kinds.
pub fn check(call: &'static str, status: i32) -> Result<()> {
    match status {
        ffi::QTTS_OK => Ok(()),
        ffi::QTTS_ERR_INVALID_INPUT | ffi::QTTS_ERR_CACHE_FULL => {
            Err(Error::InvalidInput(last_error()))
        }
        ffi::QTTS_ERR_IO => Err(Error::Io(last_error())),
        ffi::QTTS_ERR_UNSUPPORTED => Err(Error::Unsupported(last_error())),
        ffi::QTTS_ERR_CUDA | ffi::QTTS_ERR_DEVICE_STATE => {
            Err(Error::Cuda { call, status, message: last_error() })
        }
        other => Err(Error::Cuda { call, status: other, message: last_error() }),
    }
}

/// Random source of the sampler: the reference's LCG in its draw order, or
/// Philox-4x32-10 keyed by the seed (no reference counterpart).
#[derive(Clone, Copy, Debug, PartialEq, Eq, Default)]
pub enum Rng {
    #[default]
    Lcg,
    Philox,
}

/// `GenerateOptions` (generation.rs:40-77); speaker and language are the
/// config keys of the reference's `Speaker` / `Language` enums.
#[derive(Clone, Debug)]
pub struct GenerateOptions {
    pub speaker: String,
    pub language: String,
    pub max_frames: usize,
    pub decode_audio: bool,
    pub do_sample: bool,
    pub top_k: usize,
    pub top_p: f32,
    pub temperature: f32,
    pub repetition_penalty: f32,
    pub subtalker_dosample: bool,
    pub subtalker_top_k: usize,
    pub subtalker_top_p: f32,
    pub subtalker_temperature: f32,
    pub seed: u64,
    pub rng: Rng,
}

impl Default for GenerateOptions {
    fn default() -> Self {
        Self {
            speaker: "ryan".into(),
            language: "english".into(),
            max_frames: 240,
            decode_audio: true,
            do_sample: true,
            top_k: 50,
            top_p: 1.0,
            temperature: 0.9,
            repetition_penalty: 1.05,
            subtalker_dosample: true,
            subtalker_top_k: 50,
            subtalker_top_p: 1.0,
            subtalker_temperature: 0.9,
            seed: 0,
            rng: Rng::Lcg,
        }
    }
}

/// Keeps the C strings alive for the duration of a call.
struct RawOptions {
    raw: ffi::qtts_generate_options,
    _speaker: CString,
    _language: CString,
}

impl GenerateOptions {
    fn raw(&self) -> Result<RawOptions> {
        let speaker = CString::new(self.speaker.as_str())
            .map_err(|_| Error::InvalidInput("speaker contains NUL".into()))?;
        let language = CString::new(self.language.as_str())
            .map_err(|_| Error::InvalidInput("language contains NUL".into()))?;
        let max_frames = u32::try_from(self.max_frames)
            .map_err(|_| Error::InvalidInput("max_frames too large".into()))?;
        let raw = ffi::qtts_generate_options {
            speaker: speaker.as_ptr(),
            language: language.as_ptr(),
            max_frames,
            decode_audio: self.decode_audio as i32,
            do_sample: self.do_sample as i32,
            top_k: self.top_k.min(u32::MAX as usize) as u32,
            top_p: self.top_p,
            temperature: self.temperature,
            repetition_penalty: self.repetition_penalty,
            subtalker_dosample: self.subtalker_dosample as i32,
            subtalker_top_k: self.subtalker_top_k.min(u32::MAX as usize) as u32,
            subtalker_top_p: self.subtalker_top_p,
            subtalker_temperature: self.subtalker_temperature,
            seed: self.seed,
            rng: match self.rng {
                Rng::Lcg => 0,
                Rng::Philox => 1,
            },
        };
        Ok(RawOptions { raw, _speaker: speaker, _language: language })
    }
}

/// `StreamOptions` (generation.rs:79-92).
#[derive(Clone, Debug)]
pub struct StreamOptions {
    pub text_lookahead_tokens: usize,
    pub left_context_frames: usize,
}

impl Default for StreamOptions {
    fn default() -> Self {
        Self { text_lookahead_tokens: 8, left_context_frames: 25 }
    }
}

/// `TextStreamOptions` (generation.rs:211-228).
#[derive(Clone, Debug)]
pub struct TextStreamOptions {
    pub min_start_tokens: usize,
    pub min_resume_tokens: usize,
    pub flush_on_punctuation: bool,
    pub left_context_frames: usize,
}

impl Default for TextStreamOptions {
    fn default() -> Self {
        Self {
            min_start_tokens: 8,
            min_resume_tokens: 1,
            flush_on_punctuation: true,
            left_context_frames: 25,
        }
    }
}

/// `EngineOptions` (generation.rs:284-315).
#[derive(Clone, Debug)]
pub struct EngineOptions {
    pub device: i32,
    pub max_cache_steps: usize,
}

impl Default for EngineOptions {
    fn default() -> Self {
        Self { device: 0, max_cache_steps: 512 }
    }
}

/// `GeneratedCodes`: frame-major `[frames x 16]`, the EOS frame not emitted.
#[derive(Clone, Debug)]
pub struct GeneratedCodes {
    pub codes: Vec<i32>,
    pub frames: usize,
    pub ended_by_eos: bool,
}

/// `GeneratedCodesChunk` (generation.rs:238-244).
#[derive(Clone, Debug)]
pub struct GeneratedCodesChunk {
    pub codes: Vec<i32>,
    pub frames: usize,
    pub total_frames: usize,
    pub ended_by_eos: bool,
}

/// `IncrementalAudio` for codes: a chunk, a request for more text, or the end.
#[derive(Clone, Debug)]
pub enum IncrementalCodes {
    Chunk(GeneratedCodesChunk),
    NeedMoreText,
    Finished(GeneratedCodes),
}

fn path_cstring(dir: &Path) -> Result<CString> {
    CString::new(dir.to_string_lossy().as_bytes())
        .map_err(|_| Error::InvalidInput("model path contains NUL".into()))
}

/// `HipTtsEngine` on the B200 library. Not `Sync`: one thread drives it.
pub struct HipTtsEngine {
    handle: *mut ffi::qtts_engine,
    info: ffi::qtts_engine_info,
}

impl HipTtsEngine {
    fn from_handle(handle: *mut ffi::qtts_engine) -> Result<Self> {
        let mut info = ffi::qtts_engine_info::default();
        // SAFETY: handle is a live engine; info is a valid out pointer.
        check("qtts_engine_get_info", unsafe { ffi::qtts_engine_get_info(handle, &mut info) })?;
        Ok(Self { handle, info })
    }

    /// `HipTtsEngine::load` (generation.rs:254-263).
    pub fn load(model_dir: impl AsRef<Path>, device: i32) -> Result<Self> {
        let dir = path_cstring(model_dir.as_ref())?;
        let mut h = std::ptr::null_mut();
        // SAFETY: dir is NUL-terminated; h receives a new handle.
        check("qtts_engine_load", unsafe { ffi::qtts_engine_load(dir.as_ptr(), device, &mut h) })?;
        Self::from_handle(h)
    }

    /// `HipTtsEngine::load_with_max_frames` (generation.rs:265-282).
    pub fn load_with_max_frames(model_dir: impl AsRef<Path>, device: i32,
                                max_frames: usize) -> Result<Self> {
        let dir = path_cstring(model_dir.as_ref())?;
        let mut h = std::ptr::null_mut();
        // SAFETY: as in `load`.
        check("qtts_engine_load_with_max_frames", unsafe {
            ffi::qtts_engine_load_with_max_frames(dir.as_ptr(), device, max_frames, &mut h)
        })?;
        Self::from_handle(h)
    }

    /// `HipTtsEngine::load_with_options` (generation.rs:284-315).
    pub fn load_with_options(model_dir: impl AsRef<Path>, options: EngineOptions) -> Result<Self> {
        let dir = path_cstring(model_dir.as_ref())?;
        let mut h = std::ptr::null_mut();
        // SAFETY: as in `load`.
        check("qtts_engine_load_with_options", unsafe {
            ffi::qtts_engine_load_with_options(dir.as_ptr(), options.device,
                                               options.max_cache_steps, &mut h)
        })?;
        Self::from_handle(h)
    }

    pub fn max_cache_steps(&self) -> usize {
        self.info.max_cache_steps
    }

    pub fn samples_per_code_frame(&self) -> usize {
        self.info.samples_per_frame as usize
    }

    fn groups(&self) -> usize {
        self.info.num_code_groups as usize
    }

    /// `HipTtsEngine::generate_codes` (generation.rs:356-371) on content ids.
    pub fn generate_codes_from_ids(&self, content_ids: &[u32],
                                   options: &GenerateOptions) -> Result<GeneratedCodes> {
        let raw = options.raw()?;
        let mut codes = vec![0i32; options.max_frames * self.groups()];
        let (mut frames, mut ended) = (0usize, 0i32);
        // SAFETY: every pointer is valid for the sizes passed.
        check("qtts_generate_codes_from_ids", unsafe {
            ffi::qtts_generate_codes_from_ids(self.handle, content_ids.as_ptr(), content_ids.len(),
                                              &raw.raw, codes.as_mut_ptr(), codes.len(),
                                              &mut frames, &mut ended)
        })?;
        codes.truncate(frames * self.groups());
        Ok(GeneratedCodes { codes, frames, ended_by_eos: ended != 0 })
    }

    /// `generate_voice_clone_codes` (generation.rs:373-395), x-vector mode.
    pub fn generate_voice_clone_codes_from_ids(&self, content_ids: &[u32],
                                               speaker_embedding: &[f32],
                                               options: &GenerateOptions)
                                               -> Result<GeneratedCodes> {
        if speaker_embedding.len() != self.info.hidden as usize {
            return Err(Error::InvalidInput("speaker embedding width".into()));
        }
        let raw = options.raw()?;
        let mut codes = vec![0i32; options.max_frames * self.groups()];
        let (mut frames, mut ended) = (0usize, 0i32);
        // SAFETY: every pointer is valid for the sizes passed.
        check("qtts_generate_voice_clone_codes_from_ids", unsafe {
            ffi::qtts_generate_voice_clone_codes_from_ids(
                self.handle, content_ids.as_ptr(), content_ids.len(), speaker_embedding.as_ptr(),
                &raw.raw, codes.as_mut_ptr(), codes.len(), &mut frames, &mut ended)
        })?;
        codes.truncate(frames * self.groups());
        Ok(GeneratedCodes { codes, frames, ended_by_eos: ended != 0 })
    }

    /// `HipTtsEngine::decode_codes` (generation.rs:619-646): 24 kHz samples.
    pub fn decode_codes(&self, codes: &[i32]) -> Result<Vec<f32>> {
        let mut out = vec![0f32; codes.len() / self.groups() * self.samples_per_code_frame()];
        let mut n = 0usize;
        // SAFETY: every pointer is valid for the sizes passed.
        check("qtts_decode_codes", unsafe {
            ffi::qtts_decode_codes(self.handle, codes.as_ptr(), codes.len(), out.as_mut_ptr(),
                                   out.len(), &mut n)
        })?;
        out.truncate(n);
        Ok(out)
    }

    /// A streaming codec decode of up to `max_frames` frames with carried
    /// state: each chunk decodes only its own frames, and the chunks join to
    /// `decode_codes` of all of them (in place of the re-decode of
    /// left-context frames in `next_audio_chunk`, generation.rs:965-989).
    pub fn open_codec_stream(&self, max_frames: usize) -> Result<CodecStream<'_>> {
        let mut h = std::ptr::null_mut();
        // SAFETY: h receives a new codec-stream handle.
        check("qtts_codec_stream_open", unsafe {
            ffi::qtts_codec_stream_open(self.handle, max_frames, &mut h)
        })?;
        Ok(CodecStream {
            handle: h,
            samples_per_code: self.samples_per_code_frame() / self.groups(),
            _engine: PhantomData,
        })
    }

    /// `HipTtsEngine::start_stream` (generation.rs:421-440) on content ids.
    pub fn start_stream_from_ids(&self, content_ids: &[u32], options: &GenerateOptions,
                                 stream_options: &StreamOptions) -> Result<HipTtsStream<'_>> {
        let raw = options.raw()?;
        let so = ffi::qtts_stream_options {
            text_lookahead_tokens: stream_options.text_lookahead_tokens as u32,
            left_context_frames: stream_options.left_context_frames as u32,
        };
        let mut h = std::ptr::null_mut();
        // SAFETY: every pointer is valid; h receives a new stream handle.
        check("qtts_stream_start_from_ids", unsafe {
            ffi::qtts_stream_start_from_ids(self.handle, content_ids.as_ptr(), content_ids.len(),
                                            &raw.raw, &so, &mut h)
        })?;
        Ok(HipTtsStream { handle: h, groups: self.groups(), _engine: PhantomData })
    }

    /// `HipTtsEngine::start_text_stream_polling` (generation.rs:474-485).
    pub fn start_text_stream_polling(&self, options: &GenerateOptions,
                                     text_options: &TextStreamOptions)
                                     -> Result<PollingTextStream<'_>> {
        let raw = options.raw()?;
        let to = ffi::qtts_text_stream_options {
            min_start_tokens: text_options.min_start_tokens as u32,
            min_resume_tokens: text_options.min_resume_tokens as u32,
            flush_on_punctuation: text_options.flush_on_punctuation as i32,
            left_context_frames: text_options.left_context_frames as u32,
        };
        let mut h = std::ptr::null_mut();
        // SAFETY: every pointer is valid; h receives a new text-stream handle.
        check("qtts_text_stream_start", unsafe {
            ffi::qtts_text_stream_start(self.handle, &raw.raw, &to, &mut h)
        })?;
        Ok(PollingTextStream { handle: h, groups: self.groups(), _engine: PhantomData })
    }
}

impl Drop for HipTtsEngine {
    fn drop(&mut self) {
        // SAFETY: the handle came from qtts_engine_load* and is dropped once.
        unsafe { ffi::qtts_engine_destroy(self.handle) }
    }
}

/// Streaming codec decode with carried state; borrows the engine.
pub struct CodecStream<'a> {
    handle: *mut ffi::qtts_codec_stream,
    samples_per_code: usize,
    _engine: PhantomData<&'a HipTtsEngine>,
}

impl CodecStream<'_> {
    /// The next frames' codes (frame-major) -> exactly their samples.
    pub fn decode(&mut self, codes: &[i32]) -> Result<Vec<f32>> {
        let mut out = vec![0f32; codes.len() * self.samples_per_code];
        let mut n = 0usize;
        // SAFETY: every pointer is valid for the sizes passed.
        check("qtts_codec_stream_decode", unsafe {
            ffi::qtts_codec_stream_decode(self.handle, codes.as_ptr(), codes.len(),
                                          out.as_mut_ptr(), out.len(), &mut n)
        })?;
        out.truncate(n);
        Ok(out)
    }
}

impl Drop for CodecStream<'_> {
    fn drop(&mut self) {
        // SAFETY: the handle came from qtts_codec_stream_open.
        unsafe { ffi::qtts_codec_stream_destroy(self.handle) }
    }
}

/// `HipTtsStream` (generation.rs:876-997); borrows the engine.
pub struct HipTtsStream<'a> {
    handle: *mut ffi::qtts_stream,
    groups: usize,
    _engine: PhantomData<&'a HipTtsEngine>,
}

impl HipTtsStream<'_> {
    /// `next_codes_chunk` (generation.rs:876-963): `None` once the stream ended.
    pub fn next_codes_chunk(&mut self, max_chunk_frames: usize)
                            -> Result<Option<GeneratedCodesChunk>> {
        let mut codes = vec![0i32; max_chunk_frames * self.groups];
        let mut chunk = ffi::qtts_codes_chunk::default();
        // SAFETY: every pointer is valid for the sizes passed.
        check("qtts_stream_next_codes_chunk", unsafe {
            ffi::qtts_stream_next_codes_chunk(self.handle, max_chunk_frames, codes.as_mut_ptr(),
                                              codes.len(), &mut chunk)
        })?;
        if chunk.status != ffi::QTTS_CHUNK {
            return Ok(None);
        }
        codes.truncate(chunk.frames * self.groups);
        Ok(Some(GeneratedCodesChunk {
            codes,
            frames: chunk.frames,
            total_frames: chunk.total_frames,
            ended_by_eos: chunk.ended_by_eos != 0,
        }))
    }
}

impl Drop for HipTtsStream<'_> {
    fn drop(&mut self) {
        // SAFETY: the handle came from qtts_stream_start_from_ids.
        unsafe { ffi::qtts_stream_destroy(self.handle) }
    }
}

/// `PollingTextStream` (generation.rs:1086-1451) with ids in place of text.
pub struct PollingTextStream<'a> {
    handle: *mut ffi::qtts_text_stream,
    groups: usize,
    _engine: PhantomData<&'a HipTtsEngine>,
}

impl PollingTextStream<'_> {
    /// `push_text` with the tokens already split into ids.
    pub fn push_ids(&mut self, ids: &[u32]) -> Result<()> {
        // SAFETY: ids is valid for its length.
        check("qtts_text_stream_push_ids", unsafe {
            ffi::qtts_text_stream_push_ids(self.handle, ids.as_ptr(), ids.len())
        })
    }

    /// `finish_text`.
    pub fn finish_text(&mut self) -> Result<()> {
        // SAFETY: live handle.
        check("qtts_text_stream_finish", unsafe { ffi::qtts_text_stream_finish(self.handle) })
    }

    /// `next_audio_chunk`'s code half: a chunk, `NeedMoreText` or `Finished`.
    pub fn next_codes_chunk(&mut self, max_chunk_frames: usize) -> Result<IncrementalCodes> {
        let mut codes = vec![0i32; max_chunk_frames * self.groups];
        let mut chunk = ffi::qtts_codes_chunk::default();
        // SAFETY: every pointer is valid for the sizes passed.
        check("qtts_text_stream_next_codes_chunk", unsafe {
            ffi::qtts_text_stream_next_codes_chunk(self.handle, max_chunk_frames,
                                                   codes.as_mut_ptr(), codes.len(), &mut chunk)
        })?;
        Ok(match chunk.status {
            ffi::QTTS_CHUNK => {
                codes.truncate(chunk.frames * self.groups);
                IncrementalCodes::Chunk(GeneratedCodesChunk {
                    codes,
                    frames: chunk.frames,
                    total_frames: chunk.total_frames,
                    ended_by_eos: chunk.ended_by_eos != 0,
                })
            }
            ffi::QTTS_NEED_MORE_TEXT => IncrementalCodes::NeedMoreText,
            _ => IncrementalCodes::Finished(self.finish_codes()?),
        })
    }

    /// `finish_codes` (generation.rs:1459-1475): every code generated so far.
    pub fn finish_codes(&mut self) -> Result<GeneratedCodes> {
        let (mut frames, mut ended) = (0usize, 0i32);
        // SAFETY: a null buffer asks for the sizes only.
        check("qtts_text_stream_codes", unsafe {
            ffi::qtts_text_stream_codes(self.handle, std::ptr::null_mut(), 0, &mut frames,
                                        &mut ended)
        })?;
        let mut codes = vec![0i32; frames * self.groups];
        // SAFETY: codes holds frames * groups values.
        check("qtts_text_stream_codes", unsafe {
            ffi::qtts_text_stream_codes(self.handle, codes.as_mut_ptr(), codes.len(), &mut frames,
                                        &mut ended)
        })?;
        Ok(GeneratedCodes { codes, frames, ended_by_eos: ended != 0 })
    }
}

impl Drop for PollingTextStream<'_> {
    fn drop(&mut self) {
        // SAFETY: the handle came from qtts_text_stream_start.
        unsafe { ffi::qtts_text_stream_destroy(self.handle) }
    }
}

/// ABI version this binding was written against (`qtts_abi_version`).
pub const ABI_VERSION: i32 = 2;

/// Checks that the loaded library speaks this binding's ABI.
pub fn abi_matches() -> bool {
    // SAFETY: no arguments.
    unsafe { ffi::qtts_abi_version() == ABI_VERSION }
}
