/*
 * qtts_b200.h -- C ABI of the B200-native Qwen3-TTS token loop.
 *
 * This library replaces the device side of piedshag/qwen3-tts-hip's
 * HipTtsEngine (src/generation.rs): the talker prefill + decode step
 * (src/model/talker.rs, src/model/decode.rs), the CodePredictor pass that
 * fills codebooks 1..15 of every 80 ms frame (src/model/code_predictor.rs),
 * token selection (src/model/sampling.rs, src/gpu/kernels.rs) and the frame
 * loop around them. Plain pointers and sizes only; no torch or CUDA types.
 *
 * Conventions
 *  - Every function returns a qtts_status; on failure qtts_last_error()
 *    returns a message for the calling thread (errors of the reference:
 *    src/error.rs:3-44; InvalidInput keeps its meaning).
 *  - Codes are int32, frame-major [frames x num_code_groups] (16 per frame):
 *    the semantic token then the 15 acoustic tokens, the EOS frame not
 *    emitted (src/generation.rs:698-717).
 *  - Handles are not thread-safe. An engine owns one talker KV cache, as the
 *    reference does; starting a generation or stream resets it, so only the
 *    most recently started stream of an engine may be advanced.
 *  - Host buffers are owned by the caller; all device memory is owned by the
 *    engine.
 */
#ifndef QTTS_B200_H
#define QTTS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  QTTS_OK = 0,
  QTTS_ERR_INVALID_INPUT = 1, /* Error::InvalidInput (src/error.rs:40-41)          */
  QTTS_ERR_CUDA = 2,          /* replaces Error::Hip / Rocblas / Hiprtc             */
  QTTS_ERR_CACHE_FULL = 3,    /* P + max_frames > max_cache_steps (generation.rs:608-617) */
  QTTS_ERR_IO = 4,            /* model directory / safetensors problems              */
  QTTS_ERR_UNSUPPORTED = 5,   /* tokenizer (outside this library); codec without its checkpoint */
  QTTS_ERR_DEVICE_STATE = 6,  /* device reported an invalid sampling state           */
} qtts_status;

typedef struct qtts_engine qtts_engine;
typedef struct qtts_stream qtts_stream;
typedef struct qtts_text_stream qtts_text_stream;
typedef struct qtts_codec_stream qtts_codec_stream;

/* GenerateOptions (src/generation.rs:40-77). speaker/language are config keys
 * ("ryan", "english"); NULL means the reference defaults. */
typedef struct {
  const char* speaker;
  const char* language;
  uint32_t max_frames;
  int32_t decode_audio; /* codes-only entry points ignore it (as generate_codes does);
                         * audio comes from qtts_decode_codes */
  int32_t do_sample;
  uint32_t top_k;
  float top_p;
  float temperature;
  float repetition_penalty;
  int32_t subtalker_dosample;
  uint32_t subtalker_top_k;
  float subtalker_top_p;
  float subtalker_temperature;
  uint64_t seed;
  /* 0: the reference's 64-bit LCG in its draw order (token-identical sampled
   * runs); 1: Philox-4x32-10 keyed by seed (no reference counterpart). */
  int32_t rng;
} qtts_generate_options;

/* StreamOptions (src/generation.rs:79-92). */
typedef struct {
  uint32_t text_lookahead_tokens;
  uint32_t left_context_frames;
} qtts_stream_options;

/* TextStreamOptions (src/generation.rs:211-228). */
typedef struct {
  uint32_t min_start_tokens;
  uint32_t min_resume_tokens;
  int32_t flush_on_punctuation;
  uint32_t left_context_frames;
} qtts_text_stream_options;

typedef enum {
  QTTS_CHUNK = 0,          /* Some(GeneratedCodesChunk)                        */
  QTTS_CHUNK_NONE = 1,     /* None: stream ended (EOS or max_frames)           */
  QTTS_NEED_MORE_TEXT = 2, /* IncrementalAudio::NeedMoreText (generation.rs:1139-1147) */
  QTTS_FINISHED = 3,       /* IncrementalAudio::Finished                       */
} qtts_chunk_status;

/* GeneratedCodesChunk (src/generation.rs:238-244) */
typedef struct {
  size_t frames;
  size_t total_frames;
  int32_t ended_by_eos;
  int32_t status; /* qtts_chunk_status */
} qtts_codes_chunk;

typedef struct {
  uint32_t hidden;
  uint32_t vocab;
  uint32_t cp_hidden;
  uint32_t cp_vocab;
  uint32_t num_code_groups;
  uint32_t talker_layers;
  uint32_t cp_layers;
  uint32_t codec_eos;
  size_t max_cache_steps;
  size_t device_bytes; /* weights + KV + workspaces held on the device */
  int32_t reserved[2];
  int32_t has_codec;          /* speech_tokenizer/model.safetensors was loaded */
  uint32_t samples_per_frame; /* waveform samples per code frame (24 kHz): 1920 */
} qtts_engine_info;

const char* qtts_last_error(void);
int32_t qtts_abi_version(void);

/* GenerateOptions::default() (generation.rs:58-77). */
void qtts_generate_options_default(qtts_generate_options* out);
/* StreamOptions::default() / TextStreamOptions::default(). */
void qtts_stream_options_default(qtts_stream_options* out);
void qtts_text_stream_options_default(qtts_text_stream_options* out);

/* HipTtsEngine::load (generation.rs:254-263): max_cache_steps = 512. */
int32_t qtts_engine_load(const char* model_dir, int32_t device, qtts_engine** out);
/* HipTtsEngine::load_with_max_frames (generation.rs:265-282): 256 + max_frames. */
int32_t qtts_engine_load_with_max_frames(const char* model_dir, int32_t device,
                                         size_t max_frames, qtts_engine** out);
/* HipTtsEngine::load_with_options (generation.rs:284-315). */
int32_t qtts_engine_load_with_options(const char* model_dir, int32_t device,
                                      size_t max_cache_steps, qtts_engine** out);
void qtts_engine_destroy(qtts_engine* engine);
int32_t qtts_engine_get_info(const qtts_engine* engine, qtts_engine_info* out);

/* HipTtsEngine::decode_codes (generation.rs:619-646): codes [frames x 16]
 * (frame-major, n_codes = frames * 16) -> mono waveform at 24 kHz, 1920
 * samples per frame, clamped to [-1, 1], computed by the codec decoder
 * (HipCodecInitial, src/audio/codec_hip.rs:203-1087). samples holds
 * >= frames * 1920 floats; n_codes == 0 gives 0 samples. QTTS_ERR_UNSUPPORTED
 * when the model directory has no speech_tokenizer/model.safetensors. */
int32_t qtts_decode_codes(qtts_engine* engine, const int32_t* codes, size_t n_codes,
                          float* samples, size_t samples_capacity, size_t* n_samples);
/* Profiling seam (no reference counterpart): device time of the last
 * qtts_decode_codes between the codes landing and the waveform being ready,
 * and how many kernels it launched. */
int32_t qtts_last_decode_timing(const qtts_engine* engine, float* ms, size_t* launches);

/* Streaming codec decode with carried state (in place of next_audio_chunk's
 * re-decode of left-context frames, generation.rs:965-989): each causal
 * convolution keeps its last input columns and the pre-transformer keeps the
 * keys / values of every decoded frame, so a chunk decodes only its own
 * frames and its samples equal those of one qtts_decode_codes call over the
 * whole stream. open: up to max_frames frames in total (the key / value
 * cache is sized for them: 64 KiB per frame). decode: the next frames'
 * codes (frame-major, n_codes = frames * 16) -> frames * 1920 samples;
 * QTTS_ERR_INVALID_INPUT past max_frames. One stream decodes on the
 * engine's stream; destroy every codec stream before its engine. */
int32_t qtts_codec_stream_open(qtts_engine* engine, size_t max_frames, qtts_codec_stream** out);
int32_t qtts_codec_stream_decode(qtts_codec_stream* stream, const int32_t* codes, size_t n_codes,
                                 float* samples, size_t samples_capacity, size_t* n_samples);
void qtts_codec_stream_destroy(qtts_codec_stream* stream);

/* HipTtsEngine::generate_codes (generation.rs:356-371) from content token ids
 * (the ids between the chat-template prefix and suffix, text.rs:357-362);
 * tokenisation stays with the caller. codes_out holds >= max_frames*16. */
int32_t qtts_generate_codes_from_ids(qtts_engine* engine, const uint32_t* content_ids,
                                     size_t n_ids, const qtts_generate_options* options,
                                     int32_t* codes_out, size_t codes_capacity,
                                     size_t* frames_out, int32_t* ended_by_eos);

/* Batched serving (no reference counterpart; the reference serves one
 * sequence per engine): `batch` requests (1..16) generated together, their
 * content ids concatenated in `ids` with lengths[b] ids each. opts[b] may
 * differ only in seed, speaker and language. The requests are prefilled one
 * by one, then stepped in lockstep, every projection a tensor-core GEMM over
 * all rows. Codes of request b go to codes_out + b * cap_per_request
 * ([frames x 16] i32), with frames_out[b] and ended_out[b] (EOS). */
int32_t qtts_generate_codes_batch_from_ids(qtts_engine* engine, const uint32_t* ids,
                                           const size_t* lengths, size_t batch,
                                           const qtts_generate_options* opts, int32_t* codes_out,
                                           size_t cap_per_request, size_t* frames_out,
                                           int32_t* ended_out);

/* HipTtsEngine::generate_voice_clone_codes (generation.rs:373-395), x-vector
 * mode: speaker_embedding[hidden] replaces the speaker codec row
 * (text.rs:432-514). */
int32_t qtts_generate_voice_clone_codes_from_ids(qtts_engine* engine,
                                                 const uint32_t* content_ids, size_t n_ids,
                                                 const float* speaker_embedding,
                                                 const qtts_generate_options* options,
                                                 int32_t* codes_out, size_t codes_capacity,
                                                 size_t* frames_out, int32_t* ended_by_eos);

/* HipTtsEngine::rollout (generation.rs:657-749) from prepared inputs
 * (TtsPreparedInputs, text.rs:17-26): prefill [prefill_steps x hidden],
 * trailing [trailing_steps x hidden], tts_pad [hidden], all fp32. */
int32_t qtts_generate_codes_from_rows(qtts_engine* engine, const float* prefill,
                                      size_t prefill_steps, const float* trailing,
                                      size_t trailing_steps, const float* tts_pad,
                                      const qtts_generate_options* options, int32_t* codes_out,
                                      size_t codes_capacity, size_t* frames_out,
                                      int32_t* ended_by_eos);

/* TtsTextPrep::prepare_custom_voice_with_lookahead (text.rs:348-382) on the
 * device; lookahead 0 means all content in the prefill (usize::MAX). Output
 * capacities: prefill (9 + n_ids) x hidden, trailing (n_ids + 1) x hidden. */
int32_t qtts_prepare_inputs_from_ids(qtts_engine* engine, const uint32_t* content_ids,
                                     size_t n_ids, size_t lookahead, const char* speaker,
                                     const char* language, float* prefill_out,
                                     size_t* prefill_steps, float* trailing_out,
                                     size_t* trailing_steps, float* tts_pad_out);

/* HipTtsEngine::start_stream (generation.rs:421-440) + HipTtsStream. */
int32_t qtts_stream_start_from_ids(qtts_engine* engine, const uint32_t* content_ids,
                                   size_t n_ids, const qtts_generate_options* options,
                                   const qtts_stream_options* stream_options,
                                   qtts_stream** out);
/* HipTtsStream::next_codes_chunk (generation.rs:876-963). */
int32_t qtts_stream_next_codes_chunk(qtts_stream* stream, size_t max_chunk_frames,
                                     int32_t* codes_out, size_t codes_capacity,
                                     qtts_codes_chunk* chunk);
void qtts_stream_destroy(qtts_stream* stream);

/* HipTtsEngine::start_text_stream_polling (generation.rs:474-485) +
 * PollingTextStream with token ids in place of text
 * (push_text -> push_ids, finish_text, next_audio_chunk -> next_codes_chunk). */
int32_t qtts_text_stream_start(qtts_engine* engine, const qtts_generate_options* options,
                               const qtts_text_stream_options* text_options,
                               qtts_text_stream** out);
int32_t qtts_text_stream_push_ids(qtts_text_stream* stream, const uint32_t* ids, size_t n);
int32_t qtts_text_stream_finish(qtts_text_stream* stream);
int32_t qtts_text_stream_next_codes_chunk(qtts_text_stream* stream, size_t max_chunk_frames,
                                          int32_t* codes_out, size_t codes_capacity,
                                          qtts_codes_chunk* chunk);
/* Codes generated so far (PollingTextStream::finish_codes, generation.rs:1459-1475). */
int32_t qtts_text_stream_codes(qtts_text_stream* stream, int32_t* codes_out,
                               size_t codes_capacity, size_t* frames_out,
                               int32_t* ended_by_eos);
void qtts_text_stream_destroy(qtts_text_stream* stream);

/* Parity seams, the ones the reference's own parity binaries drive. */
/* HipTalker::prefill (talker.rs:150-205): normed hidden [hidden], raw logits
 * [vocab] (before suppression) and the greedy token after suppression. */
int32_t qtts_talker_prefill(qtts_engine* engine, const float* rows, size_t steps,
                            float* hidden_out, float* logits_out, int32_t* token_out);
/* HipTalker::decode_step (talker.rs:251-292) at cache offset `offset`. */
int32_t qtts_talker_decode_step(qtts_engine* engine, const float* input, size_t offset,
                                float* hidden_out, float* logits_out, int32_t* token_out);
/* Same computation as qtts_talker_decode_step, for callers that may not
 * allocate device memory while running (fixed-budget or real-time hosts):
 * this call allocates nothing. Its working memory (the input row and every
 * layer's projections, attention output and MLP activations) comes from a
 * static device array of 264 KiB held by every GPU that loads the library;
 * talkers whose step activations exceed it are rejected with
 * QTTS_ERR_INVALID_INPUT.
 * The first call on a device looks up the array's address (make it before
 * any stream capture) and keeps it for the life of the process, which
 * assumes the device's primary context is never reset meanwhile
 * (cudaDeviceReset). Calls share the array: calls that overlap on the GPU
 * race. No counterpart in the reference. */
int32_t qtts_talker_decode_step_static(qtts_engine* engine, const float* input, size_t offset,
                                       float* hidden_out, float* logits_out,
                                       int32_t* token_out);
/* HipCodePredictor::generate_from_host (code_predictor.rs:283-300) with the
 * subtalker_* fields of options (greedy when subtalker_dosample == 0).
 * tokens_out [groups-1], embedding_sum_out [hidden], logits_out
 * [(groups-1) x cp_vocab] or NULL. */
int32_t qtts_code_predictor(qtts_engine* engine, const float* talker_hidden,
                            const float* semantic_embed, const qtts_generate_options* options,
                            int32_t* tokens_out, float* embedding_sum_out, float* logits_out);

/* Measurement seam (no reference counterpart): the step trace. While
 * enabled, frame 6 of every generation records for each kernel launch of the
 * frame graph (%globaltimer, ns after the frame's first kernel entry; -1 when
 * not recorded) the first CTA's entry, the first and last CTA past the
 * dependency wait, the last CTA's exit and two in-kernel marks (the input
 * staged, the dot products done), plus two per-CTA durations since the CTA's
 * own wait (max over CTAs). Enabling or disabling recaptures the frame
 * graphs. read: the last traced frame's launches in order (*n of them; at
 * most cap copied). */
typedef struct {
  char name[48];  /* kernel kind and shape, e.g. "gemv+swiglu N=3072 K=1024" */
  int64_t entry_ns, wait_ns, exit_ns, last_wait_ns, mark4_ns, mark5_ns;
  uint64_t dur6_ns, dur7_ns;
} qtts_trace_launch;
int32_t qtts_step_trace_enable(qtts_engine* engine, int32_t on);
int32_t qtts_step_trace_read(const qtts_engine* engine, qtts_trace_launch* out, size_t cap,
                             size_t* n);

/* Self-test of the library's bounded device waits (no reference
 * counterpart): one kernel waits for a device counter that nothing
 * increments, bounded by limit_us microseconds (at most 5 s), with the
 * acquire loads and %globaltimer bound every spin-wait of the library uses. Returns
 * QTTS_ERR_DEVICE_STATE ("a bounded device wait ran out") once the bound
 * expires; the engine stays usable afterwards. */
int32_t qtts_selftest_device_wait(qtts_engine* engine, uint32_t limit_us);

/* Device time of the last generation's frame loop (CUDA events), in ms. */
int32_t qtts_last_timings(const qtts_engine* engine, float* prefill_ms, float* frames_ms,
                          size_t* frames);

/* Kernels launched by the last generation (prefill launches + frame-graph
 * nodes x graph launches). */
int32_t qtts_last_launch_count(const qtts_engine* engine, size_t* kernels);

/* Measurement hook (no reference counterpart): times `launches` back-to-back
 * launches of one talker projection kernel, cycling through all layers'
 * weights, with CUDA events on the engine stream. which: 0 gate|up+SwiGLU,
 * 1 QKV, 2 down+residual, 3 O+residual. bytes_per_launch = algorithmic bytes
 * (bf16 weights + fp32 activations in/out). Clobbers the talker workspace. */
int32_t qtts_profile_projection(qtts_engine* engine, int32_t which, int32_t launches,
                                float* ms_per_launch, double* bytes_per_launch);

#ifdef __cplusplus
}
#endif

#endif /* QTTS_B200_H */
