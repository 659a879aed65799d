/*
 * whisper4j_cuda.h — C ABI of libwhisper4j_cuda.so, the B200 (sm_100a) Whisper
 * text-decoder token loop.
 *
 * The library replaces the reference's decoder hot path
 * (com.sparrowlogic.whisper4j.nn.WhisperDecoder and the nn/tensor code under it)
 * behind plain C types, so a Java host binds it with java.lang.foreign downcalls
 * and any C/C++/Python host with its own FFI.  All entry points return an int
 * status (W4J_OK = 0, negative on error); w4j_last_error() gives the message of
 * the calling thread's last failure.  A context is bound to one CUDA device;
 * calls on one context are serialised internally, separate contexts run
 * concurrently.
 *
 * Reference interfaces each entry point replaces are cited as file:line within
 * sparrowlogic/whisper4j (W4J = src/main/java/com/sparrowlogic/whisper4j).
 */
#ifndef WHISPER4J_CUDA_H
#define WHISPER4J_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define W4J_OK 0
#define W4J_ERR_ARG -1       /* IllegalArgumentException in the reference */
#define W4J_ERR_STATE -2     /* IllegalStateException (e.g. weights missing, closed) */
#define W4J_ERR_CUDA -3      /* CUDA runtime or kernel failure */
#define W4J_ERR_OOM -4       /* device allocation failed */
#define W4J_ERR_CANCELLED -5 /* w4j_cancel() observed between steps */

/* GGML tensor types (W4J/model/GgmlLoader.java:30-36). */
#define W4J_GGML_F32 0
#define W4J_GGML_F16 1
#define W4J_GGML_Q8_0 8

/* W4J/model/ModelDimensions.java:6-17, same field order. */
typedef struct w4j_dims {
    int32_t n_mels, n_audio_ctx, n_audio_state, n_audio_head, n_audio_layer;
    int32_t n_vocab, n_text_ctx, n_text_state, n_text_head, n_text_layer;
} w4j_dims;

typedef struct w4j_ctx w4j_ctx;

/* Last error message of the calling thread ("" if none). */
const char *w4j_last_error(void);

/* Library version string. */
const char *w4j_version(void);

/*
 * Create a decoder context on `device` (replaces `new WhisperDecoder(weights, dims)`,
 * W4J/nn/WhisperDecoder.java:36-56, called at W4J/WhisperModel.java:160).
 * max_streams: independent audio chunks decoded together by one call;
 * max_beam: largest beam size used (1 for greedy only).  Device memory for the
 * KV caches is sized from these and n_text_ctx / n_audio_ctx.
 */
int w4j_ctx_create(const w4j_dims *dims, int device, int max_streams, int max_beam, w4j_ctx **out);
int w4j_ctx_destroy(w4j_ctx *ctx);

/*
 * Upload one decoder tensor straight from the GGML file's bytes (the hook next
 * to GgmlLoader.dequantize, W4J/model/GgmlLoader.java:185-202).  `ne` is the
 * GGML shape (fastest dimension first), `data` the raw payload: F32, F16 or
 * Q8_0 (34-byte blocks).  Encoder tensors ("encoder.*") are kept on the same
 * device for w4j_encoder_forward (F16 / F32 matrices; a Q8_0 encoder matrix is
 * skipped with return 1).  Other names return 1.  Unknown decoder or encoder
 * tensor names, wrong shapes and unsupported types are errors.
 */
int w4j_upload_tensor(w4j_ctx *ctx, const char *name, int ggml_type, const int64_t *ne, int n_dims,
                      const void *data, size_t nbytes);

/* Check that every decoder tensor is present (WeightStore.get, W4J/model/WeightStore.java:28-34). */
int w4j_finalize(w4j_ctx *ctx);

/*
 * Set the encoder output xa (n_audio_ctx x n_audio_state f32, row-major, host
 * memory) of stream `slot` and project the cross-attention K/V of every layer
 * into the device cache (the first-call branch of MultiHeadAttention.forward,
 * W4J/nn/MultiHeadAttention.java:65-75).  The _device variant takes a device
 * pointer on the context's device.
 */
int w4j_set_encoder_output(w4j_ctx *ctx, int slot, const float *xa, int n_audio_ctx);
int w4j_set_encoder_output_device(w4j_ctx *ctx, int slot, const float *xa_device, int n_audio_ctx);

/*
 * Run the audio encoder on the device (replaces WhisperEncoder.forward, W4J/nn/WhisperEncoder.java:42-76,
 * with Conv1d.forward, W4J/nn/Conv1d.java:38-80): mel is the log-mel spectrogram, n_mels x n_frames f32
 * row-major host memory (the reference's (1, n_mels, n_ctx) tensor), n_frames = 2 * n_audio_ctx.  The
 * encoder weights ("encoder.*") come through w4j_upload_tensor like the decoder's, F16 or F32
 * matrices.  xa_out (host, n_audio_ctx x n_audio_state f32) receives the encoder output when not
 * NULL; slot >= 0 also sets that stream's encoder output on the device (as
 * w4j_set_encoder_output_device, no host round trip), which needs a finalized decoder.
 */
int w4j_encoder_forward(w4j_ctx *ctx, const float *mel, int n_frames, float *xa_out, int slot);

/*
 * The log-mel front end on the device (replaces FeatureExtractor.extract + padOrTrim,
 * W4J/audio/FeatureExtractor.java:68-160, with the model's filters as the
 * FeatureExtractor(nMels, melFilterData, nFftBins) constructor takes them, :44-55).
 * w4j_upload_mel_filters: the GGML file's mel filters, n_mels x n_bins f32 (n_fft = 2 (n_bins - 1)).
 * w4j_log_mel: 16 kHz mono samples -> n_mels x (2 n_audio_ctx) log-mel (host, when mel_out is not NULL).
 * w4j_encode_audio: the same spectrogram straight into the encoder (w4j_encoder_forward's outputs:
 * xa_out on the host, and / or stream `slot`'s cross K/V on the device) — one chunk of
 * WhisperModel.transcribe's feature + encoder stage (W4J/WhisperModel.java:361-366).
 */
int w4j_upload_mel_filters(w4j_ctx *ctx, const float *filters, int n_mels, int n_bins);
int w4j_log_mel(w4j_ctx *ctx, const float *audio, int n_samples, float *mel_out);
int w4j_encode_audio(w4j_ctx *ctx, const float *audio, int n_samples, float *xa_out, int slot);

/*
 * The chunked transcription loop (replaces WhisperModel.transcribeChunked, W4J/WhisperModel.java:334-427,
 * with parseTimestampSegments / findLastTimestampPos / buildPromptWithContext, :430-530): the whole
 * recording (16 kHz mono f32, host) is copied to the device once; per 30 s window at the seek
 * position the library runs the log-mel, the encoder, the cross K/V projection into stream 0 and
 * decodeWithFallback, retries without the previous-text context when it made the average
 * log-probability drop below -1, skips no-speech windows, cuts the tokens into timestamped
 * segments and advances the seek from the last timestamp.  Token ids only: the host's tokenizer
 * turns them into text.  A segment is kept when it has at least one text token (the reference keeps
 * it when the decoded text is not blank; the host drops segments whose text is blank).
 */
typedef struct w4j_transcribe_opts {
    const int32_t *sot;          /* tokenizer.sotSequence() (the prompt before the no-timestamps token) */
    int32_t n_sot;
    int32_t eot, no_speech;      /* token ids (tokenizer.eot(), tokenizer.noSpeech()) */
    int32_t no_timestamps;       /* appended to the prompt when ts_begin < 0 (buildPrompt, :573-582) */
    int32_t sot_prev;            /* the previous-text marker of buildPromptWithContext (:522-524) */
    int32_t ts_begin;            /* tokenizer.timestampBegin() with timestamps, -1 without */
    const int32_t *suppress;     /* buildSuppressTokens() */
    int32_t n_suppress;
    int32_t beam_size;           /* 1: greedy */
    int32_t condition_on_previous;
    uint64_t seed;               /* temperature-fallback sampling */
} w4j_transcribe_opts;

typedef struct w4j_segment {
    float start, end;            /* seconds */
    int32_t token_begin, n_tokens;  /* the segment's tokens: w4j_transcript.tokens[token_begin ..] */
} w4j_segment;

typedef struct w4j_transcript {
    int32_t *tokens;             /* caller's buffer: every segment's tokens, in order */
    int32_t tokens_cap;
    w4j_segment *segments;       /* caller's buffer */
    int32_t segments_cap;
    int32_t n_tokens, n_segments, n_windows;  /* out: used entries, 30 s windows decoded */
} w4j_transcript;

int w4j_transcribe(w4j_ctx *ctx, const float *audio, int n_samples, const w4j_transcribe_opts *opts,
                   w4j_transcript *out);

/*
 * WhisperDecoder.forward(tokens, xa, kvCache) (W4J/nn/WhisperDecoder.java:59-104)
 * for stream `slot`.  use_cache=1 appends the tokens to the slot's self-attention
 * cache (the kvCache map); use_cache=0 runs with an empty private cache and leaves
 * the slot's cache unchanged (kvCache == null, as detectLanguage does at
 * W4J/WhisperModel.java:548).  out_logits receives n_tokens x n_vocab f32.
 */
int w4j_forward(w4j_ctx *ctx, int slot, const int32_t *tokens, int n_tokens, int use_cache, float *out_logits);

/* Empty the self-attention cache of a stream (a fresh kvCache map). */
int w4j_reset_cache(w4j_ctx *ctx, int slot);

/*
 * Decode result per stream (WhisperDecoder.DecodeResult, W4J/nn/WhisperDecoder.java:672-673):
 * out_tokens[s * max_tokens .. + out_lens[s]) are the generated ids; sum/avg
 * log-probabilities, compression ratio and no-speech probability per stream.
 */
typedef struct w4j_result {
    int32_t *tokens;         /* n_streams * max_tokens */
    int32_t *lens;           /* n_streams */
    double *sum_logprob;     /* n_streams */
    float *avg_logprob;      /* n_streams */
    float *compression;      /* n_streams (zlib ratio, WhisperDecoder.java:628-647) */
    float *no_speech_prob;   /* n_streams */
} w4j_result;

/*
 * Greedy (temperature 0) or sampled decode of n_streams independent streams
 * (slots[i] names the stream whose encoder output was set), each starting from
 * its own prompt of n_prompt tokens (prompts: n_streams x n_prompt).  Mirrors
 * WhisperDecoder.decode (W4J/nn/WhisperDecoder.java:161-204) including the
 * logit processors (:450-564) and no-speech probability (:442-448).  ts_begin
 * <= 0 disables timestamp rules.  seed drives temperature sampling.
 */
int w4j_decode(w4j_ctx *ctx, const int32_t *slots, int n_streams, const int32_t *prompts, int n_prompt,
               int32_t eot, int max_tokens, const int32_t *suppress, int n_suppress, int32_t no_speech,
               float temperature, int32_t ts_begin, uint64_t seed, w4j_result *out);

/* Beam search (WhisperDecoder.decodeBeam, W4J/nn/WhisperDecoder.java:214-394). */
int w4j_decode_beam(w4j_ctx *ctx, const int32_t *slots, int n_streams, const int32_t *prompts, int n_prompt,
                    int32_t eot, int max_tokens, const int32_t *suppress, int n_suppress, int32_t no_speech,
                    int32_t ts_begin, int beam, w4j_result *out);

/*
 * Temperature-fallback policy (WhisperDecoder.decodeWithFallback,
 * W4J/nn/WhisperDecoder.java:119-149): beam search (beam > 1) or greedy at
 * t = 0, then sampling at 0.2 .. 1.0 while needsFallback (:435-440) holds.
 * out_temperature receives the temperature of the returned result per stream.
 */
int w4j_decode_with_fallback(w4j_ctx *ctx, const int32_t *slots, int n_streams, const int32_t *prompts,
                             int n_prompt, int32_t eot, int max_tokens, const int32_t *suppress, int n_suppress,
                             int32_t no_speech, int32_t ts_begin, int beam, uint64_t seed, w4j_result *out,
                             float *out_temperature);

/* Ask a running decode on this context to stop at its next step boundary
 * (TranscriptionHandle cancellation, W4J/WhisperModel.java:620-633). */
int w4j_cancel(w4j_ctx *ctx);

/* Host-side helpers of the policy (no device work). */
float w4j_compression_ratio(const int32_t *tokens, int n);                            /* :628-647 */
int w4j_needs_fallback(float compression_ratio, float avg_logprob, float no_speech);  /* :435-440 */

/*
 * Timing of the last decode call on this context: device milliseconds from the
 * first prompt kernel to the end of the result gather (the cross K/V projection
 * of w4j_set_encoder_output excluded), the number of graph-replayed steps after
 * the prompt, and the number of kernels launched.
 */
int w4j_last_timing(w4j_ctx *ctx, double *loop_ms, int *steps, long long *kernel_launches);

/*
 * In-chain kernel timing (measurement; no counterpart in the reference).  With a kernel class
 * set, the step graphs of later decode calls are captured with CUDA event records around every
 * launch of that class, and each step is waited for, so w4j_kernel_timing returns the summed
 * device milliseconds and the number of those launches over the graph-replayed steps of the last
 * decode call.  The events cost each timed launch its overlap with the launch before it, so use
 * this for a separate profiling call, not for the timed throughput.  Classes: 0 off,
 * 1 projections, 2 self-attention, 3 cross-attention, 4 vocabulary logits, 5 token selection.
 */
#define W4J_KC_PROJ 1
#define W4J_KC_SELF_ATTN 2
#define W4J_KC_CROSS_ATTN 3
#define W4J_KC_LOGITS 4
#define W4J_KC_SELECT 5
int w4j_set_kernel_timing(w4j_ctx *ctx, int kernel_class);
int w4j_kernel_timing(w4j_ctx *ctx, double *ms, long long *launches);

/* ---------------------------------------------------------------------------
 * Op-level entry points on device buffers (plain pointers on the context's
 * device, stream 0 of the calling thread unless `stream` is given).  They run
 * single kernels of the step for tests and for hosts that drive their own loop.
 * ------------------------------------------------------------------------- */

/*
 * y = LN?(x) . W^T + b for M rows (Linear.forward, W4J/nn/Linear.java:23-26,
 * optionally preceded by LayerNorm.forward, W4J/nn/LayerNorm.java:28-30).
 * W is a GGML F16 or Q8_0 payload already on the device: F16 (N x K halves), or
 * Q8_0 repacked by w4j_q8_0_repack.  ln_g/ln_b may be NULL (no LayerNorm).
 * epilogue: 0 = store, 1 = GELU (Tensor.geluInPlace), 2 = residual y += ...
 */
int w4j_op_linear(w4j_ctx *ctx, const float *x, int M, int K, const void *W, int w_type, int N,
                  const float *bias, const float *ln_g, const float *ln_b, int epilogue, float *y, void *stream);

/* Split a GGML Q8_0 payload (N*K/32 blocks of 34 bytes, device) into the
 * device layout: int8 quants (N x K) then f16 scales (N x K/32). dst holds N*K + N*K/16 bytes. */
int w4j_q8_0_repack(const void *src_device, int N, int K, void *dst_device, void *stream);

/*
 * logits = LN(x) . E^T over the vocabulary followed by argmax and log-softmax
 * of the chosen id, for M rows (WhisperDecoder.java:102-103 then argmax :566-574
 * and logSoftmax :614-626).  x: M x d f32, E: V x d f16, ln: d f32 each;
 * outputs token ids (M) and log-probabilities (M, double).  Scratch memory for
 * the per-block partial results is taken from the context (1 <= M <= max(max_streams *
 * max_beam, n_text_ctx)).  If a bounded wait inside the kernels ran out, every out_token of
 * that call is -1 and every out_logprob NaN (the context's error word for this op is cleared
 * for the next call).  Asynchronous on `stream`.
 */
int w4j_op_logits_argmax(w4j_ctx *ctx, const float *x, int M, const void *E, int V, const float *ln_g,
                         const float *ln_b, int32_t *out_token, double *out_logprob, void *stream);

/*
 * w4j_op_logits_argmax_noalloc — no counterpart in the reference.
 *
 * The computation of w4j_op_logits_argmax (same kernels, same results) for callers that
 * cannot let the library allocate device memory: a host that has handed the whole device to
 * its own arena or caching allocator (so a cudaMalloc would fail or fragment it), a process
 * under a fixed device-memory budget, or code that only needs this one op and holds no
 * decoder context (creating one allocates the weights, caches and scratch of a whole model).
 * It takes no context and never calls cudaMalloc, cudaFree or an allocating library routine.
 *
 * Scratch: the per-block partial results live in a file-scope device array of the library
 * (W4J_NOALLOC_MAX_ROWS x W4J_NOALLOC_MAX_PARTS records of 144 bytes = 360 KiB per device),
 * found with cudaGetSymbolAddress on the first call for each device.  That first call also
 * sets kernel attributes; make it before any stream capture begins on that device.
 * Nothing in the partials has to start at zero (each call writes every record it reads).
 * One device error word must be zero when a call starts: it is zero when the library loads,
 * and each call clears it at the end.
 *
 * Limits: 1 <= M <= W4J_NOALLOC_MAX_ROWS; d a multiple of 64 in [64, 1280]; x, E, ln_g and
 * ln_b 16-byte aligned; min(SM count, V) <= W4J_NOALLOC_MAX_PARTS.  Outside them the call
 * returns W4J_ERR_ARG with the reason in w4j_last_error() and launches nothing.
 *
 * Concurrency: calls on one device share the scratch.  Two calls whose executions overlap on
 * the device (different streams without an event between them, or different host threads)
 * race and return wrong ids; order them on one stream, or with events.
 *
 * device: the GPU holding every pointer (made current on the calling thread).  x: M x d f32,
 * E: V x d f16, ln_g/ln_b: d f32; out_token (M int32) and out_logprob (M double) on the device.
 * If a bounded wait inside the kernels ran out, every out_token of that call is -1 and every
 * out_logprob NaN.  Asynchronous on `stream` (NULL = legacy default stream).
 */
/*
 * Test hook (no counterpart in the reference): the next n_launches tcgen05 vocabulary passes of
 * w4j_op_logits_argmax / w4j_op_logits_argmax_noalloc issue none of their weight copies, so
 * every bounded wait inside them runs out (about a second) and the call reports it through its
 * error word (token -1, NaN log-probability).  Lets a test exercise that path without faulting
 * the GPU.  0 turns it off.
 */
int w4j_test_withhold_logits_copies(int n_launches);

#define W4J_NOALLOC_MAX_ROWS 16
#define W4J_NOALLOC_MAX_PARTS 160
int w4j_op_logits_argmax_noalloc(int device, const float *x, int M, int d, const void *E, int V,
                                 const float *ln_g, const float *ln_b, int32_t *out_token, double *out_logprob,
                                 void *stream);

#ifdef __cplusplus
}
#endif
#endif /* WHISPER4J_CUDA_H */
