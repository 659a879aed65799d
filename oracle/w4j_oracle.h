/*
 * w4j_oracle.h — CPU restatement of whisper4j's decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never part of the
 * product library.  See w4j_oracle.c for the reference file:line each function
 * restates.
 */
#ifndef W4J_ORACLE_H
#define W4J_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int n_vocab, n_audio_ctx, n_text_ctx, n_text_state, n_text_head, n_text_layer;
} orc_dims;

typedef struct orc_model orc_model;
typedef struct orc_cache orc_cache;

const char *orc_last_error(void);
/* Wall seconds of the last decode's token loop after its first step (prompt and cross K/V
 * projection excluded), on the calling thread. */
double orc_last_loop_seconds(void);

/* Threads of the oracle's own loops (default 1, the reference's single-threaded decoder);
 * results do not depend on it. */
void orc_set_threads(int n);

orc_model *orc_model_new(const orc_dims *d);
void orc_model_free(orc_model *m);
/* name: canonical GGML tensor name; data: f32 values in the file's row-major
 * order (GGML `ne` reversed).  Returns 0 when stored, 1 when the tensor is not
 * on the decoder path (ignored), -1 on error. */
int orc_set_tensor(orc_model *m, const char *name, const float *data, long n);
int orc_model_check(const orc_model *m);
const float *orc_gelu_table(const orc_model *m);

orc_cache *orc_cache_new(const orc_model *m, int n_audio_ctx);
void orc_cache_free(orc_cache *c);
int orc_cache_len(const orc_cache *c);

/* WhisperDecoder.forward(tokens, xa, kvCache): logits (n, n_vocab). cache may be NULL. */
int orc_forward(const orc_model *m, const int *tokens, int n, const float *xa, int n_audio_ctx, orc_cache *cache,
                float *logits);

/* WhisperDecoder.decode(...) — max_steps > 0 stops after that many steps (bounded samples). */
int orc_decode(const orc_model *m, const float *xa, int n_audio_ctx, const int *prompt, int n_prompt, int eot,
               int max_tokens, const int *suppress, int n_suppress, int no_speech, float temperature, int ts_begin,
               uint64_t seed, int *out_tokens, int *out_len, double *out_sum_logprob, float *out_avg_logprob,
               float *out_no_speech_prob, int max_steps);

/* WhisperDecoder.decodeBeam(...) */
int orc_decode_beam(const orc_model *m, const float *xa, int n_audio_ctx, const int *prompt, int n_prompt, int eot,
                    int max_tokens, const int *suppress, int n_suppress, int no_speech, int ts_begin, int beam,
                    int *out_tokens, int *out_len, double *out_sum_logprob, float *out_avg_logprob,
                    float *out_no_speech_prob, int max_steps);

/* Beam-search trace (parity tests): while set, orc_decode_beam on this thread appends 5 doubles
 * per ranked candidate: step, parent beam, token, score, outcome (kept beam index, -2 finished,
 * -1 dropped or not reached).  buf = NULL stops tracing. */
void orc_set_beam_trace(double *buf, long cap_entries);
long orc_beam_trace_count(void);

/* processors exposed for unit tests */
void orc_apply_repetition_penalty(float *logits, const int *gen, int count, int n);
void orc_apply_timestamp_rules(float *logits, const int *gen, int count, int ts_begin, int eot, int n, int is_first);

/* tensor KATs (TensorTest.java / SimdOpsTest.java) */
float orc_dot(const float *a, const float *b, int n);
void orc_matmul(const float *a, const float *b, int M, int K, int N, float *out);
void orc_matmul_transb(const float *a, const float *b, int M, int K, int N, float alpha, float *out);
void orc_softmax_rows(float *x, int rows, int n);
void orc_layer_norm(const float *x, int rows, int n, const float *g, const float *b, float eps, float *y);
void orc_gelu(const orc_model *m, float *x, long n);
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);

/* ---- audio encoder (WhisperEncoder.java:42-76, Conv1d.java:38-80) ---- */
typedef struct {
    int n_mels, n_audio_ctx, n_audio_state, n_audio_head, n_audio_layer;
} orc_enc_dims;
typedef struct orc_encoder orc_encoder;

orc_encoder *orc_encoder_new(const orc_enc_dims *d);
void orc_encoder_free(orc_encoder *e);
/* name: canonical GGML tensor name, data: f32 values in row-major order (GGML `ne` reversed).
 * Returns 0 when stored, 1 when the tensor is not an encoder tensor, -1 on a bad name or size. */
int orc_encoder_set_tensor(orc_encoder *e, const char *name, const float *data, long n);
int orc_encoder_check(const orc_encoder *e);
/* mel: (n_mels, 2 n_audio_ctx) row-major, as the reference's (1, n_mels, n_ctx) input;
 * out: (n_audio_ctx, n_audio_state), the encoder output xa.  Returns 0 or -1. */
int orc_encoder_forward(const orc_encoder *e, const float *mel, float *out);

/* FeatureExtractor.extract + padOrTrim (FeatureExtractor.java:68-160): log-mel spectrogram of 16 kHz
 * mono samples with the model's filters (n_mels x n_bins, n_fft = 2 (n_bins - 1)), hop samples per
 * frame, out: n_mels x out_frames (first frames, or padded with the spectrogram's minimum). */
int orc_log_mel(const float *audio, int n_samples, const float *filters, int n_mels, int n_bins, int hop,
                int out_frames, float *out);

#ifdef __cplusplus
}
#endif
#endif
