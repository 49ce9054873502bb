/* ORACLE — TEST INFRASTRUCTURE ONLY. Not part of the product: only tests/, the smoke check in
   __graft_entry__.py and bench.py's cpu_baseline / reference arm load this library, as the checker
   or as the timed CPU baseline.

   A plain-C fp32 restatement of the reference's hot path (nemoasr-c):
     - every device kernel of src/kernels.metal (bf16 weights widened exactly, fp32 math);
     - the streaming bookkeeping of src/encoder.c, src/decoder.c and src/nemoasr.c;
     - the load-time tables of src/model.c (rel-pos table, language bias fold);
     - the host front end of src/mel.c and src/resample.c.
   Parity pin: oracle/ref_gpu_cpu.c runs the reference's own host C sources (compiled in place by
   oracle/Makefile into oracle/_ref/) on these kernels, and tests/golden/ holds the outputs of that
   build; tests check this restatement against them. */
#ifndef NEMO_ORACLE_H
#define NEMO_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- kernels (src/kernels.metal) ------------------------------------------------------- */
/* act: 0 none, 1 SiLU, 2 ReLU, 3 GLU (columns n and n+N/2 -> N/2 outputs a*sigmoid(b)). */
void or_gemm(const float *A, int lda, const uint16_t *W, int ldw, const float *bias, float *C, int ldc,
             int M, int N, int K, int act, int accumulate, float alpha);
void or_layernorm(const float *X, const float *g, const float *b, float *Y, int M, int D, float eps);
void or_layernorm2(const float *X, const float *g1, const float *b1, const float *g2, const float *b2,
                   float *Y1, float *Y2, int M, int D, float eps);
void or_attention_rel(const float *Q, int ldq, const float *K, const float *V, int ldk, const float *P,
                      const float *bias_u, const float *bias_v, float *O, int c, int L, int Lmax, int H, int dh, int D, float scale);
void or_dwconv_ln_silu(const float *din, const float *W, const float *g, const float *b, float *Y, int c, int D, int taps, float eps);
void or_conv2d_c1_s2_relu(const float *X, const float *W, const float *bias, float *Y, int T, int F, int T1, int F1, int C);
void or_dwconv2d_s2(const float *X, const float *W, const float *bias, float *Y, int T, int F, int T1, int F1, int C);
void or_flatten_cf(const float *X, float *Y, int T, int F, int C);
void or_lstm_cell(const float *gates, const float *c_in, float *c_out, float *h_out, int H);
/* joint + argmax for `rows` frames: ties -> lowest index. out_idx[r], out_val[r]; out_margin[r]
   (may be NULL) = best - second best logit. */
void or_joint_argmax(const float *enc, int enc_ld, const float *pred, const uint16_t *W, const float *bias,
                     int V, int H, int rows, int *out_idx, float *out_val, float *out_margin);

/* ---- model (src/model.c) --------------------------------------------------------------- */
typedef struct {
    int n_layers, d_model, n_heads, d_ff, sub_channels, feat_in, num_prompts, prompt_hidden;
    int pred_hidden, vocab_size, joint_hidden, max_symbols, att_left, max_right;
} or_config_t;
typedef struct or_model or_model_t;
/* Tensors by name (bf16, reference names). Returns NULL with err on a missing/mis-sized tensor. */
or_model_t *or_model_create(const or_config_t *cfg, int n, const char *const *names, const uint16_t *const *data,
                            const size_t *numel, char *err, size_t errlen);
int or_model_set_language(or_model_t *m, int prompt_index);
void or_model_free(or_model_t *m);
/* Copy of the per-layer rel-pos table [2*Lmax-1][D] (for kernel-level tests). */
const float *or_model_ptab(const or_model_t *m, int layer);
const float *or_model_prompt_bias(const or_model_t *m);

/* ---- streaming session (src/nemoasr.c + encoder.c + decoder.c) ------------------------- */
typedef struct or_session or_session_t;
or_session_t *or_open(or_model_t *m, int latency_ms, int input_rate, char *err, size_t errlen);
void or_close(or_session_t *s);
/* Feed samples; appends emitted token ids to tokens (up to max_tokens), returns how many, -1 on error. */
int or_feed(or_session_t *s, const float *samples, size_t n, int final, int *tokens, int max_tokens, char *err, size_t errlen);
/* Record every encoder row produced from now on: prompted [rows][D], joint_enc [rows][JH],
   chunk_rows[chunk] = rows of that chunk; plus one decision record per joint evaluation whose
   result was used (frame index, argmax, margin). Capacities in rows / chunks / decisions. */
void or_set_taps(or_session_t *s, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks,
                 int *dec_frame, int *dec_token, float *dec_margin, size_t cap_dec);
void or_tap_counts(const or_session_t *s, size_t *rows, size_t *chunks, size_t *decisions);
void or_stats(const or_session_t *s, double *audio_s, size_t *chunks, size_t *tokens);

/* ---- front end (src/mel.c, src/resample.c) --------------------------------------------- */
typedef struct or_mel or_mel_t;
or_mel_t *or_mel_create(void);
void or_mel_destroy(or_mel_t *m);
/* Returns the number of new 128-bin frames written to out (capacity max_frames). */
size_t or_mel_push(or_mel_t *m, const float *samples, size_t n, int final, float *out, size_t max_frames);
typedef struct or_resampler or_resampler_t;
or_resampler_t *or_resampler_create(int in_rate, int out_rate);
void or_resampler_destroy(or_resampler_t *r);
size_t or_resampler_process(or_resampler_t *r, const float *in, size_t n, float *out, size_t out_max);
size_t or_resampler_flush(or_resampler_t *r, float *out, size_t out_max);

int or_num_threads(void);

/* ---- synthetic workload (oracle_synth.c): the benchmark's random-init checkpoint and audio --- */
typedef struct {  /* same layout as nemoasr_synth_spec_t */
    uint64_t seed;
    int n_layers, d_model, ff_factor, sub_channels, num_prompts, prompt_hidden;
    int pred_hidden, joint_hidden, vocab_size;
    int att_left;
    float weight_std, blank_bias;
} or_synth_spec_t;
void or_synth_default(or_synth_spec_t *s);
int or_synth_write(const char *dir, const or_synth_spec_t *s, char *err, size_t errlen);
void or_synth_audio(uint64_t seed, int rate, size_t n, int pauses, float *out);

#ifdef __cplusplus
}
#endif
#endif
