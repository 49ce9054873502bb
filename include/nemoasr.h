/* nemoasr (B200 build): streaming Nemotron-ASR encoder step + greedy RNNT decoder on sm_100a.

   Public C API. The first block is the drop-in surface of the reference library
   (src/nemoasr.h:25-54 in nemoasr-c): the same names, argument meaning, return conventions and
   error behaviour (NULL / -1 with a message in err). The second block adds what a B200 deployment
   needs beyond it: opening a seeded random-init model of the published architecture, writing that
   model as a checkpoint in the reference's own format, and batching many independent streams on
   one GPU.

   Threading: like the reference, a session (or batch) is not thread-safe; call it from one
   thread. Different sessions may live on different threads / devices. */
#ifndef NEMOASR_B200_H
#define NEMOASR_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nemoasr nemoasr_t;

typedef struct {
    double audio_seconds;
    size_t chunks, tokens;
    double encoder_ms, decoder_ms;
} nemoasr_stats_t;

/* ---- reference surface (src/nemoasr.h) ------------------------------------------------- */

/* Replaces src/nemoasr.h:25 (nemoasr_default_model_dir): the Hugging Face cache snapshot of
   the model, if one exists. Returns 0 and fills out when found, -1 otherwise. */
int nemoasr_default_model_dir(char *out, size_t n);

/* Replaces src/nemoasr.h:31 (nemoasr_open). model_dir holds config.json + model.safetensors
   in the reference's format (bf16 tensors, reference tensor names). A model_dir of the form
   "synthetic:<seed>" opens the seeded random-init model of the full published architecture
   (same as nemoasr_open_synthetic with nemoasr_synth_default()). latency_ms: 80, 160, 320,
   560 or 1120 (must be trained for the checkpoint). input_rate: rate of the audio fed. */
nemoasr_t *nemoasr_open(const char *model_dir, const char *language, int latency_ms, int input_rate, char *err, size_t errlen);
/* Replaces src/nemoasr.h:32. */
void nemoasr_close(nemoasr_t *s);
/* Replaces src/nemoasr.h:38. Returns newly decoded text (malloc'd, free with nemoasr_free) or
   NULL when nothing new; on failure NULL with a non-empty message in err. final=1 flushes. */
char *nemoasr_feed(nemoasr_t *s, const float *samples, size_t n, int final, char *err, size_t errlen);
/* Replaces src/nemoasr.h:39. */
void nemoasr_free(char *text);
/* Replaces src/nemoasr.h:45: fresh stream on the same model (language may be NULL = keep). */
int nemoasr_reset(nemoasr_t *s, const char *language, int latency_ms, char *err, size_t errlen);
/* Replaces src/nemoasr.h:49 (warm-up, src/warmup.c:23-42): captures the CUDA graph of every chunk
   shape a stream at this latency can produce (first, steady and every final chunk), without
   running them and without touching the current stream. For the session's own latency the
   graphs go to its engine; for another latency to an engine kept for it, which the next
   nemoasr_reset to that latency takes over. A stream after that reset captures no graph. The
   engine a latency change replaces is kept the same way (one single-stream engine, ~0.1 GB of
   device memory, per latency used). */
int nemoasr_prepare_latency(nemoasr_t *s, int latency_ms, char *err, size_t errlen);
/* CUDA graphs the session's current engine has captured so far (warm-up checks). */
int nemoasr_graphs_captured(const nemoasr_t *s);
double nemoasr_load_ms(const nemoasr_t *s);      /* src/nemoasr.h:51 */
const char *nemoasr_gpu_name(const nemoasr_t *s); /* src/nemoasr.h:52 */
int nemoasr_latency_ms(const nemoasr_t *s);      /* src/nemoasr.h:53 */
void nemoasr_stats(const nemoasr_t *s, nemoasr_stats_t *out); /* src/nemoasr.h:54 */

/* Same as nemoasr_feed but returns token ids: appends up to max_tokens ids to tokens and
   returns how many were appended (-1 on error). For callers with their own detokenizer. */
int nemoasr_feed_tokens(nemoasr_t *s, const float *samples, size_t n, int final, int *tokens, int max_tokens, char *err, size_t errlen);
/* Parity taps, like the reference CLI's --dump-enc (src/main.c:99): every encoder row produced
   from now on is copied to prompted [rows][d_model] and joint_enc [rows][joint_hidden] (host
   arrays of cap_rows rows); chunk_rows[k] receives the row count of chunk k. */
void nemoasr_set_taps(nemoasr_t *s, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks);
void nemoasr_tap_counts(const nemoasr_t *s, size_t *rows, size_t *chunks);

/* ---- synthetic model (no counterpart in the reference; its checkpoint is not used) ------- */

typedef struct {
    uint64_t seed;
    int n_layers, d_model, ff_factor, sub_channels, num_prompts, prompt_hidden;
    int pred_hidden, joint_hidden, vocab_size;
    int att_left;
    float weight_std;  /* every bf16 weight and bias ~ N(0, weight_std^2); LN gamma 1, beta 0 */
    float blank_bias;  /* added to joint.joint_net.2.bias[blank] (sets the token emission rate) */
} nemoasr_synth_spec_t;

/* Full published shape: 24 layers, d_model 1024, 8x128 heads, FF 4096, 256 subsampling
   channels, prompt 128 -> 2048, LSTM 2x640, joint 640, vocab 1024 + blank, seed 1234. */
void nemoasr_synth_default(nemoasr_synth_spec_t *spec);
/* Write config.json + model.safetensors for spec into dir (created if missing). */
int nemoasr_synth_write(const char *dir, const nemoasr_synth_spec_t *spec, char *err, size_t errlen);
/* Same model as nemoasr_synth_write + nemoasr_open(dir), generated in memory. */
nemoasr_t *nemoasr_open_synthetic(const nemoasr_synth_spec_t *spec, const char *language, int latency_ms, int input_rate, char *err, size_t errlen);
/* Seeded synthetic audio: three linear 100->4000 Hz chirps (amplitude 0.15 each) + N(0, 0.05^2)
   noise; pauses=1 mutes the chirps in random 200-600 ms gaps between 1-3 s segments. */
void nemoasr_synth_audio(uint64_t seed, int rate, size_t n, int pauses, float *out);

/* ---- host front end used by nemoasr_feed (the reference keeps these internal: src/mel.h,
   src/resample.h) ------------------------------------------------------------------------ */
typedef struct nemoasr_mel nemoasr_mel_t;
typedef struct nemoasr_resampler nemoasr_resampler_t;
/* Streaming 128-bin log-mel at 16 kHz (src/mel.h:17-23): push samples, get the frames that
   became complete (at most max_frames written to out, 128 floats each). final=1 flushes. */
nemoasr_mel_t *nemoasr_mel_create(void);
size_t nemoasr_mel_push(nemoasr_mel_t *m, const float *samples, size_t n, int final, float *out, size_t max_frames);
void nemoasr_mel_destroy(nemoasr_mel_t *m);
/* Streaming windowed-sinc resampler (src/resample.h:6-11). */
nemoasr_resampler_t *nemoasr_resampler_create(int in_rate, int out_rate);
size_t nemoasr_resampler_process(nemoasr_resampler_t *r, const float *in, size_t n, float *out, size_t out_max);
size_t nemoasr_resampler_flush(nemoasr_resampler_t *r, float *out, size_t out_max);
void nemoasr_resampler_destroy(nemoasr_resampler_t *r);

/* ---- batched streams (no counterpart in the reference: it runs one stream per process) ---- */

typedef struct nemoasr_batch nemoasr_batch_t;

/* B independent streams on the current CUDA device, advanced in lockstep (every stream is fed
   the same number of samples per call). languages: B prompt keys, or NULL for "auto". */
nemoasr_batch_t *nemoasr_batch_open(const char *model_dir, const nemoasr_synth_spec_t *synth, int n_streams,
                                    const char *const *languages, int latency_ms, int input_rate, char *err, size_t errlen);
void nemoasr_batch_close(nemoasr_batch_t *b);
/* Feed n samples to each stream: samples[s] points at stream s's block. Emitted token ids are
   appended to tokens[s*max_tokens ...]; counts[s] receives the number written this call.
   Returns 0 or -1 (err). */
int nemoasr_batch_feed(nemoasr_batch_t *b, const float *const *samples, size_t n, int final,
                       int *tokens, int max_tokens, int *counts, char *err, size_t errlen);
int nemoasr_batch_reset(nemoasr_batch_t *b, char *err, size_t errlen);
void nemoasr_batch_stats(const nemoasr_batch_t *b, nemoasr_stats_t *out);
/* Greedy-decoder counts since open/reset (the emission rate of a workload): out[0] stream-frames
   decoded, out[1] of them whose first decision emitted a token (the frames that emit), out[2]
   greedy decisions, out[3] greedy-loop iterations (one decision for every still-active stream
   per iteration, src/decoder.c:97-123). out[1], out[2] are -1 for a batch of one stream (its
   persistent decoder keeps no counts). Waits for the batch's work. Returns 0 or -1 (err). */
int nemoasr_batch_decode_counts(nemoasr_batch_t *b, long long out[4], char *err, size_t errlen);
/* Device-resident input (throughput runs with the features already in HBM): after open/reset,
   read every stream's log-mel frames from d_mel (device pointer, stream s at
   d_mel + s*stream_stride floats, `frames` frames of 128 floats each) instead of fed audio. */
int nemoasr_batch_attach_mel(nemoasr_batch_t *b, const float *d_mel, int64_t stream_stride, size_t frames, char *err, size_t errlen);
/* One chunk step of every stream (encoder step + greedy decode). Returns 1 if a chunk was
   consumed (*rows encoder rows per stream, may be 0), 0 when nothing is pending, -1 on error.
   final=1 lets the last partial chunk through. Tokens as in nemoasr_batch_feed (counts are
   not cleared: ids are appended at tokens[s*max_tokens + counts[s]]). */
int nemoasr_batch_step(nemoasr_batch_t *b, int final, int *tokens, int max_tokens, int *counts, int *rows, char *err, size_t errlen);
/* Device time in ms (CUDA events on the batch's stream, from the first command of a step to the
   last token read-back) summed over all steps so far. */
double nemoasr_batch_gpu_ms(const nemoasr_batch_t *b);
/* Taps as nemoasr_set_taps; each chunk contributes n_streams * rows rows, stream-major. */
void nemoasr_batch_set_taps(nemoasr_batch_t *b, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks);

#ifdef __cplusplus
}
#endif
#endif
