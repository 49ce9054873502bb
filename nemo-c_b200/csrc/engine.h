/* Streaming engine: B independent streams advanced in lockstep through the cache-aware encoder
   step and the greedy RNNT decoder. B = 1 is the reference's single session (src/encoder.c,
   src/decoder.c); B > 1 batches streams so every GEMM has B x chunk rows. */
#ifndef NB_ENGINE_H
#define NB_ENGINE_H
#include "model.h"

typedef struct nb_engine nb_engine_t;

nb_engine_t *nb_engine_create(nb_model_t *m, int streams, int right, char *err, size_t errlen);
void nb_engine_destroy(nb_engine_t *e);
/* Back to the state after create (src/encoder.c:92-103 + src/decoder.c:48-53), keeping buffers. */
int nb_engine_reset(nb_engine_t *e, char *err, size_t errlen);
int nb_engine_right(const nb_engine_t *e);
int nb_engine_streams(const nb_engine_t *e);
/* Per-stream language prompt index (src/model.c:312-322 fold). */
int nb_engine_set_prompt(nb_engine_t *e, int stream, int prompt_index, char *err, size_t errlen);
/* Read all input from a device-resident mel sequence instead of the host queue: stream s's
   frames at d_mel + s*sstride_floats, `frames` frames each. Only right after create/reset. */
int nb_engine_attach_device_mel(nb_engine_t *e, const float *d_mel, int64_t sstride_floats, size_t frames, char *err, size_t errlen);
/* Queue nframes mel rows (128 floats each) for every stream: mel[s] points at stream s's rows. */
int nb_engine_push(nb_engine_t *e, const float *const *mel, size_t nframes, char *err, size_t errlen);
/* GPU log-mel: stage each stream's sample span (nb_mel_stage) into nb_engine_span after
   nb_engine_span_wait, then nb_engine_push_spans with the frame count. */
int nb_engine_gpu_mel(const nb_engine_t *e);
float *nb_engine_span(nb_engine_t *e, int s, size_t *cap);
int nb_engine_span_wait(nb_engine_t *e);
int nb_engine_push_spans(nb_engine_t *e, size_t nframes, char *err, size_t errlen);
/* The same in two parts, so staging and uploading can overlap: upload streams [s0, s1) of the
   staged spans (nframes frames each), then, once every stream was uploaded, transform them. */
int nb_engine_upload_spans(nb_engine_t *e, int s0, int s1, size_t nframes, char *err, size_t errlen);
int nb_engine_finish_spans(nb_engine_t *e, size_t nframes, char *err, size_t errlen);
/* GPU resampler: the sums of every stream's nb_resampler_plan job (identical across streams but
   for the FIFO contents); out[s] gets stream s's job.count outputs in pinned host memory. */
int nb_engine_resample(nb_engine_t *e, const nb_resample_job_t *jobs, const float **out, char *err, size_t errlen);
int nb_engine_gpu_resample(const nb_engine_t *e, int in_rate);
/* One encoder step + greedy decode (src/encoder.c:213-267 then src/decoder.c:92-127).
   Returns 1 if a piece was consumed, 0 if nothing to do, -1 on error. Tokens of stream s are
   appended to tokens[s*max_tokens + counts[s] ...] and counts[s] advanced; *frames = rows. */
int nb_engine_step(nb_engine_t *e, int final, int *tokens, int max_tokens, int *counts, int *frames, char *err, size_t errlen);
/* Parity taps: every encoder row produced from now on (per chunk: B*c rows, stream-major) is
   copied to prompted [rows][D] / joint_enc [rows][JH] (host), chunk_rows[k] = c of chunk k. */
void nb_engine_set_taps(nb_engine_t *e, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks);
void nb_engine_tap_counts(const nb_engine_t *e, size_t *rows, size_t *chunks);
void nb_engine_times(const nb_engine_t *e, double *enc_ms, double *dec_ms, size_t *chunks);
/* Capture the graphs of every chunk shape this engine's latency can produce (nothing runs, the
   stream state is kept): the warm-up of nemoasr_prepare_latency. */
int nb_engine_prepare(nb_engine_t *e, char *err, size_t errlen);
/* Graphs captured so far. */
int nb_engine_graphs(const nb_engine_t *e);
/* Decoder counts since reset: [0] stream-frames decoded, [1] of them whose first decision emitted
   a token, [2] greedy decisions, [3] greedy loop iterations ([1], [2] = -1 for the persistent
   single-stream decoder, which does not keep them). */
int nb_engine_decode_counts(nb_engine_t *e, long long out[4], char *err, size_t errlen);
/* Device time (CUDA events on the engine's stream) summed over every step that ran GPU work. */
double nb_engine_gpu_ms(const nb_engine_t *e);

#endif
