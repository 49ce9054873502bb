/* Internal declarations shared by the host C files of the B200 build. */
#ifndef NB_H
#define NB_H
#include "../../include/nemoasr.h"
#include "../../include/nemo_gpu.h"
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NB_MEL_SR 16000
#define NB_MEL_NFFT 512
#define NB_MEL_WIN 400
#define NB_MEL_HOP 160
#define NB_MEL_NMEL 128
#define NB_MEL_NFREQ (NB_MEL_NFFT / 2 + 1)
#define NB_MEL_CACHE 16        /* mel rows carried into the next window */
#define NB_SPAN_FRAMES 128     /* most frames one staged sample span yields (GPU log-mel) */
#define NB_EPOCH_CHUNKS 8      /* caches are compacted once per this many max-size chunks */
#define NB_MIN_CMAX 16         /* cache capacity is sized for at least this many rows per chunk */

/* ---- model configuration (the fields src/model.c:125-172 parses from config.json) -------- */
typedef struct {
    int n_layers, d_model, n_heads, head_dim, d_ff, subsampling, sub_channels, conv_kernel, feat_in;
    int num_prompts, prompt_hidden;
    int pred_hidden, pred_layers, vocab_size, blank_id, joint_hidden, num_classes, max_symbols;
    int att_left, att_right_default;
    int trained_right[8], n_trained;
    float ln_eps;
    int Lmax;          /* att_left + largest trained right context + 1 + 2 */
    int sub_freq_out;  /* frequency bins after 3 stride-2 stages (17 for 128 mel bins) */
} nb_config_t;

/* ---- tiny JSON DOM -------------------------------------------------------------------- */
typedef enum { NBJ_NULL, NBJ_BOOL, NBJ_NUM, NBJ_STR, NBJ_ARR, NBJ_OBJ } nbj_type;
typedef struct nbj {
    nbj_type type;
    double num;
    char *str;
    struct nbj **items;
    char **keys;
    size_t count;
} nbj_t;
nbj_t *nbj_parse(const char *text, size_t len, char *err, size_t errlen);
void nbj_free(nbj_t *v);
const nbj_t *nbj_get(const nbj_t *obj, const char *key);
double nbj_num(const nbj_t *v, double dflt);
const char *nbj_str(const nbj_t *v, const char *dflt);
size_t nbj_len(const nbj_t *v);
const nbj_t *nbj_at(const nbj_t *arr, size_t i);

/* ---- tensor source: a checkpoint file or the in-memory synthetic generator ---------------- */
typedef struct nb_source nb_source_t;
nb_source_t *nb_source_open_dir(const char *dir, char *err, size_t errlen);
nb_source_t *nb_source_open_synth(const nemoasr_synth_spec_t *spec, char *err, size_t errlen);
void nb_source_close(nb_source_t *s);
const nbj_t *nb_source_config(const nb_source_t *s);
/* Fetch tensor `name` as bf16 into dst (numel elements). Returns 0, or -1 with err when the
   tensor is missing, has another element count, or is not bf16. */
int nb_source_bf16(nb_source_t *s, const char *name, size_t numel, uint16_t *dst, char *err, size_t errlen);
int nb_parse_config(const nbj_t *root, nb_config_t *g, char *err, size_t errlen);

/* ---- synthetic generator -------------------------------------------------------------- */
/* Deterministic bf16 values of one named tensor of the synthetic model. Returns 0 or -1. */
int nb_synth_tensor(const nemoasr_synth_spec_t *spec, const char *name, size_t numel, uint16_t *dst);
/* config.json text of the synthetic model (malloc'd). */
char *nb_synth_config_json(const nemoasr_synth_spec_t *spec);
/* Names and element counts of every tensor of the synthetic model, in file order. */
typedef struct { char name[96]; size_t numel; int ndim; int64_t shape[4]; } nb_tensor_info_t;
int nb_synth_tensor_list(const nemoasr_synth_spec_t *spec, nb_tensor_info_t **out);

static inline float nb_bf16_to_f32(uint16_t v) {
    union { uint32_t u; float f; } x;
    x.u = (uint32_t)v << 16;
    return x.f;
}
static inline uint16_t nb_f32_to_bf16(float f) {
    union { uint32_t u; float f; } x;
    x.f = f;
    uint32_t u = x.u;
    if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t)((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* ---- host front end ------------------------------------------------------------------- */
typedef struct nb_mel nb_mel_t;
nb_mel_t *nb_mel_create(void);
void nb_mel_destroy(nb_mel_t *m);
void nb_mel_push(nb_mel_t *m, const float *samples, size_t n, int final, const float **frames, size_t *nframes);
size_t nb_mel_stage(nb_mel_t *m, const float *samples, size_t n, int final, float *span, size_t span_cap);
void nb_mel_tables(const nb_mel_t *m, const float **window, const float **fb, const double **wr, const double **wi);
size_t nb_mel_total_samples(const nb_mel_t *m);

typedef struct nb_resampler nb_resampler_t;
nb_resampler_t *nb_resampler_create(int in_rate, int out_rate);
void nb_resampler_destroy(nb_resampler_t *r);
size_t nb_resampler_process(nb_resampler_t *r, const float *in, size_t n, float *out, size_t out_max);
size_t nb_resampler_flush(nb_resampler_t *r, float *out, size_t out_max);
/* The sums of one process (+ flush when final) call, left to the GPU (nemo_resample): the input
   FIFO after appending `in`, and the outputs [out0, out0 + count) it now allows. */
typedef struct {
    const float *win;        /* input samples [start, start + len) */
    long long start;
    size_t len;
    unsigned long long nin;  /* input samples seen (zero beyond) */
    unsigned long long out0;
    size_t count;
    int in_rate, out_rate;
} nb_resample_job_t;
void nb_resampler_plan(nb_resampler_t *r, const float *in, size_t n, int final, nb_resample_job_t *job);
/* The job's outputs are done: advance past them and drop the input no later output reads. */
void nb_resampler_commit(nb_resampler_t *r, size_t count);

double nb_now_ms(void);

#ifdef __cplusplus
}
#endif
#endif
