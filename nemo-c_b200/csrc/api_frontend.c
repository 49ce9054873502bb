/* Public wrappers of the host front end (include/nemoasr.h: nemoasr_mel_*, nemoasr_resampler_*). */
#include "nb.h"
#include <string.h>

nemoasr_mel_t *nemoasr_mel_create(void) { return (nemoasr_mel_t *)nb_mel_create(); }
void nemoasr_mel_destroy(nemoasr_mel_t *m) { nb_mel_destroy((nb_mel_t *)m); }
size_t nemoasr_mel_push(nemoasr_mel_t *m, const float *samples, size_t n, int final, float *out, size_t max_frames) {
    const float *frames;
    size_t nf;
    nb_mel_push((nb_mel_t *)m, samples, n, final, &frames, &nf);
    if (nf > max_frames) nf = max_frames;
    if (nf) memcpy(out, frames, nf * NB_MEL_NMEL * sizeof(float));
    return nf;
}
nemoasr_resampler_t *nemoasr_resampler_create(int in_rate, int out_rate) { return (nemoasr_resampler_t *)nb_resampler_create(in_rate, out_rate); }
size_t nemoasr_resampler_process(nemoasr_resampler_t *r, const float *in, size_t n, float *out, size_t out_max) {
    return nb_resampler_process((nb_resampler_t *)r, in, n, out, out_max);
}
size_t nemoasr_resampler_flush(nemoasr_resampler_t *r, float *out, size_t out_max) { return nb_resampler_flush((nb_resampler_t *)r, out, out_max); }
void nemoasr_resampler_destroy(nemoasr_resampler_t *r) { nb_resampler_destroy((nb_resampler_t *)r); }

/* ---- device-resident batch input (include/nemoasr.h: nemoasr_batch_attach_mel / _step) ----- */
#include "engine.h"
nb_engine_t *nb_batch_engine(nemoasr_batch_t *b);
int nemoasr_batch_attach_mel(nemoasr_batch_t *b, const float *d_mel, int64_t stream_stride, size_t frames, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    return nb_engine_attach_device_mel(nb_batch_engine(b), d_mel, stream_stride, frames, err, errlen);
}
double nemoasr_batch_gpu_ms(const nemoasr_batch_t *b) { return nb_engine_gpu_ms(nb_batch_engine((nemoasr_batch_t *)b)); }
int nemoasr_batch_step(nemoasr_batch_t *b, int final, int *tokens, int max_tokens, int *counts, int *rows, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    return nb_engine_step(nb_batch_engine(b), final, tokens, max_tokens, counts, rows, err, errlen);
}
