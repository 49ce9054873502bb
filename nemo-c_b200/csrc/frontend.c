/* Host audio front end of the streaming API: log-mel features and sample-rate conversion.
   Same definitions as the reference's src/mel.c and src/resample.c:
   - log-mel: preemphasis 0.97, symmetric Hann(400) centred in a 512-point frame, 10 ms hop,
     centred frames with reflect padding (no edge repeat), power spectrum from a double-precision
     radix-2 FFT, 128 Slaney-normalised mel filters, log(x + 2^-24);
   - resampler: Blackman-windowed sinc with 16 zero crossings, cutoff at the lower Nyquist,
     weight-normalised, streaming with zero extension at the stream edges. */
#include "nb.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define LOOKAHEAD (NB_MEL_NFFT / 2)
#define LOG_GUARD 5.960464477539063e-08f

struct nb_mel {
    float *y;
    size_t y_len, y_cap, y_start, total, next_frame;
    float last_x;
    int have_last, closed;
    float window[NB_MEL_NFFT];
    float fb[NB_MEL_NMEL * NB_MEL_NFREQ];
    double wr[NB_MEL_NFFT / 2], wi[NB_MEL_NFFT / 2];
    int rev[NB_MEL_NFFT];
    float *out;
    size_t out_cap;
};

/* Slaney scale: linear below 1 kHz (200/3 Hz per mel), logarithmic above (27 mels per ln 6.4) */
static double slaney_mel(double hz) {
    const double fsp = 200.0 / 3.0, brk = 1000.0, brk_mel = brk / fsp, step = log(6.4) / 27.0;
    return hz < brk ? hz / fsp : brk_mel + log(hz / brk) / step;
}
static double slaney_hz(double mel) {
    const double fsp = 200.0 / 3.0, brk = 1000.0, brk_mel = brk / fsp, step = log(6.4) / 27.0;
    return mel < brk_mel ? fsp * mel : brk * exp(step * (mel - brk_mel));
}

nb_mel_t *nb_mel_create(void) {
    nb_mel_t *m = calloc(1, sizeof *m);
    m->y_cap = NB_MEL_SR * 4;
    m->y = malloc(m->y_cap * sizeof(float));
    const int off = (NB_MEL_NFFT - NB_MEL_WIN) / 2;
    for (int n = 0; n < NB_MEL_WIN; ++n) m->window[off + n] = (float)(0.5 * (1.0 - cos(2.0 * M_PI * n / (NB_MEL_WIN - 1))));
    double hz[NB_MEL_NFREQ], edge[NB_MEL_NMEL + 2];
    for (int k = 0; k < NB_MEL_NFREQ; ++k) hz[k] = (NB_MEL_SR / 2) * (double)k / (NB_MEL_NFREQ - 1);
    const double lo = slaney_mel(0.0), hi = slaney_mel(NB_MEL_SR / 2.0);
    for (int i = 0; i < NB_MEL_NMEL + 2; ++i) edge[i] = slaney_hz(lo + (hi - lo) * (double)i / (NB_MEL_NMEL + 1));
    for (int b = 0; b < NB_MEL_NMEL; ++b) {
        const double norm = 2.0 / (edge[b + 2] - edge[b]);
        for (int k = 0; k < NB_MEL_NFREQ; ++k) {
            const double rise = (hz[k] - edge[b]) / (edge[b + 1] - edge[b]);
            const double fall = (edge[b + 2] - hz[k]) / (edge[b + 2] - edge[b + 1]);
            const double tri = fmax(0.0, fmin(rise, fall));
            m->fb[b * NB_MEL_NFREQ + k] = (float)(tri * norm);
        }
    }
    for (int i = 0; i < NB_MEL_NFFT / 2; ++i) { m->wr[i] = cos(-2.0 * M_PI * i / NB_MEL_NFFT); m->wi[i] = sin(-2.0 * M_PI * i / NB_MEL_NFFT); }
    for (int i = 0; i < NB_MEL_NFFT; ++i) {
        int r = 0;
        for (int b = 0; b < 9; ++b) r |= ((i >> b) & 1) << (8 - b);
        m->rev[i] = r;
    }
    return m;
}
void nb_mel_destroy(nb_mel_t *m) { if (m) { free(m->y); free(m->out); free(m); } }
size_t nb_mel_total_samples(const nb_mel_t *m) { return m->total; }

/* iterative radix-2 Cooley-Tukey, bit-reversed input order, butterflies by stage */
static void fft(const nb_mel_t *m, double *re, double *im) {
    for (int i = 0; i < NB_MEL_NFFT; ++i) {
        const int j = m->rev[i];
        if (j > i) { double t = re[i]; re[i] = re[j]; re[j] = t; t = im[i]; im[i] = im[j]; im[j] = t; }
    }
    for (int span = 2; span <= NB_MEL_NFFT; span <<= 1) {
        const int half = span >> 1, tstep = NB_MEL_NFFT / span;
        for (int base = 0; base < NB_MEL_NFFT; base += span)
            for (int k = 0; k < half; ++k) {
                const double c = m->wr[k * tstep], s = m->wi[k * tstep];
                const int p = base + k, q = p + half;
                const double xr = re[q] * c - im[q] * s, xi = re[q] * s + im[q] * c;
                const double ar = re[p], ai = im[p];
                re[p] = ar + xr; im[p] = ai + xi;
                re[q] = ar - xr; im[q] = ai - xi;
            }
    }
}

static float sample_at(const nb_mel_t *m, long g) {
    const long N = (long)m->total;
    if (g < 0) g = -g;                 /* reflect without repeating the edge sample */
    if (g >= N) g = 2 * N - 2 - g;
    if (g < 0 || g >= N) return 0.0f;
    const long i = g - (long)m->y_start;
    return (i < 0 || i >= (long)m->y_len) ? 0.0f : m->y[i];
}

/* Append n samples (pre-emphasised) and return the range [*t0, *t0 + *count) of frames that are
   now complete: once a frame's right half is present, or every remaining frame on the final call
   (their right halves reflect). */
static void mel_advance(nb_mel_t *m, const float *samples, size_t n, int final, size_t *t0, size_t *count) {
    *t0 = m->next_frame;
    *count = 0;
    if (m->closed) return;
    if (m->y_len + n > m->y_cap) {
        while (m->y_len + n > m->y_cap) m->y_cap *= 2;
        m->y = realloc(m->y, m->y_cap * sizeof(float));
    }
    if (n) {
        /* y[i] = x[i] - 0.97 x[i-1]; the first sample of the stream is kept as it is */
        float *y = m->y + m->y_len;
        y[0] = m->have_last ? samples[0] - 0.97f * m->last_x : samples[0];
        for (size_t i = 1; i < n; ++i) y[i] = samples[i] - 0.97f * samples[i - 1];
        m->last_x = samples[n - 1];
        m->have_last = 1;
        m->y_len += n;
    }
    m->total += n;
    const size_t end = final ? m->total / NB_MEL_HOP + 1 : (m->total >= LOOKAHEAD ? (m->total - LOOKAHEAD) / NB_MEL_HOP + 1 : 0);
    if (final) m->closed = 1;
    if (end > m->next_frame) *count = end - m->next_frame;
}

/* Frames up to `end` are done: drop the samples no later frame reads. */
static void mel_retire(nb_mel_t *m, size_t end) {
    m->next_frame = end;
    const long keep = (long)m->next_frame * NB_MEL_HOP - NB_MEL_NFFT - 2;
    if (keep > (long)m->y_start) {
        size_t drop = (size_t)keep - m->y_start;
        if (drop > m->y_len) drop = m->y_len;
        memmove(m->y, m->y + drop, (m->y_len - drop) * sizeof(float));
        m->y_len -= drop;
        m->y_start += drop;
    }
}

void nb_mel_push(nb_mel_t *m, const float *samples, size_t n, int final, const float **frames, size_t *nframes) {
    *frames = NULL;
    *nframes = 0;
    size_t t0, count;
    mel_advance(m, samples, n, final, &t0, &count);
    if (!count) return;
    if (count * NB_MEL_NMEL > m->out_cap) { m->out_cap = count * NB_MEL_NMEL; m->out = realloc(m->out, m->out_cap * sizeof(float)); }
    double re[NB_MEL_NFFT], im[NB_MEL_NFFT];
    float pw[NB_MEL_NFREQ];
    for (size_t t = t0; t < t0 + count; ++t) {
        const long start = (long)t * NB_MEL_HOP - LOOKAHEAD;
        for (int k = 0; k < NB_MEL_NFFT; ++k) { re[k] = (double)(sample_at(m, start + k) * m->window[k]); im[k] = 0.0; }
        fft(m, re, im);
        for (int k = 0; k < NB_MEL_NFREQ; ++k) pw[k] = (float)(re[k] * re[k] + im[k] * im[k]);
        float *row = m->out + (t - t0) * NB_MEL_NMEL;
        for (int b = 0; b < NB_MEL_NMEL; ++b) {
            const float *f = m->fb + b * NB_MEL_NFREQ;
            float acc = 0.0f;
            for (int k = 0; k < NB_MEL_NFREQ; ++k) acc += f[k] * pw[k];
            row[b] = logf(acc + LOG_GUARD);
        }
    }
    *frames = m->out;
    *nframes = count;
    mel_retire(m, t0 + count);
}

/* Same bookkeeping as nb_mel_push, without the transform: the samples the new frames read
   (pre-emphasised, reflected at the stream edges) go to span: frame t0 + i covers
   span[i * HOP .. i * HOP + NFFT). Returns the frame count, or (size_t)-1 if span_cap is short. */
size_t nb_mel_stage(nb_mel_t *m, const float *samples, size_t n, int final, float *span, size_t span_cap) {
    size_t t0, count;
    mel_advance(m, samples, n, final, &t0, &count);
    if (!count) return 0;
    const size_t len = (count - 1) * NB_MEL_HOP + NB_MEL_NFFT;
    if (len > span_cap) return (size_t)-1;
    /* samples inside the stream and the buffer are copied as a run; only the reflected edges
       (and anything outside the buffer) go through sample_at */
    const long s0 = (long)t0 * NB_MEL_HOP - LOOKAHEAD, s1 = s0 + (long)len;
    const long lo_buf = (long)m->y_start, hi_buf = lo_buf + (long)m->y_len;
    long a = s0 > 0 ? s0 : 0, b = s1 < (long)m->total ? s1 : (long)m->total;
    if (a < lo_buf) a = lo_buf;
    if (b > hi_buf) b = hi_buf;
    if (a < b) {
        for (long g = s0; g < a; ++g) span[g - s0] = sample_at(m, g);
        memcpy(span + (a - s0), m->y + (a - lo_buf), (size_t)(b - a) * sizeof(float));
        for (long g = b; g < s1; ++g) span[g - s0] = sample_at(m, g);
    } else {
        for (long g = s0; g < s1; ++g) span[g - s0] = sample_at(m, g);
    }
    mel_retire(m, t0 + count);
    return count;
}

/* The constant tables of the transform (analysis window, filterbank, FFT twiddles). */
void nb_mel_tables(const nb_mel_t *m, const float **window, const float **fb, const double **wr, const double **wi) {
    *window = m->window;
    *fb = m->fb;
    *wr = m->wr;
    *wi = m->wi;
}

/* ---- resampler --------------------------------------------------------------------------- */
struct nb_resampler {
    double ratio, half, fc2;
    float *buf;
    size_t len, cap;
    unsigned long long start, nin, nout;
    int same, in_rate, out_rate;
};

nb_resampler_t *nb_resampler_create(int in_rate, int out_rate) {
    nb_resampler_t *r = calloc(1, sizeof *r);
    r->same = in_rate == out_rate;
    r->in_rate = in_rate;
    r->out_rate = out_rate;
    r->ratio = (double)in_rate / (double)out_rate;
    r->half = 16.0 * fmax(r->ratio, 1.0);
    r->fc2 = fmin(1.0, 1.0 / r->ratio);
    r->cap = 8192;
    r->buf = malloc(r->cap * sizeof(float));
    return r;
}
void nb_resampler_destroy(nb_resampler_t *r) { if (r) { free(r->buf); free(r); } }

static double taper(const nb_resampler_t *r, double u) {
    const double x = u / r->half;
    if (x <= -1.0 || x >= 1.0) return 0.0;
    const double blackman = 0.42 + 0.5 * cos(M_PI * x) + 0.08 * cos(2.0 * M_PI * x);
    const double a = M_PI * r->fc2 * u;
    return r->fc2 * (fabs(a) < 1e-9 ? 1.0 : sin(a) / a) * blackman;
}

/* output nout may be produced now: its last tap has arrived, or (final) its first tap is input */
static int ready(const nb_resampler_t *r, unsigned long long nout, int final, long *a, long *b) {
    const double t = (double)nout * r->ratio;
    *a = (long)ceil(t - r->half);
    *b = (long)floor(t + r->half);
    return final ? (unsigned long long)*a < r->nin : (unsigned long long)(*b + 1) <= r->nin;
}

/* drop input no longer reachable by any future output */
static void retire(nb_resampler_t *r) {
    const long keep = (long)floor((double)r->nout * r->ratio - r->half) - 2;
    if (keep > (long)r->start) {
        size_t drop = (size_t)keep - (size_t)r->start;
        if (drop > r->len) drop = r->len;
        memmove(r->buf, r->buf + drop, (r->len - drop) * sizeof(float));
        r->len -= drop;
        r->start += drop;
    }
}

static void append(nb_resampler_t *r, const float *in, size_t n) {
    if (r->len + n > r->cap) {
        while (r->len + n > r->cap) r->cap *= 2;
        r->buf = realloc(r->buf, r->cap * sizeof(float));
    }
    memcpy(r->buf + r->len, in, n * sizeof(float));
    r->len += n;
    r->nin += n;
}

static size_t produce(nb_resampler_t *r, float *out, size_t out_max, int final) {
    size_t k = 0;
    long a, b;
    while (k < out_max && ready(r, r->nout, final, &a, &b)) {
        const double t = (double)r->nout * r->ratio;
        double acc = 0.0, wsum = 0.0;
        for (long i = a; i <= b; ++i) {
            const double h = taper(r, (double)i - t);
            wsum += h;
            if (i < 0 || (unsigned long long)i >= r->nin) continue;
            const long j = i - (long)r->start;
            if (j < 0 || (size_t)j >= r->len) continue;
            acc += h * r->buf[j];
        }
        out[k++] = (float)(wsum > 0 ? acc / wsum : 0.0);
        r->nout++;
    }
    retire(r);
    return k;
}

size_t nb_resampler_process(nb_resampler_t *r, const float *in, size_t n, float *out, size_t out_max) {
    if (r->same) { const size_t k = n < out_max ? n : out_max; memcpy(out, in, k * sizeof(float)); return k; }
    append(r, in, n);
    return produce(r, out, out_max, 0);
}
size_t nb_resampler_flush(nb_resampler_t *r, float *out, size_t out_max) { return r->same ? 0 : produce(r, out, out_max, 1); }

/* How many outputs from j on are ready (the same count as testing ready() one output at a
   time). From a ready output on, the ready outputs form one run: the first and last taps only
   grow with the output index. The run's end is estimated from the tap formula and then settled
   with ready() itself, a step or two either way. */
static size_t ready_run(const nb_resampler_t *r, unsigned long long j, int final) {
    long a, b;
    if (!ready(r, j, final, &a, &b)) return 0;
    /* last ready output: final, ceil(k ratio - half) <= nin - 1; else floor(k ratio + half) <= nin - 1 */
    const double est = ((double)r->nin - 1.0 + (final ? r->half : -r->half)) / r->ratio;
    unsigned long long k = est > (double)j ? (unsigned long long)est : j;
    while (k > j && !ready(r, k, final, &a, &b)) --k;
    while (ready(r, k + 1, final, &a, &b)) ++k;
    return (size_t)(k - j + 1);
}

/* process (when n > 0) followed by flush (when final) of a resampler whose rates differ, with
   the sums left to the caller: both calls' outputs form one run from nout on. */
void nb_resampler_plan(nb_resampler_t *r, const float *in, size_t n, int final, nb_resample_job_t *job) {
    size_t count = 0;
    if (n) {
        append(r, in, n);
        count = ready_run(r, r->nout, 0);
    }
    if (final) count += ready_run(r, r->nout + count, 1);
    job->win = r->buf;
    job->start = (long long)r->start;
    job->len = r->len;
    job->nin = r->nin;
    job->out0 = r->nout;
    job->count = count;
    job->in_rate = r->in_rate;
    job->out_rate = r->out_rate;
}

void nb_resampler_commit(nb_resampler_t *r, size_t count) {
    r->nout += count;
    retire(r);
}
