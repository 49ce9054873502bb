/* ORACLE — TEST INFRASTRUCTURE ONLY (see oracle.h). CPU restatement of the reference's streaming
   host code: model tables (src/model.c), the cache-aware encoder step (src/encoder.c), greedy RNNT
   decoding (src/decoder.c), the session glue (src/nemoasr.c), the log-mel front end (src/mel.c)
   and the windowed-sinc resampler (src/resample.c). Device buffers of the reference are plain
   heap arrays here; every kernel call goes to oracle_kernels.c. */
#define _GNU_SOURCE
#include "oracle.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MEL_SR 16000
#define MEL_NFFT 512
#define MEL_WIN 400
#define MEL_HOP 160
#define MEL_NMEL 128
#define MEL_NFREQ (MEL_NFFT / 2 + 1)
#define MEL_CACHE 16           /* src/encoder.c:10 */
#define CACHE_EPOCH_CHUNKS 8   /* src/kernel_params.h:16 */
#define MMA_MIN_ROWS 16        /* src/kernel_params.h:15 */
#define DEC_MAX_BATCH 16       /* src/kernel_params.h:17 */

static float bf2f(uint16_t v) {
    union { uint32_t u; float f; } x;
    x.u = (uint32_t)v << 16;
    return x.f;
}

/* ================================ model (src/model.c) ================================= */
typedef struct {
    const uint16_t *ff1_w1, *ff1_w2, *ff2_w1, *ff2_w2, *wo, *wpos, *pw1, *pw2;
    uint16_t *wqkv; /* q, k, v rows back to back (model.c:241-242) */
    float *ln_ff1_g, *ln_ff1_b, *ln_att_g, *ln_att_b, *ln_conv_g, *ln_conv_b, *ln_ff2_g, *ln_ff2_b, *ln_out_g, *ln_out_b;
    float *bn_g, *bn_b, *dw_w, *bias_u, *bias_v, *ptab;
} or_layer_t;

struct or_model {
    or_config_t c;
    int D, H, dh, FF, CH, F3, Lmax, blank, NC;
    float eps;
    int n;
    uint16_t **data; /* owned copies */
    char **names;
    size_t *numel;
    float *conv0_w, *conv0_b, *conv2_w, *conv2_b, *conv5_w, *conv5_b, *conv3_b, *conv6_b, *pre_out_b;
    const uint16_t *conv3_w, *conv6_w, *pre_out_w;
    or_layer_t *L;
    const uint16_t *prompt_w0, *prompt_w2, *prompt_b0;
    float *prompt_b2, *prompt_b0_eff;
    const uint16_t *lstm_wx[2], *lstm_wh[2];
    float *lstm_b[2];
    const uint16_t *embed;
    const uint16_t *joint_enc_w, *joint_pred_w, *joint_out_w;
    float *joint_enc_b, *joint_pred_b, *joint_out_b;
};

static const uint16_t *find(or_model_t *m, const char *name, size_t numel, char *err, size_t errlen) {
    for (int i = 0; i < m->n; ++i) {
        if (strcmp(m->names[i], name)) continue;
        if (numel && m->numel[i] != numel) { snprintf(err, errlen, "tensor %s has %zu elements, expected %zu", name, m->numel[i], numel); return NULL; }
        return m->data[i];
    }
    snprintf(err, errlen, "missing tensor %s", name);
    return NULL;
}
static float *widen(const uint16_t *src, size_t n) {
    float *d = malloc(n * sizeof(float));
    for (size_t i = 0; i < n; ++i) d[i] = bf2f(src[i]);
    return d;
}

or_model_t *or_model_create(const or_config_t *cfg, int n, const char *const *names, const uint16_t *const *data,
                            const size_t *numel, char *err, size_t errlen) {
    or_model_t *m = calloc(1, sizeof *m);
    m->c = *cfg;
    m->D = cfg->d_model; m->H = cfg->n_heads; m->dh = m->D / m->H; m->FF = cfg->d_ff; m->CH = cfg->sub_channels;
    int f = cfg->feat_in;
    for (int i = 0; i < 3; ++i) f = f / 2 + 1;          /* model.c:226-228 */
    m->F3 = f;
    m->Lmax = cfg->att_left + cfg->max_right + 1 + 2;   /* model.c:168 */
    m->blank = cfg->vocab_size;
    m->NC = cfg->vocab_size + 1;
    m->eps = 1e-5f;                                       /* model.c:149 */
    m->n = n;
    m->data = calloc((size_t)n, sizeof *m->data);
    m->names = calloc((size_t)n, sizeof *m->names);
    m->numel = calloc((size_t)n, sizeof *m->numel);
    for (int i = 0; i < n; ++i) {
        m->names[i] = strdup(names[i]);
        m->numel[i] = numel[i];
        m->data[i] = malloc(numel[i] * 2);
        memcpy(m->data[i], data[i], numel[i] * 2);
    }
    const size_t D = (size_t)m->D, CH = (size_t)m->CH, PH = (size_t)cfg->pred_hidden, JH = (size_t)cfg->joint_hidden;
    const uint16_t *t;
#define BF(name, cnt, dst) do { if (!(t = find(m, name, cnt, err, errlen))) goto fail; dst = t; } while (0)
#define F32(name, cnt, dst) do { if (!(t = find(m, name, cnt, err, errlen))) goto fail; dst = widen(t, cnt); } while (0)
    F32("encoder.pre_encode.conv.0.weight", CH * 9, m->conv0_w);
    F32("encoder.pre_encode.conv.0.bias", CH, m->conv0_b);
    F32("encoder.pre_encode.conv.2.weight", CH * 9, m->conv2_w);
    F32("encoder.pre_encode.conv.2.bias", CH, m->conv2_b);
    BF("encoder.pre_encode.conv.3.weight", CH * CH, m->conv3_w);
    F32("encoder.pre_encode.conv.3.bias", CH, m->conv3_b);
    F32("encoder.pre_encode.conv.5.weight", CH * 9, m->conv5_w);
    F32("encoder.pre_encode.conv.5.bias", CH, m->conv5_b);
    BF("encoder.pre_encode.conv.6.weight", CH * CH, m->conv6_w);
    F32("encoder.pre_encode.conv.6.bias", CH, m->conv6_b);
    BF("encoder.pre_encode.out.weight", D * CH * (size_t)m->F3, m->pre_out_w);
    F32("encoder.pre_encode.out.bias", D, m->pre_out_b);
    m->L = calloc((size_t)cfg->n_layers, sizeof *m->L);
    char nm[160];
    for (int l = 0; l < cfg->n_layers; ++l) {
        or_layer_t *L = &m->L[l];
#define LB(field, suffix, cnt) do { snprintf(nm, sizeof nm, "encoder.layers.%d.%s", l, suffix); BF(nm, cnt, L->field); } while (0)
#define LF(field, suffix, cnt) do { snprintf(nm, sizeof nm, "encoder.layers.%d.%s", l, suffix); F32(nm, cnt, L->field); } while (0)
        LB(ff1_w1, "feed_forward1.linear1.weight", (size_t)m->FF * D);
        LB(ff1_w2, "feed_forward1.linear2.weight", (size_t)m->FF * D);
        LB(ff2_w1, "feed_forward2.linear1.weight", (size_t)m->FF * D);
        LB(ff2_w2, "feed_forward2.linear2.weight", (size_t)m->FF * D);
        const uint16_t *wq, *wk, *wv;
        LB(wo, "self_attn.linear_out.weight", D * D);
        LB(wpos, "self_attn.linear_pos.weight", D * D);
        snprintf(nm, sizeof nm, "encoder.layers.%d.self_attn.linear_q.weight", l); BF(nm, D * D, wq);
        snprintf(nm, sizeof nm, "encoder.layers.%d.self_attn.linear_k.weight", l); BF(nm, D * D, wk);
        snprintf(nm, sizeof nm, "encoder.layers.%d.self_attn.linear_v.weight", l); BF(nm, D * D, wv);
        L->wqkv = malloc(3 * D * D * 2);
        memcpy(L->wqkv, wq, D * D * 2);
        memcpy(L->wqkv + D * D, wk, D * D * 2);
        memcpy(L->wqkv + 2 * D * D, wv, D * D * 2);
        LB(pw1, "conv.pointwise_conv1.weight", 2 * D * D);
        LB(pw2, "conv.pointwise_conv2.weight", D * D);
        LF(ln_ff1_g, "norm_feed_forward1.weight", D); LF(ln_ff1_b, "norm_feed_forward1.bias", D);
        LF(ln_att_g, "norm_self_att.weight", D); LF(ln_att_b, "norm_self_att.bias", D);
        LF(ln_conv_g, "norm_conv.weight", D); LF(ln_conv_b, "norm_conv.bias", D);
        LF(ln_ff2_g, "norm_feed_forward2.weight", D); LF(ln_ff2_b, "norm_feed_forward2.bias", D);
        LF(ln_out_g, "norm_out.weight", D); LF(ln_out_b, "norm_out.bias", D);
        LF(bn_g, "conv.batch_norm.weight", D); LF(bn_b, "conv.batch_norm.bias", D);
        LF(dw_w, "conv.depthwise_conv.weight", D * 9);
        LF(bias_u, "self_attn.pos_bias_u", D); LF(bias_v, "self_attn.pos_bias_v", D);
#undef LB
#undef LF
    }
    const size_t PRH = (size_t)cfg->prompt_hidden, NP = (size_t)cfg->num_prompts;
    BF("prompt_kernel.0.weight", PRH * (D + NP), m->prompt_w0);
    BF("prompt_kernel.0.bias", PRH, m->prompt_b0);
    BF("prompt_kernel.2.weight", D * PRH, m->prompt_w2);
    F32("prompt_kernel.2.bias", D, m->prompt_b2);
    m->prompt_b0_eff = calloc(PRH, sizeof(float));
    for (int l = 0; l < 2; ++l) {
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.Wx", l); BF(nm, 4 * PH * PH, m->lstm_wx[l]);
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.Wh", l); BF(nm, 4 * PH * PH, m->lstm_wh[l]);
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.bias", l); F32(nm, 4 * PH, m->lstm_b[l]);
    }
    BF("decoder.prediction.embed.weight", (size_t)(cfg->vocab_size + 1) * PH, m->embed);
    BF("joint.enc.weight", JH * D, m->joint_enc_w); F32("joint.enc.bias", JH, m->joint_enc_b);
    BF("joint.pred.weight", JH * PH, m->joint_pred_w); F32("joint.pred.bias", JH, m->joint_pred_b);
    BF("joint.joint_net.2.weight", (size_t)m->NC * JH, m->joint_out_w);
    F32("joint.joint_net.2.bias", (size_t)m->NC, m->joint_out_b);
#undef BF
#undef F32
    /* rel-pos table (model.c:286-306): pe row r <-> position Lmax-1-r, sin/cos in double,
       then ptab = pe . Wpos^T per layer (no bias). */
    {
        const int P = 2 * m->Lmax - 1;
        float *pe = malloc((size_t)P * D * sizeof(float));
        for (int r = 0; r < P; ++r) {
            const double pos = (double)(m->Lmax - 1 - r);
            for (size_t i = 0; i < D / 2; ++i) {
                const double div = exp((double)(2 * i) * -(log(10000.0) / (double)D));
                pe[(size_t)r * D + 2 * i] = (float)sin(pos * div);
                pe[(size_t)r * D + 2 * i + 1] = (float)cos(pos * div);
            }
        }
        for (int l = 0; l < cfg->n_layers; ++l) {
            m->L[l].ptab = malloc((size_t)P * D * sizeof(float));
            or_gemm(pe, (int)D, m->L[l].wpos, (int)D, NULL, m->L[l].ptab, (int)D, P, (int)D, (int)D, 0, 0, 1.0f);
        }
        free(pe);
    }
    or_model_set_language(m, 0);
    return m;
fail:
    or_model_free(m);
    return NULL;
}

/* model.c:312-322: b_eff[n] = b0[n] + W0[n][D + idx] */
int or_model_set_language(or_model_t *m, int idx) {
    if (idx < 0 || idx >= m->c.num_prompts) return -1;
    const size_t ld = (size_t)m->D + (size_t)m->c.num_prompts;
    for (int n = 0; n < m->c.prompt_hidden; ++n)
        m->prompt_b0_eff[n] = bf2f(m->prompt_b0[n]) + bf2f(m->prompt_w0[(size_t)n * ld + (size_t)m->D + (size_t)idx]);
    return 0;
}
const float *or_model_ptab(const or_model_t *m, int layer) { return m->L[layer].ptab; }
const float *or_model_prompt_bias(const or_model_t *m) { return m->prompt_b0_eff; }

void or_model_free(or_model_t *m) {
    if (!m) return;
    if (m->L) {
        for (int l = 0; l < m->c.n_layers; ++l) {
            or_layer_t *L = &m->L[l];
            float *fs[] = { L->ln_ff1_g, L->ln_ff1_b, L->ln_att_g, L->ln_att_b, L->ln_conv_g, L->ln_conv_b, L->ln_ff2_g, L->ln_ff2_b,
                            L->ln_out_g, L->ln_out_b, L->bn_g, L->bn_b, L->dw_w, L->bias_u, L->bias_v, L->ptab };
            for (size_t i = 0; i < sizeof fs / sizeof *fs; ++i) free(fs[i]);
            free(L->wqkv);
        }
        free(m->L);
    }
    float *fs[] = { m->conv0_w, m->conv0_b, m->conv2_w, m->conv2_b, m->conv5_w, m->conv5_b, m->conv3_b, m->conv6_b, m->pre_out_b,
                    m->prompt_b2, m->prompt_b0_eff, m->lstm_b[0], m->lstm_b[1], m->joint_enc_b, m->joint_pred_b, m->joint_out_b };
    for (size_t i = 0; i < sizeof fs / sizeof *fs; ++i) free(fs[i]);
    for (int i = 0; i < m->n; ++i) { free(m->data[i]); free(m->names[i]); }
    free(m->data); free(m->names); free(m->numel);
    free(m);
}

/* ================================ mel (src/mel.c) ===================================== */
#define LOG_GUARD 5.960464477539063e-08f
#define LOOKAHEAD (MEL_NFFT / 2)
struct or_mel {
    float *y;
    size_t y_len, y_cap, y_start;
    float last_x;
    int have_last;
    size_t total, next_frame;
    int closed;
    float window[MEL_NFFT];
    float fb[MEL_NMEL * MEL_NFREQ];
    double cos_t[MEL_NFFT / 2], sin_t[MEL_NFFT / 2];
    int bitrev[MEL_NFFT];
};
/* Slaney mel scale (mel.c:25-35) */
static double hz_to_mel(double f) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp, logstep = log(6.4) / 27.0;
    return f >= min_log_hz ? min_log_mel + log(f / min_log_hz) / logstep : f / f_sp;
}
static double mel_to_hz(double m) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp, logstep = log(6.4) / 27.0;
    return m >= min_log_mel ? min_log_hz * exp(logstep * (m - min_log_mel)) : f_sp * m;
}
or_mel_t *or_mel_create(void) {
    or_mel_t *m = calloc(1, sizeof *m);
    m->y_cap = MEL_SR * 4;
    m->y = malloc(m->y_cap * sizeof(float));
    const int left = (MEL_NFFT - MEL_WIN) / 2; /* symmetric Hann(400) centred in 512 (mel.c:61-63) */
    for (int n = 0; n < MEL_WIN; ++n) m->window[left + n] = (float)(0.5 * (1.0 - cos(2.0 * M_PI * n / (MEL_WIN - 1))));
    /* Slaney-normalised triangular filters (mel.c:37-55) */
    double freqs[MEL_NFREQ], fpts[MEL_NMEL + 2];
    for (int i = 0; i < MEL_NFREQ; ++i) freqs[i] = (MEL_SR / 2) * (double)i / (MEL_NFREQ - 1);
    const double mlo = hz_to_mel(0.0), mhi = hz_to_mel(MEL_SR / 2.0);
    for (int i = 0; i < MEL_NMEL + 2; ++i) fpts[i] = mel_to_hz(mlo + (mhi - mlo) * (double)i / (MEL_NMEL + 1));
    for (int b = 0; b < MEL_NMEL; ++b) {
        const double enorm = 2.0 / (fpts[b + 2] - fpts[b]);
        for (int k = 0; k < MEL_NFREQ; ++k) {
            const double down = (freqs[k] - fpts[b]) / (fpts[b + 1] - fpts[b]);
            const double up = (fpts[b + 2] - freqs[k]) / (fpts[b + 2] - fpts[b + 1]);
            double v = fmin(down, up);
            if (v < 0) v = 0;
            m->fb[b * MEL_NFREQ + k] = (float)(v * enorm);
        }
    }
    for (int i = 0; i < MEL_NFFT / 2; ++i) { m->cos_t[i] = cos(-2.0 * M_PI * i / MEL_NFFT); m->sin_t[i] = sin(-2.0 * M_PI * i / MEL_NFFT); }
    for (int i = 0; i < MEL_NFFT; ++i) {
        int r = 0;
        for (int b = 0; b < 9; ++b) if (i & (1 << b)) r |= 1 << (8 - b);
        m->bitrev[i] = r;
    }
    return m;
}
void or_mel_destroy(or_mel_t *m) { if (m) { free(m->y); free(m); } }
/* radix-2 decimation-in-time FFT in double (mel.c:84-102) */
static void fft512(const or_mel_t *m, double *re, double *im) {
    for (int i = 0; i < MEL_NFFT; ++i) {
        const int j = m->bitrev[i];
        if (j > i) { double t = re[i]; re[i] = re[j]; re[j] = t; t = im[i]; im[i] = im[j]; im[j] = t; }
    }
    for (int len = 2; len <= MEL_NFFT; len <<= 1) {
        const int half = len >> 1, step = MEL_NFFT / len;
        for (int i = 0; i < MEL_NFFT; i += len)
            for (int k = 0; k < half; ++k) {
                const double wr = m->cos_t[k * step], wi = m->sin_t[k * step];
                const double ur = re[i + k], ui = im[i + k];
                const double vr = re[i + k + half] * wr - im[i + k + half] * wi;
                const double vi = re[i + k + half] * wi + im[i + k + half] * wr;
                re[i + k] = ur + vr; im[i + k] = ui + vi;
                re[i + k + half] = ur - vr; im[i + k + half] = ui - vi;
            }
    }
}
/* reflect padding without edge repeat (mel.c:104-113) */
static float sample_at(const or_mel_t *m, long g) {
    const long N = (long)m->total;
    if (g < 0) g = -g;
    if (g >= N) g = 2 * N - 2 - g;
    if (g < 0 || g >= N) return 0.0f;
    const long i = g - (long)m->y_start;
    if (i < 0 || i >= (long)m->y_len) return 0.0f;
    return m->y[i];
}
/* mel.c:115-173 */
size_t or_mel_push(or_mel_t *m, const float *samples, size_t n, int final, float *out, size_t max_frames) {
    if (m->closed) return 0;
    if (m->y_len + n > m->y_cap) {
        while (m->y_len + n > m->y_cap) m->y_cap *= 2;
        m->y = realloc(m->y, m->y_cap * sizeof(float));
    }
    for (size_t i = 0; i < n; ++i) {
        const float x = samples[i];
        m->y[m->y_len++] = m->have_last ? x - 0.97f * m->last_x : x;
        m->last_x = x;
        m->have_last = 1;
    }
    m->total += n;
    size_t frame_end = final ? m->total / MEL_HOP + 1 : (m->total >= LOOKAHEAD ? (m->total - LOOKAHEAD) / MEL_HOP + 1 : 0);
    if (final) m->closed = 1;
    if (frame_end <= m->next_frame) return 0;
    size_t count = frame_end - m->next_frame;
    if (count > max_frames) { count = max_frames; frame_end = m->next_frame + count; }
    double re[MEL_NFFT], im[MEL_NFFT];
    float power[MEL_NFREQ];
    for (size_t t = m->next_frame; t < frame_end; ++t) {
        const long start = (long)t * MEL_HOP - LOOKAHEAD;
        for (int k = 0; k < MEL_NFFT; ++k) { re[k] = (double)(sample_at(m, start + k) * m->window[k]); im[k] = 0.0; }
        fft512(m, re, im);
        for (int k = 0; k < MEL_NFREQ; ++k) power[k] = (float)(re[k] * re[k] + im[k] * im[k]);
        float *row = out + (t - m->next_frame) * MEL_NMEL;
        for (int b = 0; b < MEL_NMEL; ++b) {
            const float *w = m->fb + b * MEL_NFREQ;
            float acc = 0.0f;
            for (int k = 0; k < MEL_NFREQ; ++k) acc += w[k] * power[k];
            row[b] = logf(acc + LOG_GUARD);
        }
    }
    m->next_frame = frame_end;
    const long keep_from = (long)m->next_frame * MEL_HOP - MEL_NFFT - 2;
    if (keep_from > (long)m->y_start) {
        size_t drop = (size_t)keep_from - m->y_start;
        if (drop > m->y_len) drop = m->y_len;
        memmove(m->y, m->y + drop, (m->y_len - drop) * sizeof(float));
        m->y_len -= drop;
        m->y_start += drop;
    }
    return count;
}

/* ============================ resampler (src/resample.c) ============================== */
struct or_resampler {
    double ratio, half, cutoff2;
    float *buf;
    size_t len, cap;
    unsigned long long start, in_count, out_count;
    int passthrough;
};
or_resampler_t *or_resampler_create(int in_rate, int out_rate) {
    or_resampler_t *r = calloc(1, sizeof *r);
    r->passthrough = in_rate == out_rate;
    r->ratio = (double)in_rate / (double)out_rate;
    r->half = 16 * fmax(r->ratio, 1.0);       /* 16 zero crossings (resample.c:6, :21) */
    r->cutoff2 = fmin(1.0, 1.0 / r->ratio);
    r->cap = 8192;
    r->buf = malloc(r->cap * sizeof(float));
    return r;
}
void or_resampler_destroy(or_resampler_t *r) { if (r) { free(r->buf); free(r); } }
/* 2fc * sinc(2fc u) * Blackman(u / half) (resample.c:34-42) */
static double rs_kernel(const or_resampler_t *r, double u) {
    const double x = u / r->half;
    if (x <= -1.0 || x >= 1.0) return 0.0;
    const double w = 0.42 + 0.5 * cos(M_PI * x) + 0.08 * cos(2.0 * M_PI * x);
    const double a = M_PI * r->cutoff2 * u;
    const double s = fabs(a) < 1e-9 ? 1.0 : sin(a) / a;
    return r->cutoff2 * s * w;
}
/* resample.c:52-82: weight-normalised sum over the kernel support, zero outside the stream */
static size_t rs_produce(or_resampler_t *r, float *out, size_t out_max, int final) {
    size_t produced = 0;
    while (produced < out_max) {
        const double t = (double)r->out_count * r->ratio;
        const long k0 = (long)ceil(t - r->half), k1 = (long)floor(t + r->half);
        if (!final && (unsigned long long)(k1 + 1) > r->in_count) break;
        if (final && (unsigned long long)k0 >= r->in_count) break;
        double acc = 0.0, wsum = 0.0;
        for (long k = k0; k <= k1; ++k) {
            const double h = rs_kernel(r, (double)k - t);
            wsum += h;
            if (k < 0 || (unsigned long long)k >= r->in_count) continue;
            const long i = k - (long)r->start;
            if (i < 0 || (size_t)i >= r->len) continue;
            acc += h * r->buf[i];
        }
        out[produced++] = (float)(wsum > 0 ? acc / wsum : 0.0);
        r->out_count++;
    }
    const double tn = (double)r->out_count * r->ratio;
    const long keep_from = (long)floor(tn - r->half) - 2;
    if (keep_from > (long)r->start) {
        size_t drop = (size_t)keep_from - (size_t)r->start;
        if (drop > r->len) drop = r->len;
        memmove(r->buf, r->buf + drop, (r->len - drop) * sizeof(float));
        r->len -= drop;
        r->start += drop;
    }
    return produced;
}
size_t or_resampler_process(or_resampler_t *r, const float *in, size_t n, float *out, size_t out_max) {
    if (r->passthrough) { const size_t k = n < out_max ? n : out_max; memcpy(out, in, k * sizeof(float)); return k; }
    if (r->len + n > r->cap) {
        while (r->len + n > r->cap) r->cap *= 2;
        r->buf = realloc(r->buf, r->cap * sizeof(float));
    }
    memcpy(r->buf + r->len, in, n * sizeof(float));
    r->len += n;
    r->in_count += n;
    return rs_produce(r, out, out_max, 0);
}
size_t or_resampler_flush(or_resampler_t *r, float *out, size_t out_max) { return r->passthrough ? 0 : rs_produce(r, out, out_max, 1); }

/* ================================ encoder (src/encoder.c) ============================= */
typedef struct {
    or_model_t *m;
    int right, chunk_frames, chunk_mel, cmax, Lmax, left, conv_left;
    float *pending;
    size_t pending_n, pending_cap;
    float mel_cache[MEL_CACHE * MEL_NMEL];
    int mel_cache_n;
    size_t consumed, emitted;
    int closed;
    float *win, *c0, *c1, *c2, *c3, *c4, *flat, *pre_out;
    float *h, *tmp, *t2, *ff, *att, *y, *ph, *prompted, *joint_enc;
    float **kv, **din;
    int cap_rows, pos, cache_len;
} or_encoder_t;

static int sub_len(int n) { return n / 2 + 1; }

/* encoder.c:39-82 */
static or_encoder_t *enc_create(or_model_t *m, int right) {
    or_encoder_t *e = calloc(1, sizeof *e);
    e->m = m;
    e->right = right;
    e->chunk_frames = right + 1;
    e->chunk_mel = e->chunk_frames * 8;
    e->cmax = e->chunk_frames + 2;
    if (e->cmax < MMA_MIN_ROWS) e->cmax = MMA_MIN_ROWS;
    e->left = m->c.att_left;
    e->Lmax = m->Lmax;
    e->conv_left = 8;
    const size_t D = (size_t)m->D, CH = (size_t)m->CH, F = 128;
    const size_t nwin = MEL_CACHE + (size_t)e->chunk_mel + 1;
    const size_t T1 = nwin / 2 + 1, F1 = F / 2 + 1, T2 = T1 / 2 + 1, F2 = F1 / 2 + 1, T3 = T2 / 2 + 1, F3 = F2 / 2 + 1;
    e->win = calloc(nwin * F, sizeof(float));
    e->c0 = calloc(T1 * F1 * CH, sizeof(float));
    e->c1 = calloc(T2 * F2 * CH, sizeof(float));
    e->c2 = calloc(T2 * F2 * CH, sizeof(float));
    e->c3 = calloc(T3 * F3 * CH, sizeof(float));
    e->c4 = calloc(T3 * F3 * CH, sizeof(float));
    e->flat = calloc(T3 * F3 * CH, sizeof(float));
    e->pre_out = calloc(T3 * D, sizeof(float));
    const size_t cm = (size_t)e->cmax;
    e->h = calloc(cm * D, sizeof(float));
    e->tmp = calloc(cm * D, sizeof(float));
    e->ff = calloc(cm * (size_t)m->FF, sizeof(float));
    e->att = calloc(cm * D, sizeof(float));
    e->t2 = calloc(cm * D, sizeof(float));
    e->y = calloc(cm * D, sizeof(float));
    e->ph = calloc(cm * (size_t)m->c.prompt_hidden, sizeof(float));
    e->prompted = calloc(cm * D, sizeof(float));
    e->joint_enc = calloc(cm * (size_t)m->c.joint_hidden, sizeof(float));
    e->cap_rows = e->left + CACHE_EPOCH_CHUNKS * e->cmax;
    e->pos = e->conv_left;
    e->kv = calloc((size_t)m->c.n_layers, sizeof *e->kv);
    e->din = calloc((size_t)m->c.n_layers, sizeof *e->din);
    for (int l = 0; l < m->c.n_layers; ++l) {
        e->kv[l] = calloc((size_t)e->cap_rows * 3 * D, sizeof(float));
        e->din[l] = calloc((size_t)e->cap_rows * D, sizeof(float));
    }
    return e;
}
static void enc_destroy(or_encoder_t *e) {
    if (!e) return;
    float *b[] = { e->win, e->c0, e->c1, e->c2, e->c3, e->c4, e->flat, e->pre_out, e->h, e->tmp, e->t2, e->ff, e->att, e->y, e->ph, e->prompted, e->joint_enc };
    for (size_t i = 0; i < sizeof b / sizeof *b; ++i) free(b[i]);
    for (int l = 0; l < e->m->c.n_layers; ++l) { free(e->kv[l]); free(e->din[l]); }
    free(e->kv); free(e->din); free(e->pending);
    free(e);
}
static void enc_push(or_encoder_t *e, const float *mel, size_t nframes) {
    if (!nframes) return;
    if (e->pending_n + nframes > e->pending_cap) {
        e->pending_cap = (e->pending_n + nframes) * 2;
        e->pending = realloc(e->pending, e->pending_cap * MEL_NMEL * sizeof(float));
    }
    memcpy(e->pending + e->pending_n * MEL_NMEL, mel, nframes * MEL_NMEL * sizeof(float));
    e->pending_n += nframes;
}
/* encoder.c:121-142 */
static void run_pre_encode(or_encoder_t *e, int nwin) {
    or_model_t *m = e->m;
    const int CH = m->CH, F = 128;
    const int T1 = sub_len(nwin), F1 = F / 2 + 1, T2 = T1 / 2 + 1, F2 = F1 / 2 + 1, T3 = T2 / 2 + 1, F3 = F2 / 2 + 1;
    or_conv2d_c1_s2_relu(e->win, m->conv0_w, m->conv0_b, e->c0, nwin, F, T1, F1, CH);
    or_dwconv2d_s2(e->c0, m->conv2_w, m->conv2_b, e->c1, T1, F1, T2, F2, CH);
    or_gemm(e->c1, CH, m->conv3_w, CH, m->conv3_b, e->c2, CH, T2 * F2, CH, CH, 2, 0, 1.0f);
    or_dwconv2d_s2(e->c2, m->conv5_w, m->conv5_b, e->c3, T2, F2, T3, F3, CH);
    or_gemm(e->c3, CH, m->conv6_w, CH, m->conv6_b, e->c4, CH, T3 * F3, CH, CH, 2, 0, 1.0f);
    or_flatten_cf(e->c4, e->flat, T3, F3, CH);
    or_gemm(e->flat, CH * F3, m->pre_out_w, CH * F3, m->pre_out_b, e->pre_out, m->D, T3, m->D, CH * F3, 0, 0, 1.0f);
}
/* encoder.c:145-197: 24 conformer blocks, then prompt and joint encoder projection */
static void run_blocks(or_encoder_t *e, int c) {
    or_model_t *m = e->m;
    const int D = m->D, FF = m->FF, H = m->H, dh = m->dh;
    const int L = e->cache_len + c, pos = e->pos;
    float *h = e->h, *t = e->tmp, *t2 = e->t2;
    for (int l = 0; l < m->c.n_layers; ++l) {
        or_layer_t *W = &m->L[l];
        float *kv = e->kv[l], *din = e->din[l];
        if (l == 0) or_layernorm(h, W->ln_ff1_g, W->ln_ff1_b, t2, c, D, m->eps);
        or_gemm(t2, D, W->ff1_w1, D, NULL, e->ff, FF, c, FF, D, 1, 0, 1.0f);
        or_gemm(e->ff, FF, W->ff1_w2, FF, NULL, h, D, c, D, FF, 0, 1, 0.5f);
        or_layernorm(h, W->ln_att_g, W->ln_att_b, t, c, D, m->eps);
        or_gemm(t, D, W->wqkv, D, NULL, kv + (size_t)pos * 3 * D, 3 * D, c, 3 * D, D, 0, 0, 1.0f);
        const float *kvw = kv + (size_t)(pos - e->cache_len) * 3 * D;
        or_attention_rel(kv + (size_t)pos * 3 * D, 3 * D, kvw + D, kvw + 2 * D, 3 * D, W->ptab, W->bias_u, W->bias_v, e->att,
                         c, L, e->Lmax, H, dh, D, 1.0f / sqrtf((float)dh));
        or_gemm(e->att, D, W->wo, D, NULL, h, D, c, D, D, 0, 1, 1.0f);
        or_layernorm(h, W->ln_conv_g, W->ln_conv_b, t, c, D, m->eps);
        or_gemm(t, D, W->pw1, D, NULL, din + (size_t)pos * D, D, c, 2 * D, D, 3, 0, 1.0f);
        or_dwconv_ln_silu(din + (size_t)(pos - e->conv_left) * D, W->dw_w, W->bn_g, W->bn_b, e->y, c, D, 9, m->eps);
        or_gemm(e->y, D, W->pw2, D, NULL, h, D, c, D, D, 0, 1, 1.0f);
        or_layernorm(h, W->ln_ff2_g, W->ln_ff2_b, t, c, D, m->eps);
        or_gemm(t, D, W->ff2_w1, D, NULL, e->ff, FF, c, FF, D, 1, 0, 1.0f);
        or_gemm(e->ff, FF, W->ff2_w2, FF, NULL, h, D, c, D, FF, 0, 1, 0.5f);
        if (l + 1 < m->c.n_layers) {
            or_layer_t *Wn = &m->L[l + 1];
            or_layernorm2(h, W->ln_out_g, W->ln_out_b, Wn->ln_ff1_g, Wn->ln_ff1_b, t, t2, c, D, m->eps);
        } else {
            or_layernorm(h, W->ln_out_g, W->ln_out_b, t, c, D, m->eps);
        }
        float *sw = h; h = t; t = sw;
    }
    const int PH = m->c.prompt_hidden, JH = m->c.joint_hidden;
    or_gemm(h, D, m->prompt_w0, D + m->c.num_prompts, m->prompt_b0_eff, e->ph, PH, c, PH, D, 2, 0, 1.0f);
    or_gemm(e->ph, PH, m->prompt_w2, PH, m->prompt_b2, e->prompted, D, c, D, PH, 0, 0, 1.0f);
    or_gemm(e->prompted, D, m->joint_enc_w, D, m->joint_enc_b, e->joint_enc, JH, c, JH, D, 0, 0, 1.0f);
    e->pos += c;
    e->cache_len = L < e->left ? L : e->left;
}
/* encoder.c:201-211: move the live history to the front once per epoch */
static void compact_caches(or_encoder_t *e) {
    const size_t D = (size_t)e->m->D;
    const int src_kv = e->pos - e->cache_len, src_din = e->pos - e->conv_left, dst_din = e->cache_len - e->conv_left;
    for (int l = 0; l < e->m->c.n_layers; ++l) {
        if (e->cache_len > 0) memmove(e->kv[l], e->kv[l] + (size_t)src_kv * 3 * D, (size_t)e->cache_len * 3 * D * sizeof(float));
        memmove(e->din[l] + (size_t)dst_din * D, e->din[l] + (size_t)src_din * D, (size_t)e->conv_left * D * sizeof(float));
    }
    e->pos = e->cache_len;
}
/* encoder.c:213-267. Returns 1 if a piece was consumed (*frames rows in e->prompted /
   e->joint_enc), 0 if nothing to do, -1 on error. */
static int enc_step(or_encoder_t *e, int final, int *frames, char *err, size_t errlen) {
    *frames = 0;
    if (e->closed) return 0;
    if (e->pending_n == 0) { if (final) e->closed = 1; return 0; }
    if ((int)e->pending_n < e->chunk_mel && !final) return 0;
    size_t take = (size_t)e->chunk_mel < e->pending_n ? (size_t)e->chunk_mel : e->pending_n;
    if (final && e->pending_n <= (size_t)e->chunk_mel) take = e->pending_n;
    const int include_boundary = final && e->pending_n == take;
    const int nwin = e->mel_cache_n + (int)take;
    memcpy(e->win, e->mel_cache, (size_t)e->mel_cache_n * MEL_NMEL * sizeof(float));
    memcpy(e->win + (size_t)e->mel_cache_n * MEL_NMEL, e->pending, take * MEL_NMEL * sizeof(float));
    const size_t end = e->consumed + take;
    const size_t base = (e->consumed - (size_t)e->mel_cache_n) / 8;
    const size_t lo = e->emitted - base;
    const int T3 = sub_len(sub_len(sub_len(nwin)));
    const size_t hi = include_boundary ? (size_t)T3 : end / 8 - base;
    e->consumed = end;
    const int keep = nwin < MEL_CACHE ? nwin : MEL_CACHE;
    memcpy(e->mel_cache, e->win + (size_t)(nwin - keep) * MEL_NMEL, (size_t)keep * MEL_NMEL * sizeof(float));
    e->mel_cache_n = keep;
    memmove(e->pending, e->pending + take * MEL_NMEL, (e->pending_n - take) * MEL_NMEL * sizeof(float));
    e->pending_n -= take;
    if (final && e->pending_n == 0) e->closed = 1;
    if (hi <= lo) { e->emitted = base + (lo > hi ? lo : hi); return 1; }
    e->emitted = base + hi;
    const int c = (int)(hi - lo);
    if (c > e->cmax) { snprintf(err, errlen, "chunk of %d rows exceeds buffer %d", c, e->cmax); return -1; }
    if (e->pos + c > e->cap_rows) compact_caches(e);
    run_pre_encode(e, nwin);
    memcpy(e->h, e->pre_out + lo * (size_t)e->m->D, (size_t)c * (size_t)e->m->D * sizeof(float));
    run_blocks(e, c);
    *frames = c;
    return 1;
}

/* ================================ decoder (src/decoder.c) ============================= */
typedef struct {
    or_model_t *m;
    float *x, *gates, *pred_out;
    float *h[2], *c[2], *hp[2], *cp[2];
    int last_token, pred_valid;
} or_decoder_t;

static void dec_reset(or_decoder_t *d) {
    const size_t PH = (size_t)d->m->c.pred_hidden;
    for (int l = 0; l < 2; ++l) { memset(d->h[l], 0, PH * sizeof(float)); memset(d->c[l], 0, PH * sizeof(float)); }
    d->last_token = d->m->blank;
    d->pred_valid = 0;
}
static or_decoder_t *dec_create(or_model_t *m) {
    or_decoder_t *d = calloc(1, sizeof *d);
    d->m = m;
    const size_t PH = (size_t)m->c.pred_hidden;
    d->x = calloc(PH, sizeof(float));
    d->gates = calloc(4 * PH, sizeof(float));
    d->pred_out = calloc((size_t)m->c.joint_hidden, sizeof(float));
    for (int l = 0; l < 2; ++l) {
        d->h[l] = calloc(PH, sizeof(float)); d->c[l] = calloc(PH, sizeof(float));
        d->hp[l] = calloc(PH, sizeof(float)); d->cp[l] = calloc(PH, sizeof(float));
    }
    dec_reset(d);
    return d;
}
static void dec_destroy(or_decoder_t *d) {
    if (!d) return;
    free(d->x); free(d->gates); free(d->pred_out);
    for (int l = 0; l < 2; ++l) { free(d->h[l]); free(d->c[l]); free(d->hp[l]); free(d->cp[l]); }
    free(d);
}
/* decoder.c:58-77: input embed(last) (zeros for blank), 2 LSTM layers from the committed state
   into the provisional state, then the joint prediction projection. */
static void encode_pred(or_decoder_t *d) {
    or_model_t *m = d->m;
    const int PH = m->c.pred_hidden, JH = m->c.joint_hidden;
    if (d->last_token == m->blank) memset(d->x, 0, (size_t)PH * sizeof(float));
    else for (int i = 0; i < PH; ++i) d->x[i] = bf2f(m->embed[(size_t)d->last_token * PH + i]);
    const float *in = d->x;
    for (int l = 0; l < 2; ++l) {
        or_gemm(in, PH, m->lstm_wx[l], PH, m->lstm_b[l], d->gates, 4 * PH, 1, 4 * PH, PH, 0, 0, 1.0f);
        or_gemm(d->h[l], PH, m->lstm_wh[l], PH, NULL, d->gates, 4 * PH, 1, 4 * PH, PH, 0, 1, 1.0f);
        or_lstm_cell(d->gates, d->c[l], d->cp[l], d->hp[l], PH);
        in = d->hp[l];
    }
    or_gemm(d->hp[1], PH, m->joint_pred_w, PH, m->joint_pred_b, d->pred_out, JH, 1, JH, PH, 0, 0, 1.0f);
}

struct or_session {
    or_model_t *m;
    or_encoder_t *enc;
    or_decoder_t *dec;
    or_mel_t *mel;
    or_resampler_t *rs;
    int input_rate, finished;
    float *tmp, *melbuf;
    size_t tmp_cap, melbuf_cap;
    double audio_s;
    size_t chunks, tokens;
    /* taps */
    float *tap_prompted, *tap_joint;
    size_t tap_cap, tap_rows;
    int *tap_chunk_rows;
    size_t tap_chunk_cap, tap_chunks;
    int *dec_frame, *dec_token;
    float *dec_margin;
    size_t dec_cap, dec_n, frame_base;
};

/* decoder.c:92-127: greedy loop. Frames [t, t+rows) are scored with the current prediction
   (speculating blank); the first non-blank emits, commits the provisional state and re-scores
   the frames after it; max_symbols emissions on one frame move on to the next frame. */
static int dec_run(or_session_t *s, const float *joint_enc, int frames, int *out, int max_out) {
    or_decoder_t *d = s->dec;
    or_model_t *m = d->m;
    const int JH = m->c.joint_hidden;
    int n = 0, t = 0, symbols = 0;
    int idx[DEC_MAX_BATCH];
    float val[DEC_MAX_BATCH], mar[DEC_MAX_BATCH];
    while (t < frames) {
        int rows = frames - t;
        if (rows > DEC_MAX_BATCH) rows = DEC_MAX_BATCH;
        if (!d->pred_valid) encode_pred(d);
        or_joint_argmax(joint_enc + (size_t)t * JH, JH, d->pred_out, m->joint_out_w, m->joint_out_b, m->NC, JH, rows, idx, val, mar);
        d->pred_valid = 1;
        int i = 0;
        for (; i < rows; ++i) {
            const int pred = idx[i];
            if (s->dec_frame && s->dec_n < s->dec_cap) {
                s->dec_frame[s->dec_n] = (int)s->frame_base + t + i;
                s->dec_token[s->dec_n] = pred;
                s->dec_margin[s->dec_n] = mar[i];
            }
            s->dec_n++;
            if (pred == m->blank) { symbols = 0; continue; }
            if (n < max_out) out[n++] = pred;
            d->last_token = pred;
            for (int l = 0; l < 2; ++l) {
                float *sw = d->h[l]; d->h[l] = d->hp[l]; d->hp[l] = sw;
                sw = d->c[l]; d->c[l] = d->cp[l]; d->cp[l] = sw;
            }
            d->pred_valid = 0;
            symbols++;
            if (symbols >= m->c.max_symbols) { symbols = 0; i++; }
            break;
        }
        t += i;
    }
    return n;
}

static const int LAT_MS[] = { 80, 160, 320, 560, 1120 };  /* nemoasr.c:58-59 */
static const int LAT_R[] = { 0, 1, 3, 6, 13 };

or_session_t *or_open(or_model_t *m, int latency_ms, int input_rate, char *err, size_t errlen) {
    int right = -1;
    for (int i = 0; i < 5; ++i) if (LAT_MS[i] == latency_ms) right = LAT_R[i];
    if (right < 0) { snprintf(err, errlen, "latency must be one of 80, 160, 320, 560, 1120 ms"); return NULL; }
    if (input_rate <= 0) { snprintf(err, errlen, "input_rate must be positive"); return NULL; }
    or_session_t *s = calloc(1, sizeof *s);
    s->m = m;
    s->enc = enc_create(m, right);
    s->dec = dec_create(m);
    s->mel = or_mel_create();
    s->input_rate = input_rate;
    if (input_rate != MEL_SR) s->rs = or_resampler_create(input_rate, MEL_SR);
    return s;
}
void or_close(or_session_t *s) {
    if (!s) return;
    enc_destroy(s->enc);
    dec_destroy(s->dec);
    or_mel_destroy(s->mel);
    or_resampler_destroy(s->rs);
    free(s->tmp);
    free(s->melbuf);
    free(s);
}
void or_set_taps(or_session_t *s, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks,
                 int *dec_frame, int *dec_token, float *dec_margin, size_t cap_dec) {
    s->tap_prompted = prompted; s->tap_joint = joint_enc; s->tap_cap = cap_rows; s->tap_rows = 0;
    s->tap_chunk_rows = chunk_rows; s->tap_chunk_cap = cap_chunks; s->tap_chunks = 0;
    s->dec_frame = dec_frame; s->dec_token = dec_token; s->dec_margin = dec_margin; s->dec_cap = cap_dec; s->dec_n = 0;
}
void or_tap_counts(const or_session_t *s, size_t *rows, size_t *chunks, size_t *decisions) {
    *rows = s->tap_rows; *chunks = s->tap_chunks; *decisions = s->dec_n;
}
void or_stats(const or_session_t *s, double *audio_s, size_t *chunks, size_t *tokens) {
    *audio_s = s->audio_s; *chunks = s->chunks; *tokens = s->tokens;
}

/* nemoasr.c:112-132 */
static int run_pending(or_session_t *s, int final, int *tokens, int max_tokens, int *nout, char *err, size_t errlen) {
    int rc, frames;
    while ((rc = enc_step(s->enc, final, &frames, err, errlen)) == 1) {
        if (frames <= 0) continue;
        s->chunks++;
        const or_model_t *m = s->m;
        if (s->tap_prompted) {
            for (int r = 0; r < frames && s->tap_rows < s->tap_cap; ++r, ++s->tap_rows) {
                memcpy(s->tap_prompted + s->tap_rows * (size_t)m->D, s->enc->prompted + (size_t)r * m->D, (size_t)m->D * sizeof(float));
                memcpy(s->tap_joint + s->tap_rows * (size_t)m->c.joint_hidden, s->enc->joint_enc + (size_t)r * m->c.joint_hidden,
                       (size_t)m->c.joint_hidden * sizeof(float));
            }
            if (s->tap_chunks < s->tap_chunk_cap) s->tap_chunk_rows[s->tap_chunks] = frames;
            s->tap_chunks++;
        }
        const int room = max_tokens - *nout;
        int buf[4096];
        const int n = dec_run(s, s->enc->joint_enc, frames, buf, 4096);
        s->frame_base += (size_t)frames;
        for (int i = 0; i < n && i < room; ++i) tokens[*nout + i] = buf[i];
        *nout += n < room ? n : room;
        s->tokens += (size_t)n;
    }
    return rc;
}

/* nemoasr.c:134-160 */
int or_feed(or_session_t *s, const float *samples, size_t n, int final, int *tokens, int max_tokens, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    if (s->finished) return 0;
    const float *in = samples;
    size_t count = n;
    if (s->rs) {
        const size_t need = (size_t)((double)n * MEL_SR / s->input_rate) + 4096;
        if (need > s->tmp_cap) { s->tmp_cap = need * 2; s->tmp = realloc(s->tmp, s->tmp_cap * sizeof(float)); }
        count = n ? or_resampler_process(s->rs, samples, n, s->tmp, s->tmp_cap) : 0;
        if (final) count += or_resampler_flush(s->rs, s->tmp + count, s->tmp_cap - count);
        in = s->tmp;
    }
    s->audio_s += (double)count / MEL_SR;
    int nout = 0;
    if (!(final && count == 0 && s->mel->total == 0)) {
        const size_t maxf = (s->mel->total + count) / MEL_HOP + 2;
        if (maxf * MEL_NMEL > s->melbuf_cap) { s->melbuf_cap = maxf * MEL_NMEL; s->melbuf = realloc(s->melbuf, s->melbuf_cap * sizeof(float)); }
        const size_t nf = or_mel_push(s->mel, in, count, final, s->melbuf, maxf);
        if (nf) enc_push(s->enc, s->melbuf, nf);
        if (run_pending(s, final, tokens, max_tokens, &nout, err, errlen) < 0) return -1;
    }
    if (final) s->finished = 1;
    return nout;
}
