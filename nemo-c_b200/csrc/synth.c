/* Seeded random-init model of the Nemotron-ASR streaming shape, and seeded synthetic audio.

   The reference loads a trained checkpoint (src/model.c:185-310). This build has none, so every
   run uses a deterministic random model: each tensor has its own counter-based normal stream
   keyed by (seed, tensor name), so any tensor can be regenerated alone, in any order, on any
   thread. Tensor names, shapes and the bf16 storage type are those src/model.c:216-282 loads. */
#include "nb.h"
#include <errno.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

static uint64_t splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}
static uint64_t fnv1a(const char *s) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (; *s; ++s) { h ^= (unsigned char)*s; h *= 0x100000001b3ull; }
    return h;
}
/* Standard normal number i of stream `key` (Box-Muller on one 64-bit counter hash). */
static double normal_at(uint64_t key, uint64_t i) {
    uint64_t x = splitmix64(key ^ splitmix64(i));
    double u1 = ((double)(x >> 32) + 1.0) * (1.0 / 4294967296.0);
    double u2 = (double)(x & 0xffffffffu) * (1.0 / 4294967296.0);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

void nemoasr_synth_default(nemoasr_synth_spec_t *s) {
    memset(s, 0, sizeof *s);
    s->seed = 1234;
    s->n_layers = 24;
    s->d_model = 1024;
    s->ff_factor = 4;
    s->sub_channels = 256;
    s->num_prompts = 128;
    s->prompt_hidden = 2048;
    s->pred_hidden = 640;
    s->joint_hidden = 640;
    s->vocab_size = 1024;
    s->att_left = 56;
    s->weight_std = 0.02f;
    /* With this random model an emitting frame runs to max_symbols, so the blank offset sets
       how many frames emit: 0.383 makes ~35% of frames emit on the 4 s / 560 ms chirp stream. */
    s->blank_bias = 0.383f;
}

typedef enum { K_NORMAL, K_ONES, K_ZEROS, K_JOINT_BIAS } tkind;

static int sub_freq(int f) { for (int i = 0; i < 3; ++i) f = f / 2 + 1; return f; }

/* Build the tensor table. Returns count; fills info (if non-NULL) and kinds. */
static int build_table(const nemoasr_synth_spec_t *sp, nb_tensor_info_t *info, tkind *kinds) {
    const int64_t D = sp->d_model, CH = sp->sub_channels, FF = (int64_t)sp->d_model * sp->ff_factor;
    const int64_t PH = sp->pred_hidden, JH = sp->joint_hidden, V = sp->vocab_size, PRH = sp->prompt_hidden;
    const int64_t NP = sp->num_prompts, F3 = sub_freq(128);
    int n = 0;
#define T(nm, k, nd, a, b, c, d)                                                                   \
    do {                                                                                           \
        if (info) {                                                                                \
            snprintf(info[n].name, sizeof info[n].name, "%s", nm);                                 \
            info[n].ndim = nd; info[n].shape[0] = a; info[n].shape[1] = b; info[n].shape[2] = c; info[n].shape[3] = d; \
            info[n].numel = (size_t)(a) * (nd > 1 ? (size_t)(b) : 1) * (nd > 2 ? (size_t)(c) : 1) * (nd > 3 ? (size_t)(d) : 1); \
            kinds[n] = k;                                                                          \
        }                                                                                          \
        ++n;                                                                                       \
    } while (0)
    char nm[96];
    T("encoder.pre_encode.conv.0.weight", K_NORMAL, 4, CH, 1, 3, 3);
    T("encoder.pre_encode.conv.0.bias", K_NORMAL, 1, CH, 0, 0, 0);
    T("encoder.pre_encode.conv.2.weight", K_NORMAL, 4, CH, 1, 3, 3);
    T("encoder.pre_encode.conv.2.bias", K_NORMAL, 1, CH, 0, 0, 0);
    T("encoder.pre_encode.conv.3.weight", K_NORMAL, 4, CH, CH, 1, 1);
    T("encoder.pre_encode.conv.3.bias", K_NORMAL, 1, CH, 0, 0, 0);
    T("encoder.pre_encode.conv.5.weight", K_NORMAL, 4, CH, 1, 3, 3);
    T("encoder.pre_encode.conv.5.bias", K_NORMAL, 1, CH, 0, 0, 0);
    T("encoder.pre_encode.conv.6.weight", K_NORMAL, 4, CH, CH, 1, 1);
    T("encoder.pre_encode.conv.6.bias", K_NORMAL, 1, CH, 0, 0, 0);
    T("encoder.pre_encode.out.weight", K_NORMAL, 2, D, CH * F3, 0, 0);
    T("encoder.pre_encode.out.bias", K_NORMAL, 1, D, 0, 0, 0);
    for (int l = 0; l < sp->n_layers; ++l) {
#define L(suffix, k, nd, a, b, c) do { snprintf(nm, sizeof nm, "encoder.layers.%d.%s", l, suffix); T(nm, k, nd, a, b, c, 0); } while (0)
        L("feed_forward1.linear1.weight", K_NORMAL, 2, FF, D, 0);
        L("feed_forward1.linear2.weight", K_NORMAL, 2, D, FF, 0);
        L("feed_forward2.linear1.weight", K_NORMAL, 2, FF, D, 0);
        L("feed_forward2.linear2.weight", K_NORMAL, 2, D, FF, 0);
        L("self_attn.linear_q.weight", K_NORMAL, 2, D, D, 0);
        L("self_attn.linear_k.weight", K_NORMAL, 2, D, D, 0);
        L("self_attn.linear_v.weight", K_NORMAL, 2, D, D, 0);
        L("self_attn.linear_out.weight", K_NORMAL, 2, D, D, 0);
        L("self_attn.linear_pos.weight", K_NORMAL, 2, D, D, 0);
        L("conv.pointwise_conv1.weight", K_NORMAL, 3, 2 * D, D, 1);
        L("conv.pointwise_conv2.weight", K_NORMAL, 3, D, D, 1);
        L("norm_feed_forward1.weight", K_ONES, 1, D, 0, 0);
        L("norm_feed_forward1.bias", K_ZEROS, 1, D, 0, 0);
        L("norm_self_att.weight", K_ONES, 1, D, 0, 0);
        L("norm_self_att.bias", K_ZEROS, 1, D, 0, 0);
        L("norm_conv.weight", K_ONES, 1, D, 0, 0);
        L("norm_conv.bias", K_ZEROS, 1, D, 0, 0);
        L("norm_feed_forward2.weight", K_ONES, 1, D, 0, 0);
        L("norm_feed_forward2.bias", K_ZEROS, 1, D, 0, 0);
        L("norm_out.weight", K_ONES, 1, D, 0, 0);
        L("norm_out.bias", K_ZEROS, 1, D, 0, 0);
        L("conv.batch_norm.weight", K_ONES, 1, D, 0, 0);
        L("conv.batch_norm.bias", K_ZEROS, 1, D, 0, 0);
        L("conv.depthwise_conv.weight", K_NORMAL, 3, D, 1, 9);
        L("self_attn.pos_bias_u", K_NORMAL, 2, D / 128, 128, 0);
        L("self_attn.pos_bias_v", K_NORMAL, 2, D / 128, 128, 0);
#undef L
    }
    T("prompt_kernel.0.weight", K_NORMAL, 2, PRH, D + NP, 0, 0);
    T("prompt_kernel.0.bias", K_NORMAL, 1, PRH, 0, 0, 0);
    T("prompt_kernel.2.weight", K_NORMAL, 2, D, PRH, 0, 0);
    T("prompt_kernel.2.bias", K_NORMAL, 1, D, 0, 0, 0);
    for (int l = 0; l < 2; ++l) {
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.Wx", l); T(nm, K_NORMAL, 2, 4 * PH, PH, 0, 0);
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.Wh", l); T(nm, K_NORMAL, 2, 4 * PH, PH, 0, 0);
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.bias", l); T(nm, K_NORMAL, 1, 4 * PH, 0, 0, 0);
    }
    T("decoder.prediction.embed.weight", K_NORMAL, 2, V + 1, PH, 0, 0);
    T("joint.enc.weight", K_NORMAL, 2, JH, D, 0, 0);
    T("joint.enc.bias", K_NORMAL, 1, JH, 0, 0, 0);
    T("joint.pred.weight", K_NORMAL, 2, JH, PH, 0, 0);
    T("joint.pred.bias", K_NORMAL, 1, JH, 0, 0, 0);
    T("joint.joint_net.2.weight", K_NORMAL, 2, V + 1, JH, 0, 0);
    T("joint.joint_net.2.bias", K_JOINT_BIAS, 1, V + 1, 0, 0, 0);
#undef T
    return n;
}

int nb_synth_tensor_list(const nemoasr_synth_spec_t *spec, nb_tensor_info_t **out) {
    int n = build_table(spec, NULL, NULL);
    nb_tensor_info_t *info = calloc((size_t)n, sizeof *info);
    tkind *kinds = calloc((size_t)n, sizeof *kinds);
    build_table(spec, info, kinds);
    free(kinds);
    *out = info;
    return n;
}

int nb_synth_tensor(const nemoasr_synth_spec_t *spec, const char *name, size_t numel, uint16_t *dst) {
    int n = build_table(spec, NULL, NULL);
    nb_tensor_info_t *info = calloc((size_t)n, sizeof *info);
    tkind *kinds = calloc((size_t)n, sizeof *kinds);
    build_table(spec, info, kinds);
    int idx = -1;
    for (int i = 0; i < n; ++i) if (!strcmp(info[i].name, name)) { idx = i; break; }
    int rc = -1;
    if (idx >= 0 && info[idx].numel == numel) {
        const tkind k = kinds[idx];
        const uint64_t key = splitmix64(spec->seed) ^ fnv1a(name);
        const double sd = spec->weight_std;
        if (k == K_ONES || k == K_ZEROS) {
            const uint16_t v = k == K_ONES ? 0x3f80 : 0;
            for (size_t i = 0; i < numel; ++i) dst[i] = v;
        } else {
#pragma omp parallel for schedule(static) if (numel > (1u << 16))
            for (long long i = 0; i < (long long)numel; ++i) dst[i] = nb_f32_to_bf16((float)(sd * normal_at(key, (uint64_t)i)));
            if (k == K_JOINT_BIAS) {
                const size_t blank = (size_t)spec->vocab_size;
                dst[blank] = nb_f32_to_bf16(nb_bf16_to_f32(dst[blank]) + spec->blank_bias);
            }
        }
        rc = 0;
    }
    free(info);
    free(kinds);
    return rc;
}

static void sb_printf(char **buf, size_t *len, size_t *cap, const char *fmt, ...) __attribute__((format(printf, 4, 5)));
#include <stdarg.h>
static void sb_printf(char **buf, size_t *len, size_t *cap, const char *fmt, ...) {
    for (;;) {
        va_list ap;
        va_start(ap, fmt);
        int k = vsnprintf(*buf + *len, *cap - *len, fmt, ap);
        va_end(ap);
        if (k >= 0 && (size_t)k < *cap - *len) { *len += (size_t)k; return; }
        *cap = (*cap + (size_t)(k > 0 ? k : 64)) * 2;
        *buf = realloc(*buf, *cap);
    }
}

/* config.json in the layout src/model.c:125-172 parses. Vocabulary: piece 0 "<unk>", the rest
   "▁tok<i>" (so every emitted id maps to visible text " tok<i>"). Prompt dictionary:
   "auto" -> 0, "en-US" -> 1, "lang<i>" -> i for the remaining slots. */
char *nb_synth_config_json(const nemoasr_synth_spec_t *sp) {
    size_t len = 0, cap = 4096;
    char *b = malloc(cap);
    b[0] = 0;
    sb_printf(&b, &len, &cap,
              "{\n \"encoder\": {\"feat_in\": 128, \"n_layers\": %d, \"d_model\": %d, \"n_heads\": %d, "
              "\"ff_expansion_factor\": %d, \"subsampling_factor\": 8, \"subsampling_conv_channels\": %d, "
              "\"conv_kernel_size\": 9, \"att_context_size\": [[%d, 13], [%d, 6], [%d, 3], [%d, 1], [%d, 0]]},\n",
              sp->n_layers, sp->d_model, sp->d_model / 128, sp->ff_factor, sp->sub_channels,
              sp->att_left, sp->att_left, sp->att_left, sp->att_left, sp->att_left);
    sb_printf(&b, &len, &cap, " \"preprocessor\": {\"sample_rate\": 16000, \"features\": 128},\n");
    sb_printf(&b, &len, &cap, " \"prompt\": {\"num_prompts\": %d, \"prompt_hidden\": %d, \"prompt_dictionary\": {\"auto\": 0",
              sp->num_prompts, sp->prompt_hidden);
    if (sp->num_prompts > 1) sb_printf(&b, &len, &cap, ", \"en-US\": 1");
    for (int i = 2; i < sp->num_prompts; ++i) sb_printf(&b, &len, &cap, ", \"lang%d\": %d", i, i);
    sb_printf(&b, &len, &cap, "}},\n");
    sb_printf(&b, &len, &cap, " \"decoder\": {\"pred_hidden\": %d, \"pred_rnn_layers\": 2, \"vocab_size\": %d},\n",
              sp->pred_hidden, sp->vocab_size);
    sb_printf(&b, &len, &cap, " \"joint\": {\"joint_hidden\": %d, \"num_classes\": %d},\n", sp->joint_hidden, sp->vocab_size);
    sb_printf(&b, &len, &cap, " \"max_symbols\": 10,\n \"default_att_context_size\": [%d, 13],\n \"vocabulary\": [\"<unk>\"", sp->att_left);
    for (int i = 1; i < sp->vocab_size; ++i) sb_printf(&b, &len, &cap, ", \"\xe2\x96\x81tok%d\"", i);
    sb_printf(&b, &len, &cap, "]\n}\n");
    return b;
}

int nemoasr_synth_write(const char *dir, const nemoasr_synth_spec_t *spec, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    if (mkdir(dir, 0755) != 0 && errno != EEXIST) { snprintf(err, errlen, "cannot create %s", dir); return -1; }
    char path[4096];
    snprintf(path, sizeof path, "%s/config.json", dir);
    FILE *f = fopen(path, "wb");
    if (!f) { snprintf(err, errlen, "cannot write %s", path); return -1; }
    char *cfg = nb_synth_config_json(spec);
    fputs(cfg, f);
    free(cfg);
    fclose(f);

    nb_tensor_info_t *info;
    int n = nb_synth_tensor_list(spec, &info);
    /* safetensors: u64 header length, JSON header, raw little-endian data */
    size_t len = 0, cap = 65536;
    char *h = malloc(cap);
    h[0] = 0;
    sb_printf(&h, &len, &cap, "{\"__metadata__\": {\"format\": \"pt\"}");
    size_t off = 0;
    for (int i = 0; i < n; ++i) {
        sb_printf(&h, &len, &cap, ", \"%s\": {\"dtype\": \"BF16\", \"shape\": [", info[i].name);
        for (int d = 0; d < info[i].ndim; ++d) sb_printf(&h, &len, &cap, "%s%lld", d ? ", " : "", (long long)info[i].shape[d]);
        sb_printf(&h, &len, &cap, "], \"data_offsets\": [%zu, %zu]}", off, off + info[i].numel * 2);
        off += info[i].numel * 2;
    }
    sb_printf(&h, &len, &cap, "}");
    while (len % 8) sb_printf(&h, &len, &cap, " ");
    snprintf(path, sizeof path, "%s/model.safetensors", dir);
    f = fopen(path, "wb");
    if (!f) { free(h); free(info); snprintf(err, errlen, "cannot write %s", path); return -1; }
    uint64_t hl = len;
    fwrite(&hl, 8, 1, f);
    fwrite(h, 1, len, f);
    free(h);
    int rc = 0;
    for (int i = 0; i < n && !rc; ++i) {
        uint16_t *buf = malloc(info[i].numel * 2);
        if (nb_synth_tensor(spec, info[i].name, info[i].numel, buf)) rc = -1;
        else if (fwrite(buf, 2, info[i].numel, f) != info[i].numel) rc = -1;
        free(buf);
    }
    if (fclose(f) != 0) rc = -1;
    free(info);
    if (rc) snprintf(err, errlen, "failed writing %s", path);
    return rc;
}

/* ---- audio -------------------------------------------------------------------------------- */
/* Chirp k sweeps 100 -> 4000 Hz linearly over a period of CHIRP_PERIOD[k] seconds and restarts
   (sawtooth frequency), starting at phase CHIRP_PHASE[k]. */
static const double CHIRP_PERIOD[3] = { 1.0, 1.7, 2.9 };
static const double CHIRP_PHASE[3] = { 0.0, 2.0943951023931953, 4.1887902047863905 };

void nemoasr_synth_audio(uint64_t seed, int rate, size_t n, int pauses, float *out) {
    const double f0 = 100.0, f1 = 4000.0;
    const uint64_t nkey = splitmix64(seed ^ 0x6e6f697365ull);      /* noise stream */
    const uint64_t pkey = splitmix64(seed ^ 0x7061757365ull);      /* pause schedule */
    /* pause schedule: speech for U[1,3] s, then silence (chirps muted) for U[0.2,0.6] s, ... */
    double seg_end = 0.0, gap_end = 0.0;
    uint64_t seg = 0;
    if (pauses) {
        double u = (double)(splitmix64(pkey + 2 * seg) >> 11) * (1.0 / 9007199254740992.0);
        seg_end = 1.0 + 2.0 * u;
        u = (double)(splitmix64(pkey + 2 * seg + 1) >> 11) * (1.0 / 9007199254740992.0);
        gap_end = seg_end + 0.2 + 0.4 * u;
    }
    for (size_t i = 0; i < n; ++i) {
        const double t = (double)i / rate;
        double amp = 1.0;
        if (pauses) {
            while (t >= gap_end) {
                ++seg;
                double u = (double)(splitmix64(pkey + 2 * seg) >> 11) * (1.0 / 9007199254740992.0);
                seg_end = gap_end + 1.0 + 2.0 * u;
                u = (double)(splitmix64(pkey + 2 * seg + 1) >> 11) * (1.0 / 9007199254740992.0);
                gap_end = seg_end + 0.2 + 0.4 * u;
            }
            if (t >= seg_end) amp = 0.0;
        }
        double s = 0.0;
        for (int k = 0; k < 3; ++k) {
            const double P = CHIRP_PERIOD[k], q = t / P, nper = floor(q), fr = q - nper;
            /* phase = 2*pi * integral of f: f0*t + (f1-f0)*P*(nper/2 + fr^2/2) */
            const double ph = 6.283185307179586 * (f0 * t + (f1 - f0) * P * (0.5 * nper + 0.5 * fr * fr)) + CHIRP_PHASE[k];
            s += 0.15 * sin(ph);
        }
        out[i] = (float)(amp * s + 0.05 * normal_at(nkey, (uint64_t)i));
    }
}
