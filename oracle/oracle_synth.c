/* ORACLE — TEST INFRASTRUCTURE ONLY.

   The benchmark's synthetic workload (random-init checkpoint of the Nemotron-ASR streaming shape
   in the reference's file format, and seeded chirp + noise audio), generated here so that the
   CPU reference arm of bench.py never loads the product library. Same definition as the
   product's generator: every tensor value is weight_std * N(0,1) from a counter-based normal
   stream keyed by (seed, tensor name) (SplitMix64 finaliser, then Box-Muller on the two 32-bit
   halves of one 64-bit hash), rounded to bf16 to nearest even; LayerNorm gains 1, shifts 0; the
   blank entry of the joint bias offset by blank_bias. Tensor names and shapes are those the
   reference loads (src/model.c:216-282). tests/test_oracle_synth.py checks that both generators
   write identical bytes. */
#include "oracle.h"
#include <errno.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

static uint64_t mix(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

static uint64_t name_hash(const char *s) { /* FNV-1a, 64 bit */
    uint64_t h = 0xcbf29ce484222325ull;
    while (*s) h = (h ^ (unsigned char)*s++) * 0x100000001b3ull;
    return h;
}

static double gauss(uint64_t key, uint64_t i) {
    const uint64_t x = mix(key ^ mix(i));
    const double u1 = ((double)(x >> 32) + 1.0) / 4294967296.0, u2 = (double)(x & 0xffffffffu) / 4294967296.0;
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static uint16_t to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t)((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
static float from_bf16(uint16_t v) {
    const uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

void or_synth_default(or_synth_spec_t *s) {
    memset(s, 0, sizeof *s);
    s->seed = 1234;
    s->n_layers = 24; s->d_model = 1024; s->ff_factor = 4; s->sub_channels = 256;
    s->num_prompts = 128; s->prompt_hidden = 2048; s->pred_hidden = 640; s->joint_hidden = 640;
    s->vocab_size = 1024; s->att_left = 56;
    s->weight_std = 0.02f;
    s->blank_bias = 0.383f;
}

/* ---- tensor table ------------------------------------------------------------------------ */
enum { G_NORMAL, G_ONE, G_ZERO, G_JBIAS };
typedef struct { char name[96]; int kind, ndim; long long dim[4]; } tdesc;
typedef struct { tdesc *t; int n, cap; } ttab;

static void add(ttab *tb, int kind, int ndim, long long a, long long b, long long c, long long d, const char *fmt, ...) {
    if (tb->n == tb->cap) { tb->cap = tb->cap ? 2 * tb->cap : 256; tb->t = realloc(tb->t, (size_t)tb->cap * sizeof *tb->t); }
    tdesc *x = &tb->t[tb->n++];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(x->name, sizeof x->name, fmt, ap);
    va_end(ap);
    x->kind = kind; x->ndim = ndim;
    x->dim[0] = a; x->dim[1] = b; x->dim[2] = c; x->dim[3] = d;
}
static size_t numel(const tdesc *x) {
    size_t n = 1;
    for (int i = 0; i < x->ndim; ++i) n *= (size_t)x->dim[i];
    return n;
}

/* In the order the product writes them (the file layout must match byte for byte). */
static ttab tensors(const or_synth_spec_t *s) {
    ttab tb = { 0 };
    const long long D = s->d_model, CH = s->sub_channels, FF = (long long)s->d_model * s->ff_factor, PH = s->pred_hidden;
    const long long JH = s->joint_hidden, V = s->vocab_size, PRH = s->prompt_hidden, NP = s->num_prompts;
    long long F3 = 128;
    for (int i = 0; i < 3; ++i) F3 = F3 / 2 + 1;
    static const int conv_idx[5] = { 0, 2, 3, 5, 6 };
    for (int i = 0; i < 5; ++i) {
        const int pw = conv_idx[i] == 3 || conv_idx[i] == 6;
        add(&tb, G_NORMAL, 4, CH, pw ? CH : 1, pw ? 1 : 3, pw ? 1 : 3, "encoder.pre_encode.conv.%d.weight", conv_idx[i]);
        add(&tb, G_NORMAL, 1, CH, 0, 0, 0, "encoder.pre_encode.conv.%d.bias", conv_idx[i]);
    }
    add(&tb, G_NORMAL, 2, D, CH * F3, 0, 0, "encoder.pre_encode.out.weight");
    add(&tb, G_NORMAL, 1, D, 0, 0, 0, "encoder.pre_encode.out.bias");
    for (int l = 0; l < s->n_layers; ++l) {
        const char *p = "encoder.layers";
        for (int f = 1; f <= 2; ++f) {
            add(&tb, G_NORMAL, 2, FF, D, 0, 0, "%s.%d.feed_forward%d.linear1.weight", p, l, f);
            add(&tb, G_NORMAL, 2, D, FF, 0, 0, "%s.%d.feed_forward%d.linear2.weight", p, l, f);
        }
        static const char *att[5] = { "q", "k", "v", "out", "pos" };
        for (int i = 0; i < 5; ++i) add(&tb, G_NORMAL, 2, D, D, 0, 0, "%s.%d.self_attn.linear_%s.weight", p, l, att[i]);
        add(&tb, G_NORMAL, 3, 2 * D, D, 1, 0, "%s.%d.conv.pointwise_conv1.weight", p, l);
        add(&tb, G_NORMAL, 3, D, D, 1, 0, "%s.%d.conv.pointwise_conv2.weight", p, l);
        static const char *norms[5] = { "norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out" };
        for (int i = 0; i < 5; ++i) {
            add(&tb, G_ONE, 1, D, 0, 0, 0, "%s.%d.%s.weight", p, l, norms[i]);
            add(&tb, G_ZERO, 1, D, 0, 0, 0, "%s.%d.%s.bias", p, l, norms[i]);
        }
        add(&tb, G_ONE, 1, D, 0, 0, 0, "%s.%d.conv.batch_norm.weight", p, l);
        add(&tb, G_ZERO, 1, D, 0, 0, 0, "%s.%d.conv.batch_norm.bias", p, l);
        add(&tb, G_NORMAL, 3, D, 1, 9, 0, "%s.%d.conv.depthwise_conv.weight", p, l);
        add(&tb, G_NORMAL, 2, D / 128, 128, 0, 0, "%s.%d.self_attn.pos_bias_u", p, l);
        add(&tb, G_NORMAL, 2, D / 128, 128, 0, 0, "%s.%d.self_attn.pos_bias_v", p, l);
    }
    add(&tb, G_NORMAL, 2, PRH, D + NP, 0, 0, "prompt_kernel.0.weight");
    add(&tb, G_NORMAL, 1, PRH, 0, 0, 0, "prompt_kernel.0.bias");
    add(&tb, G_NORMAL, 2, D, PRH, 0, 0, "prompt_kernel.2.weight");
    add(&tb, G_NORMAL, 1, D, 0, 0, 0, "prompt_kernel.2.bias");
    for (int l = 0; l < 2; ++l) {
        add(&tb, G_NORMAL, 2, 4 * PH, PH, 0, 0, "decoder.prediction.dec_rnn.lstm.%d.Wx", l);
        add(&tb, G_NORMAL, 2, 4 * PH, PH, 0, 0, "decoder.prediction.dec_rnn.lstm.%d.Wh", l);
        add(&tb, G_NORMAL, 1, 4 * PH, 0, 0, 0, "decoder.prediction.dec_rnn.lstm.%d.bias", l);
    }
    add(&tb, G_NORMAL, 2, V + 1, PH, 0, 0, "decoder.prediction.embed.weight");
    add(&tb, G_NORMAL, 2, JH, D, 0, 0, "joint.enc.weight");
    add(&tb, G_NORMAL, 1, JH, 0, 0, 0, "joint.enc.bias");
    add(&tb, G_NORMAL, 2, JH, PH, 0, 0, "joint.pred.weight");
    add(&tb, G_NORMAL, 1, JH, 0, 0, 0, "joint.pred.bias");
    add(&tb, G_NORMAL, 2, V + 1, JH, 0, 0, "joint.joint_net.2.weight");
    add(&tb, G_JBIAS, 1, V + 1, 0, 0, 0, "joint.joint_net.2.bias");
    return tb;
}

static void fill(const or_synth_spec_t *s, const tdesc *x, uint16_t *dst) {
    const size_t n = numel(x);
    if (x->kind == G_ONE || x->kind == G_ZERO) {
        for (size_t i = 0; i < n; ++i) dst[i] = x->kind == G_ONE ? 0x3f80 : 0;
        return;
    }
    const uint64_t key = mix(s->seed) ^ name_hash(x->name);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (long long i = 0; i < (long long)n; ++i) dst[i] = to_bf16((float)(s->weight_std * gauss(key, (uint64_t)i)));
    if (x->kind == G_JBIAS) dst[s->vocab_size] = to_bf16(from_bf16(dst[s->vocab_size]) + s->blank_bias);
}

/* growable text buffer */
typedef struct { char *p; size_t n, cap; } sbuf;
static void put(sbuf *b, const char *fmt, ...) {
    for (;;) {
        va_list ap;
        va_start(ap, fmt);
        const int k = vsnprintf(b->p ? b->p + b->n : NULL, b->p ? b->cap - b->n : 0, fmt, ap);
        va_end(ap);
        if (b->p && k >= 0 && (size_t)k < b->cap - b->n) { b->n += (size_t)k; return; }
        b->cap = (b->cap + (size_t)(k > 0 ? k : 64) + 1) * 2;
        b->p = realloc(b->p, b->cap);
    }
}

static void config_json(const or_synth_spec_t *s, sbuf *b) {
    const int a = s->att_left;
    put(b, "{\n \"encoder\": {\"feat_in\": 128, \"n_layers\": %d, \"d_model\": %d, \"n_heads\": %d, \"ff_expansion_factor\": %d, "
           "\"subsampling_factor\": 8, \"subsampling_conv_channels\": %d, \"conv_kernel_size\": 9, "
           "\"att_context_size\": [[%d, 13], [%d, 6], [%d, 3], [%d, 1], [%d, 0]]},\n",
        s->n_layers, s->d_model, s->d_model / 128, s->ff_factor, s->sub_channels, a, a, a, a, a);
    put(b, " \"preprocessor\": {\"sample_rate\": 16000, \"features\": 128},\n");
    put(b, " \"prompt\": {\"num_prompts\": %d, \"prompt_hidden\": %d, \"prompt_dictionary\": {\"auto\": 0", s->num_prompts, s->prompt_hidden);
    if (s->num_prompts > 1) put(b, ", \"en-US\": 1");
    for (int i = 2; i < s->num_prompts; ++i) put(b, ", \"lang%d\": %d", i, i);
    put(b, "}},\n \"decoder\": {\"pred_hidden\": %d, \"pred_rnn_layers\": 2, \"vocab_size\": %d},\n", s->pred_hidden, s->vocab_size);
    put(b, " \"joint\": {\"joint_hidden\": %d, \"num_classes\": %d},\n", s->joint_hidden, s->vocab_size);
    put(b, " \"max_symbols\": 10,\n \"default_att_context_size\": [%d, 13],\n \"vocabulary\": [\"<unk>\"", a);
    for (int i = 1; i < s->vocab_size; ++i) put(b, ", \"\xe2\x96\x81tok%d\"", i);
    put(b, "]\n}\n");
}

int or_synth_write(const char *dir, const or_synth_spec_t *s, char *err, size_t errlen) {
    if (mkdir(dir, 0755) != 0 && errno != EEXIST) { snprintf(err, errlen, "cannot create %s", dir); return -1; }
    char path[4096];
    sbuf cfg = { 0 };
    config_json(s, &cfg);
    snprintf(path, sizeof path, "%s/config.json", dir);
    FILE *f = fopen(path, "wb");
    if (!f) { free(cfg.p); snprintf(err, errlen, "cannot write %s", path); return -1; }
    fwrite(cfg.p, 1, cfg.n, f);
    fclose(f);
    free(cfg.p);

    ttab tb = tensors(s);
    sbuf h = { 0 };
    put(&h, "{\"__metadata__\": {\"format\": \"pt\"}");
    size_t off = 0;
    for (int i = 0; i < tb.n; ++i) {
        const tdesc *x = &tb.t[i];
        put(&h, ", \"%s\": {\"dtype\": \"BF16\", \"shape\": [", x->name);
        for (int d = 0; d < x->ndim; ++d) put(&h, "%s%lld", d ? ", " : "", x->dim[d]);
        put(&h, "], \"data_offsets\": [%zu, %zu]}", off, off + numel(x) * 2);
        off += numel(x) * 2;
    }
    put(&h, "}");
    while (h.n % 8) put(&h, " ");
    snprintf(path, sizeof path, "%s/model.safetensors", dir);
    f = fopen(path, "wb");
    int rc = f ? 0 : -1;
    if (f) {
        const uint64_t hl = h.n;
        rc |= fwrite(&hl, 8, 1, f) != 1 || fwrite(h.p, 1, h.n, f) != h.n;
        for (int i = 0; i < tb.n && !rc; ++i) {
            const size_t n = numel(&tb.t[i]);
            uint16_t *buf = malloc(n * 2);
            fill(s, &tb.t[i], buf);
            rc |= fwrite(buf, 2, n, f) != n;
            free(buf);
        }
        rc |= fclose(f) != 0;
    }
    free(h.p);
    free(tb.t);
    if (rc) snprintf(err, errlen, "failed writing %s", path);
    return rc ? -1 : 0;
}

/* Three chirps sweeping 100 -> 4000 Hz with sawtooth frequency over periods 1.0, 1.7 and 2.9 s
   (phases 0, 2pi/3, 4pi/3; amplitude 0.15 each) plus N(0, 0.05^2) noise; with pauses, speech
   segments of U[1,3] s alternate with silences (chirps muted) of U[0.2,0.6] s. */
void or_synth_audio(uint64_t seed, int rate, size_t n, int pauses, float *out) {
    static const double period[3] = { 1.0, 1.7, 2.9 }, phase0[3] = { 0.0, 2.0943951023931953, 4.1887902047863905 };
    const uint64_t nkey = mix(seed ^ 0x6e6f697365ull), pkey = mix(seed ^ 0x7061757365ull);
    const double inv53 = 1.0 / 9007199254740992.0;
    uint64_t seg = 0;
    double seg_end = 0.0, gap_end = 0.0;
    if (pauses) {
        seg_end = 1.0 + 2.0 * ((double)(mix(pkey) >> 11) * inv53);
        gap_end = seg_end + 0.2 + 0.4 * ((double)(mix(pkey + 1) >> 11) * inv53);
    }
    for (size_t i = 0; i < n; ++i) {
        const double t = (double)i / rate;
        double amp = 1.0;
        if (pauses) {
            while (t >= gap_end) {
                ++seg;
                seg_end = gap_end + 1.0 + 2.0 * ((double)(mix(pkey + 2 * seg) >> 11) * inv53);
                gap_end = seg_end + 0.2 + 0.4 * ((double)(mix(pkey + 2 * seg + 1) >> 11) * inv53);
            }
            if (t >= seg_end) amp = 0.0;
        }
        double acc = 0.0;
        for (int k = 0; k < 3; ++k) {
            const double q = t / period[k], whole = floor(q), fr = q - whole;
            acc += 0.15 * sin(6.283185307179586 * (100.0 * t + 3900.0 * period[k] * (0.5 * whole + 0.5 * fr * fr)) + phase0[k]);
        }
        out[i] = (float)(amp * acc + 0.05 * gauss(nkey, (uint64_t)i));
    }
}
