/* Weights into one HBM arena, the per-layer rel-pos table, language prompt folding, vocabulary.
   Same tensors, shapes and conversions as src/model.c:185-322. */
#include "model.h"
#include <cuda_runtime_api.h>
#include <ctype.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ALIGN 256

static void *arena_take(nb_model_t *m, size_t bytes) {
    size_t off = (m->arena_used + ALIGN - 1) & ~(size_t)(ALIGN - 1);
    if (off + bytes > m->arena_bytes) return NULL;
    m->arena_used = off + bytes;
    return (char *)m->arena + off;
}

typedef struct { nb_model_t *m; nb_source_t *src; char *err; size_t errlen; uint16_t *tmp; size_t tmp_n; float *ftmp; int failed; } ld_t;

static uint16_t *host_bf16(ld_t *L, const char *name, size_t numel) {
    if (L->failed) return NULL;
    if (numel > L->tmp_n) {
        free(L->tmp);
        L->tmp = malloc(numel * 2);
        L->tmp_n = numel;
    }
    if (nb_source_bf16(L->src, name, numel, L->tmp, L->err, L->errlen)) { L->failed = 1; return NULL; }
    return L->tmp;
}
static uint16_t *dev_bf16(ld_t *L, const char *name, size_t numel) {
    uint16_t *h = host_bf16(L, name, numel);
    if (!h) return NULL;
    uint16_t *d = arena_take(L->m, numel * 2);
    if (!d) { snprintf(L->err, L->errlen, "weight arena overflow at %s", name); L->failed = 1; return NULL; }
    if (cudaMemcpy(d, h, numel * 2, cudaMemcpyHostToDevice) != cudaSuccess) { snprintf(L->err, L->errlen, "upload %s failed", name); L->failed = 1; return NULL; }
    return d;
}
static float *dev_f32(ld_t *L, const char *name, size_t numel) {
    uint16_t *h = host_bf16(L, name, numel);
    if (!h) return NULL;
    float *f = malloc(numel * sizeof(float));
    for (size_t i = 0; i < numel; ++i) f[i] = nb_bf16_to_f32(h[i]);
    float *d = arena_take(L->m, numel * sizeof(float));
    int ok = d && cudaMemcpy(d, f, numel * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess;
    free(f);
    if (!ok) { snprintf(L->err, L->errlen, "upload %s failed", name); L->failed = 1; return NULL; }
    return d;
}

/* Upper bound of the arena: all bf16 weights once, fp32 tensors twice their bf16 size, ptab. */
static size_t arena_estimate(const nb_config_t *g) {
    const size_t D = (size_t)g->d_model, FF = (size_t)g->d_ff, CH = (size_t)g->sub_channels, PH = (size_t)g->pred_hidden;
    const size_t JH = (size_t)g->joint_hidden, V = (size_t)g->vocab_size + 1, PRH = (size_t)g->prompt_hidden, NP = (size_t)g->num_prompts;
    const size_t P = 2 * (size_t)g->Lmax - 1;
    size_t b = 0;
    b += 4 * CH * 9 * 4 + 4 * CH * 4 + 2 * CH * CH * 2 + D * CH * (size_t)g->sub_freq_out * 2 + D * 4;
    size_t per = 4 * FF * D * 2 + 3 * D * D * 2 + D * D * 2 + 2 * D * D * 2 + D * D * 2;
    per += 12 * D * 4 + D * 9 * 4 + 2 * D * 4 + P * D * 4;
    b += (size_t)g->n_layers * (per + 32 * ALIGN);
    b += PRH * (D + NP) * 2 + D * PRH * 2 + D * 4;
    b += 2 * (4 * PH * 2 * PH * 2 + 4 * PH * 4) + V * PH * 2;
    b += JH * D * 2 + JH * 4 + JH * PH * 2 + JH * 4 + V * JH * 2 + V * 4;
    return b + 64 * ALIGN;
}

static char *xstrdup(const char *s) { size_t n = strlen(s) + 1; char *d = malloc(n); memcpy(d, s, n); return d; }

nb_model_t *nb_model_load(nb_source_t *src, char *err, size_t errlen) {
    const double t0 = nb_now_ms();
    nb_model_t *m = calloc(1, sizeof *m);
    if (nb_parse_config(nb_source_config(src), &m->g, err, errlen)) { free(m); return NULL; }
    const nb_config_t *g = &m->g;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) { snprintf(err, errlen, "no CUDA device (this build runs only on B200 GPUs)"); free(m); return NULL; }
    cudaGetDevice(&m->device);
    struct cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, m->device);
    snprintf(m->gpu_name, sizeof m->gpu_name, "%s", prop.name);
    if (prop.major != 10) { snprintf(err, errlen, "%s is sm_%d%d; this build is compiled for sm_100a (B200) only", prop.name, prop.major, prop.minor); free(m); return NULL; }
    m->arena_bytes = arena_estimate(g);
    if (cudaMalloc(&m->arena, m->arena_bytes) != cudaSuccess) { snprintf(err, errlen, "cannot allocate %zu MB weight arena", m->arena_bytes >> 20); free(m); return NULL; }
    ld_t L = { m, src, err, errlen, NULL, 0, NULL, 0 };
    const size_t D = (size_t)g->d_model, CH = (size_t)g->sub_channels, FF = (size_t)g->d_ff, PH = (size_t)g->pred_hidden;
    const size_t JH = (size_t)g->joint_hidden, PRH = (size_t)g->prompt_hidden, NP = (size_t)g->num_prompts;
    m->conv0_w = dev_f32(&L, "encoder.pre_encode.conv.0.weight", CH * 9);
    m->conv0_b = dev_f32(&L, "encoder.pre_encode.conv.0.bias", CH);
    m->conv2_w = dev_f32(&L, "encoder.pre_encode.conv.2.weight", CH * 9);
    m->conv2_b = dev_f32(&L, "encoder.pre_encode.conv.2.bias", CH);
    m->conv3_w = dev_bf16(&L, "encoder.pre_encode.conv.3.weight", CH * CH);
    m->conv3_b = dev_f32(&L, "encoder.pre_encode.conv.3.bias", CH);
    m->conv5_w = dev_f32(&L, "encoder.pre_encode.conv.5.weight", CH * 9);
    m->conv5_b = dev_f32(&L, "encoder.pre_encode.conv.5.bias", CH);
    m->conv6_w = dev_bf16(&L, "encoder.pre_encode.conv.6.weight", CH * CH);
    m->conv6_b = dev_f32(&L, "encoder.pre_encode.conv.6.bias", CH);
    m->pre_out_w = dev_bf16(&L, "encoder.pre_encode.out.weight", D * CH * (size_t)g->sub_freq_out);
    m->pre_out_b = dev_f32(&L, "encoder.pre_encode.out.bias", D);
    m->L = calloc((size_t)g->n_layers, sizeof *m->L);
    char nm[160];
    for (int l = 0; l < g->n_layers && !L.failed; ++l) {
        nb_layer_t *Y = &m->L[l];
#define LB(f, s, n) do { snprintf(nm, sizeof nm, "encoder.layers.%d.%s", l, s); Y->f = dev_bf16(&L, nm, n); } while (0)
#define LF(f, s, n) do { snprintf(nm, sizeof nm, "encoder.layers.%d.%s", l, s); Y->f = dev_f32(&L, nm, n); } while (0)
        LB(ff1_w1, "feed_forward1.linear1.weight", FF * D);
        LB(ff1_w2, "feed_forward1.linear2.weight", FF * D);
        LB(ff2_w1, "feed_forward2.linear1.weight", FF * D);
        LB(ff2_w2, "feed_forward2.linear2.weight", FF * D);
        /* q, k, v back to back: one [3D][D] matrix (src/model.c:240-242) */
        Y->wqkv = arena_take(m, 3 * D * D * 2);
        if (!Y->wqkv) { snprintf(err, errlen, "weight arena overflow"); L.failed = 1; break; }
        const char *qkv[3] = { "self_attn.linear_q.weight", "self_attn.linear_k.weight", "self_attn.linear_v.weight" };
        for (int i = 0; i < 3 && !L.failed; ++i) {
            snprintf(nm, sizeof nm, "encoder.layers.%d.%s", l, qkv[i]);
            uint16_t *h = host_bf16(&L, nm, D * D);
            if (h && cudaMemcpy(Y->wqkv + (size_t)i * D * D, h, D * D * 2, cudaMemcpyHostToDevice) != cudaSuccess) L.failed = 1;
        }
        LB(wo, "self_attn.linear_out.weight", D * D);
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
    /* prompt: W0 keeps its [PH][D + NP] layout (the GEMM reads the first D columns with
       ldw = D + NP, as src/encoder.c:191); the one-hot columns and b0 stay on the host. */
    m->prompt_w0 = dev_bf16(&L, "prompt_kernel.0.weight", PRH * (D + NP));
    if (!L.failed) {
        m->prompt_onehot_host = malloc(PRH * NP * 2);
        for (size_t n = 0; n < PRH; ++n) memcpy(m->prompt_onehot_host + n * NP, L.tmp + n * (D + NP) + D, NP * 2);
    }
    uint16_t *b0 = host_bf16(&L, "prompt_kernel.0.bias", PRH);
    if (b0) { m->prompt_b0_host = malloc(PRH * 2); memcpy(m->prompt_b0_host, b0, PRH * 2); }
    m->prompt_w2 = dev_bf16(&L, "prompt_kernel.2.weight", D * PRH);
    m->prompt_b2 = dev_f32(&L, "prompt_kernel.2.bias", D);
    /* LSTM: [Wx | Wh] per gate row, so gates = W . [x ; h] + b in one GEMM */
    for (int l = 0; l < 2 && !L.failed; ++l) {
        uint16_t *cat = malloc(4 * PH * 2 * PH * 2);
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.Wx", l);
        uint16_t *h = host_bf16(&L, nm, 4 * PH * PH);
        if (h) for (size_t r = 0; r < 4 * PH; ++r) memcpy(cat + r * 2 * PH, h + r * PH, PH * 2);
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.Wh", l);
        h = host_bf16(&L, nm, 4 * PH * PH);
        if (h) for (size_t r = 0; r < 4 * PH; ++r) memcpy(cat + r * 2 * PH + PH, h + r * PH, PH * 2);
        m->lstm_w[l] = arena_take(m, 4 * PH * 2 * PH * 2);
        if (!L.failed && (!m->lstm_w[l] || cudaMemcpy(m->lstm_w[l], cat, 4 * PH * 2 * PH * 2, cudaMemcpyHostToDevice) != cudaSuccess)) {
            snprintf(err, errlen, "upload LSTM %d failed", l);
            L.failed = 1;
        }
        free(cat);
        snprintf(nm, sizeof nm, "decoder.prediction.dec_rnn.lstm.%d.bias", l);
        m->lstm_b[l] = dev_f32(&L, nm, 4 * PH);
    }
    m->embed = dev_bf16(&L, "decoder.prediction.embed.weight", (size_t)(g->vocab_size + 1) * PH);
    m->joint_enc_w = dev_bf16(&L, "joint.enc.weight", JH * D);
    m->joint_enc_b = dev_f32(&L, "joint.enc.bias", JH);
    m->joint_pred_w = dev_bf16(&L, "joint.pred.weight", JH * PH);
    m->joint_pred_b = dev_f32(&L, "joint.pred.bias", JH);
    m->joint_out_w = dev_bf16(&L, "joint.joint_net.2.weight", (size_t)g->num_classes * JH);
    m->joint_out_b = dev_f32(&L, "joint.joint_net.2.bias", (size_t)g->num_classes);
    free(L.tmp);
    if (L.failed) { nb_model_free(m); return NULL; }

    /* rel-pos table (src/model.c:286-306): pe row r <-> position Lmax-1-r in double, then
       ptab = pe . Wpos^T per layer on the GPU (no bias) */
    {
        const int P = 2 * g->Lmax - 1;
        float *pe = malloc((size_t)P * D * sizeof(float));
        for (int r = 0; r < P; ++r) {
            const double pos = (double)(g->Lmax - 1 - r);
            for (size_t i = 0; i < D / 2; ++i) {
                const double div = exp((double)(2 * i) * -(log(10000.0) / (double)D));
                pe[(size_t)r * D + 2 * i] = (float)sin(pos * div);
                pe[(size_t)r * D + 2 * i + 1] = (float)cos(pos * div);
            }
        }
        float *d_pe = NULL;
        uint16_t *d_wpos = NULL;
        int rc = cudaMalloc((void **)&d_pe, (size_t)P * D * sizeof(float)) != cudaSuccess || cudaMalloc((void **)&d_wpos, D * D * 2) != cudaSuccess;
        if (!rc) rc = cudaMemcpy(d_pe, pe, (size_t)P * D * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess;
        for (int l = 0; l < g->n_layers && !rc; ++l) {
            snprintf(nm, sizeof nm, "encoder.layers.%d.self_attn.linear_pos.weight", l);
            L.tmp = NULL; L.tmp_n = 0;
            uint16_t *h = host_bf16(&L, nm, D * D);
            if (!h) { rc = 1; break; }
            rc = cudaMemcpy(d_wpos, h, D * D * 2, cudaMemcpyHostToDevice) != cudaSuccess;
            free(L.tmp);
            m->L[l].ptab = arena_take(m, (size_t)P * D * sizeof(float));
            if (rc || !m->L[l].ptab) { rc = 1; break; }
            nemo_gemm_args_t a = { 0 };
            a.A = d_pe; a.lda = (int64_t)D; a.a_fmt = NEMO_FMT_F32;
            a.W = d_wpos; a.ldw = (int64_t)D;
            a.C = m->L[l].ptab; a.ldc = (int64_t)D; a.c_fmt = NEMO_FMT_F32;
            a.M = P; a.N = (int)D; a.K = (int)D; a.alpha = 1.0f;
            if (nemo_gemm(&a, NULL)) { snprintf(err, errlen, "ptab: %s", nemo_gpu_last_error()); rc = 1; break; }
            rc = cudaDeviceSynchronize() != cudaSuccess;
        }
        cudaFree(d_pe);
        cudaFree(d_wpos);
        free(pe);
        if (rc) {
            if (!err[0]) snprintf(err, errlen, "rel-pos table build failed: %s", cudaGetErrorString(cudaGetLastError()));
            nb_model_free(m);
            return NULL;
        }
    }

    /* vocabulary and prompt dictionary */
    const nbj_t *cfg = nb_source_config(src);
    const nbj_t *voc = nbj_get(cfg, "vocabulary");
    m->n_pieces = (int)nbj_len(voc);
    m->pieces = calloc((size_t)m->n_pieces + 1, sizeof *m->pieces);
    for (int i = 0; i < m->n_pieces; ++i) m->pieces[i] = xstrdup(nbj_str(nbj_at(voc, (size_t)i), ""));
    const nbj_t *pd = nbj_get(nbj_get(cfg, "prompt"), "prompt_dictionary");
    m->n_lang = (int)nbj_len(pd);
    m->lang_keys = calloc((size_t)m->n_lang + 1, sizeof *m->lang_keys);
    m->lang_idx = calloc((size_t)m->n_lang + 1, sizeof *m->lang_idx);
    for (int i = 0; i < m->n_lang; ++i) {
        m->lang_keys[i] = xstrdup(pd->keys[i]);
        m->lang_idx[i] = (int)nbj_num(pd->items[i], -1);
    }
    m->load_ms = nb_now_ms() - t0;
    return m;
}

void nb_model_free(nb_model_t *m) {
    if (!m) return;
    if (m->arena) cudaFree(m->arena);
    if (m->enc1_image) cudaFree(m->enc1_image);
    if (m->enc1_fold) cudaFree(m->enc1_fold);
    free(m->L);
    free(m->prompt_b0_host);
    free(m->prompt_onehot_host);
    for (int i = 0; i < m->n_pieces; ++i) free(m->pieces[i]);
    free(m->pieces);
    for (int i = 0; i < m->n_lang; ++i) free(m->lang_keys[i]);
    free(m->lang_keys);
    free(m->lang_idx);
    free(m);
}

int nb_model_prompt_index(const nb_model_t *m, const char *lang) {
    for (int i = 0; i < m->n_lang; ++i) if (!strcmp(m->lang_keys[i], lang)) return m->lang_idx[i];
    return -1;
}

void nb_model_prompt_bias(const nb_model_t *m, int idx, float *out) {
    const int NP = m->g.num_prompts;
    for (int n = 0; n < m->g.prompt_hidden; ++n)
        out[n] = nb_bf16_to_f32(m->prompt_b0_host[n]) + nb_bf16_to_f32(m->prompt_onehot_host[(size_t)n * NP + idx]);
}

int nb_model_right_trained(const nb_model_t *m, int right) {
    for (int i = 0; i < m->g.n_trained; ++i) if (m->g.trained_right[i] == right) return 1;
    return 0;
}

/* <unk> <pad> <s> </s> and <xx-YY> language tags produce no text (src/tokenizer.c:19-33) */
static int is_lang_tag(const char *p) {
    const size_t n = strlen(p);
    if (n < 7 || p[0] != '<' || p[n - 1] != '>') return 0;
    const char *dash = strchr(p, '-');
    if (!dash) return 0;
    const size_t a = (size_t)(dash - p) - 1, b = n - 2 - a - 1;
    if (a < 2 || a > 3 || b < 2 || b > 4) return 0;
    for (size_t i = 1; i < 1 + a; ++i) if (!islower((unsigned char)p[i])) return 0;
    for (size_t i = (size_t)(dash - p) + 1; i < n - 1; ++i) if (!isalpha((unsigned char)p[i])) return 0;
    return 1;
}
char *nb_model_token_text(const nb_model_t *m, int id) {
    if (id < 0 || id >= m->n_pieces) return xstrdup("");
    const char *p = m->pieces[id];
    if (!strcmp(p, "<unk>") || !strcmp(p, "<pad>") || !strcmp(p, "<s>") || !strcmp(p, "</s>") || is_lang_tag(p)) return xstrdup("");
    const size_t n = strlen(p);
    char *out = malloc(n + 1);
    size_t o = 0;
    for (size_t i = 0; i < n;) {
        if (i + 2 < n && (unsigned char)p[i] == 0xE2 && (unsigned char)p[i + 1] == 0x96 && (unsigned char)p[i + 2] == 0x81) { out[o++] = ' '; i += 3; }
        else out[o++] = p[i++];
    }
    out[o] = 0;
    return out;
}
