/* Streaming engine: host bookkeeping of src/encoder.c / src/decoder.c for B lockstep streams,
   device buffers laid out [stream][row][...], and the per-chunk launch sequence. */
#include "engine.h"
#include "engine_dev.h"
#include <cuda_runtime_api.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define NB_MAX_GRAPHS 512
#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { snprintf(err, errlen, "%s: %s", #x, cudaGetErrorString(e_)); goto fail; } } while (0)
#define KL(x) do { if ((x) != 0) { snprintf(err, errlen, "%s", nemo_gpu_last_error()); return -1; } } while (0)

struct nb_engine {
    nb_model_t *m;
    int B, right, chunk_frames, chunk_mel, cmax, left, conv_left, Lmax, cap_rows, nwin_max;
    int fmt_layer, fmt_conv;   /* activation format feeding the GEMMs (fp32 or bf16 hi/lo planes) */
    cudaStream_t st;
    /* host bookkeeping (identical for every stream: they are fed in lockstep) */
    float **pending;
    size_t pending_n, pending_cap;
    float *mel_cache;          /* [B][16][128] */
    int mel_cache_n;
    size_t consumed, emitted;
    int closed, pos, cache_len;
    /* optional device-resident mel source [B][sstride] (frames of 128 floats), replacing the
       host queue: the window of every step is then a device-to-device 2D copy */
    const float *dev_mel;
    int64_t dev_mel_sstride;
    size_t dev_mel_frames;
    /* log-mel on the GPU (NEMO_HOST_MEL=1 keeps it on the host): each stream's sample span is
       staged in pinned memory, the frames go to a device queue the windows are read from */
    int use_gpu_mel;
    float *h_span, *d_span;    /* [B][span_cap] */
    size_t span_cap;
    float *d_melq;             /* [B][qcap][128] */
    size_t qcap, q_base, q_end; /* absolute frame index of queue row 0; frames produced */
    cudaEvent_t span_ev;       /* the last span upload has been read */
    /* GPU resampler (input rates other than 16 kHz): each stream's input FIFO staged in pinned
       memory, the outputs come back to pinned memory for the mel bookkeeping */
    float *h_rs_in, *d_rs_in, *d_rs_out, *h_rs_out;  /* [B][rs_in_cap], [B][rs_out_cap] */
    size_t rs_in_cap, rs_out_cap;
    /* device */
    float *d_win, *h_win;      /* [B][nwin_max][128]; h_win pinned */
    float *c0, *c1, *c2, *c3, *c4, *flat;
    float *hbuf[2], *xin, *ff, *att, *y, *ph, *prompted, *prompted_x, *joint_enc;
    float *kv, *din;           /* [layers][B][cap_rows][3D] and [layers][B][cap_rows][D] */
    float *b_eff;              /* [B][PH] */
    int *d_params, *h_params;  /* pos, cache_len, lo */
    DecState dec;
    int *h_cnt, *h_ntok, *h_tokens;
    int *prompt_idx;
    /* taps */
    float *tap_prompted, *tap_joint;
    size_t tap_cap, tap_rows;
    int *tap_chunk_rows;
    size_t tap_chunk_cap, tap_chunks;
    double enc_ms, dec_ms, gpu_ms;
    size_t chunks;
    long long frames_decoded, dec_iterations;  /* since reset: stream-frames decoded, greedy loop iterations */
    cudaEvent_t ev0, ev1, ev_mid;  /* step start, step end, encoder done */
    int dec_pending_slot, dec_pending_max_it;  /* decoder graph launched, its counters not read yet */
    /* captured CUDA graphs: encoder step per (window rows, chunk rows), decoder iteration per
       chunk rows; NEMO_GRAPHS=0 launches kernel by kernel instead */
    int use_graphs;
    /* one stream: the conformer blocks run as one persistent kernel (NEMO_PERSISTENT=0 disables) */
    int use_enc1, enc1_grid, enc1_optin;
    int enc1_tail;             /* the prompt and joint encoder projections run as the launch's last stages */
    NbEnc1Layer *enc1_layers;  /* host copy, passed by value at each launch */
    uint8_t *enc1_image;       /* the model's weights laid out per CTA of the persistent grid (owned by the model) */
    float *enc1_fold;          /* and its LayerNorm fold constants (owned by the model) */
    NbEnc1Args enc1_args;      /* launch arguments (large: the layer table travels by value) */
    /* one stream: the greedy loop of a chunk runs as one persistent kernel (NEMO_PERSISTENT=0 disables) */
    int use_dec1, dec1_grid;
    float *d_dec1;             /* H0 [2][PH] | H1 [2][PH] | PRED [JH] | part_v [16][grid] */
    int *d_dec1_i;             /* part_i [16][grid] | err */
    unsigned *d_dec1_bar;
    /* several streams: the greedy loop as four tensor-core GEMMs with decoder epilogues and one
       step kernel per iteration (NEMO_DEC_FUSED=0 keeps the kernel-by-kernel iteration) */
    int dec_fused;
    int dec_unroll;              /* greedy iterations per pass of the decoder graph's WHILE body */
    uint16_t *dec_wg1;           /* [8PH][PH]: gate-interleaved W1x rows, then W0h rows */
    uint16_t *dec_wg2;           /* [JH + 4PH][PH]: Wp rows, then gate-interleaved W1h rows */
    float *dec_b1i;              /* interleaved b1 */
    float *dec_table;            /* [vocab + 1][4PH]: b0 + W0x . embed[v], interleaved */
    float *dec_r0, *dec_r1;      /* [B][4PH]: W0h . h0 and b1 + W1h . h1 of each stream's committed state */
    float *dec_pv;               /* [B][dec_np]: joint argmax partials (value, column) per column tile half */
    int *dec_pi, dec_np;
    unsigned *d_enc1_bar;
    int *d_enc1_err;
    struct { int kind, k1, k2; cudaGraphExec_t exec; uint64_t kernels; } graphs[NB_MAX_GRAPHS];
    int ngraphs;
};

uint64_t nb_graph_kernel_nodes(cudaGraph_t g);

double nb_engine_gpu_ms(const nb_engine_t *e) { return e->gpu_ms; }

static int sub_len(int n) { return n / 2 + 1; }

static void *dalloc(size_t bytes, int *fail) {
    void *p = NULL;
    if (*fail) return NULL;
    if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) { *fail = 1; return NULL; }
    cudaMemset(p, 0, bytes ? bytes : 16);
    return p;
}

/* Row pitch of the joint logits: a multiple of 4 floats, so the GEMM epilogue stores 16 bytes at a time. */
static int logits_ld(const nb_config_t *g) { return (g->num_classes + 3) & ~3; }

/* One stream: prepare the persistent encoder kernel (every conformer block of a chunk in one
   launch) when the device and model shapes allow it; otherwise the blocks run kernel by kernel. */
static int enc1_setup(nb_engine_t *e, char *err, size_t errlen) {
    const char *ev = getenv("NEMO_PERSISTENT");
    if (ev && !strcmp(ev, "0")) return 0;
    const nb_model_t *m = e->m;
    const nb_config_t *g = &m->g;
    int dev = 0, sms = 0, optin = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    const int D = g->d_model, FF = g->d_ff;
    if (!coop || sms <= 0 || D % 128 || D > 1024 || g->n_heads * 128 != D || e->cmax > 16 || e->Lmax > 72 || g->n_layers > NB_ENC1_MAX_LAYERS ||
        g->conv_kernel > 9)
        return 0;
    /* per-CTA weight rows must fit the kernel's 32-row accumulator tiles and two of the largest
       entries its weight ring (0 otherwise) */
    const int ring = nb_encoder1_ring_bytes(D, FF, sms, (size_t)optin, e->cmax, e->left + e->cmax);  /* the largest chunk */
    if (!ring || nb_encoder1_smem(ring, e->cmax, e->left + e->cmax) > (size_t)optin) return 0;
    NbEnc1Layer *L = calloc((size_t)g->n_layers, sizeof *L);
    const size_t kv_s = (size_t)e->cap_rows * 3 * D, din_s = (size_t)e->cap_rows * D;
    for (int l = 0; l < g->n_layers; ++l) {
        const nb_layer_t *W = &m->L[l];
        NbEnc1Layer *o = &L[l];
        o->ff1_w1 = W->ff1_w1; o->ff1_w2 = W->ff1_w2; o->wqkv = W->wqkv; o->wo = W->wo; o->pw1 = W->pw1; o->pw2 = W->pw2;
        o->ff2_w1 = W->ff2_w1; o->ff2_w2 = W->ff2_w2;
        o->ln_ff1_g = W->ln_ff1_g; o->ln_ff1_b = W->ln_ff1_b; o->ln_att_g = W->ln_att_g; o->ln_att_b = W->ln_att_b;
        o->ln_conv_g = W->ln_conv_g; o->ln_conv_b = W->ln_conv_b; o->ln_ff2_g = W->ln_ff2_g; o->ln_ff2_b = W->ln_ff2_b;
        o->ln_out_g = W->ln_out_g; o->ln_out_b = W->ln_out_b;
        o->bn_g = W->bn_g; o->bn_b = W->bn_b; o->dw_w = W->dw_w; o->bias_u = W->bias_u; o->bias_v = W->bias_v; o->ptab = W->ptab;
        o->kv = e->kv + (size_t)l * kv_s;
        o->din = e->din + (size_t)l * din_s;
    }
    e->enc1_layers = L;
    /* the encoder's tail (prompt projections, joint encoder projection) as three more stages when
       its widths fit the stage shapes: K <= 1024 or a multiple of 1024, at most 32 rows per CTA */
    const int PRH = g->prompt_hidden, JH = g->joint_hidden, NP = g->num_prompts;
    const int tail = PRH % 128 == 0 && (PRH <= 1024 || PRH % 1024 == 0) && JH % 16 == 0 && (D + NP) % 8 == 0 && (PRH + sms - 1) / sms <= 32 &&
                     (JH + sms - 1) / sms <= 32 && (PRH <= 1024 || (D + sms / (PRH / 1024) - 1) / (sms / (PRH / 1024)) <= 32);
    /* the weights re-laid out in the order the persistent grid reads them (one bulk copy per CTA
       and projection), built once per model; without room for the copy the blocks run kernel by
       kernel */
    nb_model_t *mm = e->m;
    if (!mm->enc1_image || mm->enc1_grid != sms) {
        if (mm->enc1_image) cudaFree(mm->enc1_image);
        if (mm->enc1_fold) cudaFree(mm->enc1_fold);
        mm->enc1_image = NULL;
        mm->enc1_fold = NULL;
        mm->enc1_grid = 0;
        const size_t img = nb_encoder1_image_bytes(D, FF, g->n_layers) + (tail ? nb_encoder1_tail_image_bytes(D, PRH, JH) : 0),
                     fb = nb_encoder1_fold_bytes(D, FF, g->n_layers);
        if (cudaMalloc((void **)&mm->enc1_image, img) != cudaSuccess || cudaMalloc((void **)&mm->enc1_fold, fb) != cudaSuccess) {
            cudaGetLastError();
            if (mm->enc1_image) cudaFree(mm->enc1_image);
            mm->enc1_image = NULL;
            mm->enc1_fold = NULL;
            return 0;
        }
        NbEnc1Args *q = &e->enc1_args;
        memset(q, 0, sizeof *q);
        memcpy(q->L, L, (size_t)g->n_layers * sizeof *L);
        q->layers = g->n_layers; q->D = D; q->FF = FF;
        q->tail = tail; q->PRH = PRH; q->JH = JH; q->pw0_ld = D + NP;
        q->pw0 = m->prompt_w0; q->pw2 = m->prompt_w2; q->jw = m->joint_enc_w;
        if (nb_encoder1_repack(q, sms, mm->enc1_image, mm->enc1_fold, e->st) || cudaStreamSynchronize(e->st) != cudaSuccess) {
            snprintf(err, errlen, "persistent encoder set-up: %s", nemo_gpu_last_error());
            return -1;
        }
        mm->enc1_grid = sms;
    }
    e->enc1_image = mm->enc1_image;
    e->enc1_fold = mm->enc1_fold;
    const int rc = cudaMalloc((void **)&e->d_enc1_bar, 2 * sizeof(unsigned)) != cudaSuccess || cudaMalloc((void **)&e->d_enc1_err, sizeof(int)) != cudaSuccess ||
                   cudaMemset(e->d_enc1_err, 0, sizeof(int)) != cudaSuccess;
    if (rc) { snprintf(err, errlen, "persistent encoder set-up: %s", cudaGetErrorString(cudaGetLastError())); return -1; }
    e->use_enc1 = 1;
    e->enc1_tail = tail;
    e->enc1_grid = sms;
    e->enc1_optin = optin;
    return 0;
}

/* Several streams with bf16 hi/lo activations: the fused greedy iteration's weights (gate-
   interleaved, the recurrent halves appended to the GEMMs that read the same input), the
   per-token gate table of layer 0 and the per-stream recurrent gate parts. */
static int dec_fused_setup(nb_engine_t *e, char *err, size_t errlen) {
    const char *ev = getenv("NEMO_DEC_FUSED");
    if (ev && !strcmp(ev, "0")) return 0;
    const nb_model_t *m = e->m;
    const nb_config_t *g = &m->g;
    const size_t PH = (size_t)g->pred_hidden, JH = (size_t)g->joint_hidden, NV = (size_t)g->vocab_size + 1;
    if (g->pred_layers != 2 || PH % 16 || JH % 16 || g->num_classes > (int)NV || g->blank_id < 0 || g->blank_id >= (int)NV) return 0;
    if (nb_dec_joint_parts(g->num_classes) > 32) return 0;  /* the step kernel reduces the argmax partials within one warp */
    int fail = 0;
    uint16_t *w0i = dalloc(4 * PH * 2 * PH * 2, &fail), *w1i = dalloc(4 * PH * 2 * PH * 2, &fail);
    float *b0i = dalloc(4 * PH * 4, &fail);
    e->dec_b1i = dalloc(4 * PH * 4, &fail);
    e->dec_table = dalloc(NV * 4 * PH * 4, &fail);
    e->dec_wg1 = dalloc(8 * PH * PH * 2, &fail);
    e->dec_wg2 = dalloc((JH + 4 * PH) * PH * 2, &fail);
    e->dec_r0 = dalloc((size_t)e->B * 4 * PH * 4, &fail);
    e->dec_r1 = dalloc((size_t)e->B * 4 * PH * 4, &fail);
    e->dec_np = nb_dec_joint_parts(g->num_classes);
    e->dec_pv = dalloc((size_t)e->B * e->dec_np * 4, &fail);
    e->dec_pi = dalloc((size_t)e->B * e->dec_np * 4, &fail);
    int rc = fail ? -1 : 0;
    const size_t row = PH * 2;  /* bytes of PH bf16 */
    if (!rc)
        rc = nb_dec_interleave(m->lstm_w[0], w0i, m->lstm_b[0], b0i, (int)PH, (int)(2 * PH), e->st) ||
             nb_dec_interleave(m->lstm_w[1], w1i, m->lstm_b[1], e->dec_b1i, (int)PH, (int)(2 * PH), e->st) ||
             nb_dec_gate_table(w0i, (int64_t)(2 * PH), m->embed, (int)NV, (int)PH, b0i, g->blank_id, e->dec_table, e->st) ||
             cudaMemcpy2DAsync(e->dec_wg1, row, w1i, 2 * row, row, 4 * PH, cudaMemcpyDeviceToDevice, e->st) != cudaSuccess ||
             cudaMemcpy2DAsync(e->dec_wg1 + 4 * PH * PH, row, w0i + PH, 2 * row, row, 4 * PH, cudaMemcpyDeviceToDevice, e->st) != cudaSuccess ||
             cudaMemcpyAsync(e->dec_wg2, m->joint_pred_w, JH * row, cudaMemcpyDeviceToDevice, e->st) != cudaSuccess ||
             cudaMemcpy2DAsync(e->dec_wg2 + JH * PH, row, w1i + PH, 2 * row, row, 4 * PH, cudaMemcpyDeviceToDevice, e->st) != cudaSuccess ||
             cudaStreamSynchronize(e->st) != cudaSuccess;
    if (w0i) cudaFree(w0i);
    if (w1i) cudaFree(w1i);
    if (b0i) cudaFree(b0i);
    if (rc) {
        snprintf(err, errlen, "decoder tables: %s", fail ? "out of device memory" : nemo_gpu_last_error());
        return -1;
    }
    e->dec_fused = 1;
    return 0;
}

/* One stream: prepare the persistent greedy decoder when the model's shapes fit it. */
static int dec1_setup(nb_engine_t *e, char *err, size_t errlen) {
    const char *ev = getenv("NEMO_PERSISTENT");
    if (ev && !strcmp(ev, "0")) return 0;
    const nb_config_t *g = &e->m->g;
    int dev = 0, sms = 0, optin = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    if (!coop || sms <= 0 || g->pred_layers != 2 || !nb_decoder1_fits(g->pred_hidden, g->joint_hidden, g->num_classes, sms, e->cmax, (size_t)optin))
        return 0;
    const size_t PH = (size_t)g->pred_hidden, JH = (size_t)g->joint_hidden;
    if (cudaMalloc((void **)&e->d_dec1, (4 * PH + 4 * PH + JH + (size_t)sms * 16) * sizeof(float)) != cudaSuccess ||
        cudaMalloc((void **)&e->d_dec1_i, ((size_t)sms * 16 + 1) * sizeof(int)) != cudaSuccess ||
        cudaMalloc((void **)&e->d_dec1_bar, 2 * sizeof(unsigned)) != cudaSuccess || cudaMemset(e->d_dec1_i, 0, ((size_t)sms * 16 + 1) * sizeof(int)) != cudaSuccess) {
        snprintf(err, errlen, "persistent decoder set-up: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    e->use_dec1 = 1;
    e->dec1_grid = sms;
    return 0;
}

nb_engine_t *nb_engine_create(nb_model_t *m, int B, int right, char *err, size_t errlen) {
    if (B <= 0) { snprintf(err, errlen, "stream count must be positive"); return NULL; }
    nb_engine_t *e = calloc(1, sizeof *e);
    const nb_config_t *g = &m->g;
    e->m = m;
    e->B = B;
    e->right = right;
    e->chunk_frames = right + 1;
    e->chunk_mel = e->chunk_frames * g->subsampling;
    e->cmax = e->chunk_frames + 2;                  /* final boundary window (src/encoder.c:45) */
    if (e->cmax < NB_MIN_CMAX) e->cmax = NB_MIN_CMAX;
    e->left = g->att_left;
    e->Lmax = g->Lmax;
    e->conv_left = g->conv_kernel - 1;
    e->cap_rows = e->left + NB_EPOCH_CHUNKS * e->cmax; /* src/encoder.c:73 */
    e->nwin_max = NB_MEL_CACHE + e->chunk_mel + 1;
    /* GEMM inputs travel as bf16 hi/lo planes into the tensor-core kernel; NEMO_GEMM=cuda keeps
       them fp32 and routes every GEMM through the CUDA-core kernels instead */
    const char *gm = getenv("NEMO_GEMM");
    const int fmt = (gm && !strcmp(gm, "cuda")) ? NEMO_FMT_F32 : NEMO_FMT_BF16X2;
    e->fmt_layer = fmt;
    e->fmt_conv = fmt;
    if (e->left + e->cmax > 96) { snprintf(err, errlen, "attention window %d exceeds 96 rows", e->left + e->cmax); free(e); return NULL; }
    int fail = 0;
    const size_t D = (size_t)g->d_model, CH = (size_t)g->sub_channels, FF = (size_t)g->d_ff, PH = (size_t)g->pred_hidden;
    const size_t JH = (size_t)g->joint_hidden, PRH = (size_t)g->prompt_hidden, Bz = (size_t)B, cm = (size_t)e->cmax;
    const size_t T1 = (size_t)sub_len(e->nwin_max), F1 = 128 / 2 + 1, T2 = T1 / 2 + 1, F2 = F1 / 2 + 1, T3 = T2 / 2 + 1, F3 = F2 / 2 + 1;
    CK(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));
    CK(cudaEventCreate(&e->ev0));
    CK(cudaEventCreate(&e->ev1));
    CK(cudaEventCreate(&e->ev_mid));
    e->dec_pending_slot = -1;
    e->d_win = dalloc(Bz * (size_t)e->nwin_max * 128 * 4, &fail);
    CK(cudaMallocHost((void **)&e->h_win, Bz * (size_t)e->nwin_max * 128 * 4));
    e->c0 = NULL; /* the first subsampling stage is fused into the second (no [T1][F1][C] map) */
    (void)T1; (void)F1;
    e->c1 = dalloc(Bz * T2 * F2 * CH * 4, &fail);
    e->c2 = dalloc(Bz * T2 * F2 * CH * 4, &fail);
    e->c3 = dalloc(Bz * T3 * F3 * CH * 4, &fail);
    e->c4 = dalloc(Bz * T3 * F3 * CH * 4, &fail);
    e->flat = dalloc(Bz * cm * CH * F3 * 4, &fail);
    e->hbuf[0] = dalloc(Bz * cm * D * 4, &fail);
    e->hbuf[1] = dalloc(Bz * cm * D * 4, &fail);
    e->xin = dalloc(Bz * cm * D * 4, &fail);
    e->ff = dalloc(Bz * cm * FF * 4, &fail);
    e->att = dalloc(Bz * cm * D * 4, &fail);
    e->y = dalloc(Bz * cm * D * 4, &fail);
    e->ph = dalloc(Bz * cm * PRH * 4, &fail);
    e->prompted = dalloc(Bz * cm * D * 4, &fail);
    e->prompted_x = fmt == NEMO_FMT_F32 ? e->prompted : dalloc(Bz * cm * D * 4, &fail);
    e->joint_enc = dalloc(Bz * cm * JH * 4, &fail);
    e->kv = dalloc((size_t)g->n_layers * Bz * (size_t)e->cap_rows * 3 * D * 4, &fail);
    e->din = dalloc((size_t)g->n_layers * Bz * (size_t)e->cap_rows * D * 4, &fail);
    e->b_eff = dalloc(Bz * PRH * 4, &fail);
    e->d_params = dalloc(8 * sizeof(int), &fail);
    CK(cudaMallocHost((void **)&e->h_params, 8 * sizeof(int)));
    /* decoder state */
    DecState *d = &e->dec;
    d->streams = B;
    d->tok_cap = e->cmax * g->max_symbols;
    int **ints[] = { &d->t, &d->symbols, &d->active, &d->pred_valid, &d->last_token, &d->ntok, &d->need_idx, &d->need_pos, &d->erow, &d->idx };
    for (size_t i = 0; i < sizeof ints / sizeof *ints; ++i) *ints[i] = dalloc(Bz * sizeof(int), &fail);
    d->tokens = dalloc(Bz * (size_t)d->tok_cap * sizeof(int), &fail);
    d->cnt = dalloc(8 * sizeof(int), &fail);
    d->stats = dalloc(4 * sizeof(int), &fail);
    d->h = dalloc(2 * Bz * PH * 4, &fail);
    d->c = dalloc(2 * Bz * PH * 4, &fail);
    d->hp = dalloc(2 * Bz * PH * 4, &fail);
    d->cp = dalloc(2 * Bz * PH * 4, &fail);
    d->pred = dalloc(Bz * JH * 4, &fail);
    d->A0 = dalloc(Bz * 2 * PH * 4, &fail);
    d->A1 = dalloc(Bz * 2 * PH * 4, &fail);
    d->gates = dalloc(Bz * 4 * PH * 4, &fail);
    d->hp1c = dalloc(Bz * PH * 4, &fail);
    d->predc = dalloc(Bz * JH * 4, &fail);
    d->fmt = fmt;
    d->a_plane = (int64_t)Bz * 2 * PH;
    d->h_plane = (int64_t)Bz * PH;
    d->jx = dalloc(Bz * JH * 4, &fail);
    d->logits = dalloc(Bz * (size_t)logits_ld(g) * 4, &fail);
    if (fail) { snprintf(err, errlen, "out of device memory for %d streams", B); goto fail; }
    CK(cudaMallocHost((void **)&e->h_cnt, 8 * sizeof(int)));
    CK(cudaMallocHost((void **)&e->h_ntok, Bz * sizeof(int)));
    CK(cudaMallocHost((void **)&e->h_tokens, Bz * (size_t)d->tok_cap * sizeof(int)));
    e->pending = calloc(Bz, sizeof *e->pending);
    e->mel_cache = calloc(Bz * NB_MEL_CACHE * 128, sizeof(float));
    e->prompt_idx = calloc(Bz, sizeof(int));
    {
        float *be = malloc(PRH * 4);
        nb_model_prompt_bias(m, 0, be);
        for (int s = 0; s < B; ++s) CK(cudaMemcpy(e->b_eff + (size_t)s * PRH, be, PRH * 4, cudaMemcpyHostToDevice));
        free(be);
    }
    {
        const char *hm = getenv("NEMO_HOST_MEL");
        e->use_gpu_mel = !(hm && !strcmp(hm, "1"));
        if (e->use_gpu_mel) {
            e->span_cap = (size_t)(NB_SPAN_FRAMES - 1) * NB_MEL_HOP + NB_MEL_NFFT;
            e->qcap = 2 * ((size_t)e->chunk_mel + NB_MEL_CACHE + NB_SPAN_FRAMES) + 16;
            CK(cudaMallocHost((void **)&e->h_span, Bz * e->span_cap * sizeof(float)));
            CK(cudaEventCreateWithFlags(&e->span_ev, cudaEventDisableTiming));
            e->d_span = dalloc(Bz * e->span_cap * sizeof(float), &fail);
            e->d_melq = dalloc(Bz * e->qcap * 128 * sizeof(float), &fail);
            if (fail) { snprintf(err, errlen, "out of device memory for the mel queue of %d streams", B); goto fail; }
        }
    }
    if (nb_gemm_tc_init()) { snprintf(err, errlen, "%s", nemo_gpu_last_error()); goto fail; }
    {
        const char *gr = getenv("NEMO_GRAPHS");
        e->use_graphs = !(gr && !strcmp(gr, "0"));
    }
    if (B == 1 && fmt == NEMO_FMT_BF16X2 && enc1_setup(e, err, errlen)) goto fail;
    if (B == 1 && dec1_setup(e, err, errlen)) goto fail;
    if (B > 1 && fmt == NEMO_FMT_BF16X2 && dec_fused_setup(e, err, errlen)) goto fail;
    {
        /* iterations after the last active stream finished do no work but the joint GEMM; a few
           per WHILE pass amortise the conditional node's per-pass cost */
        const char *du = getenv("NEMO_DEC_UNROLL");
        e->dec_unroll = du ? atoi(du) : 4;
        if (e->dec_unroll < 1) e->dec_unroll = 1;
        if (e->dec_unroll > 16) e->dec_unroll = 16;
    }
    if (nb_engine_reset(e, err, errlen)) goto fail;
    return e;
fail:
    nb_engine_destroy(e);
    return NULL;
}

void nb_engine_destroy(nb_engine_t *e) {
    if (!e) return;
    if (e->st) cudaStreamSynchronize(e->st);
    float *f[] = { e->d_win, e->c0, e->c1, e->c2, e->c3, e->c4, e->flat, e->hbuf[0], e->hbuf[1], e->xin, e->ff, e->att, e->y, e->ph,
                   e->prompted, e->joint_enc, e->kv, e->din, e->b_eff, e->dec.h, e->dec.c, e->dec.hp, e->dec.cp, e->dec.pred, e->dec.A0,
                   e->dec.A1, e->dec.gates, e->dec.hp1c, e->dec.predc };
    for (size_t i = 0; i < sizeof f / sizeof *f; ++i) if (f[i]) cudaFree(f[i]);
    if (e->prompted_x && e->prompted_x != e->prompted) cudaFree(e->prompted_x);
    if (e->dec.jx) cudaFree(e->dec.jx);
    if (e->dec.logits) cudaFree(e->dec.logits);
    int *n[] = { e->d_params, e->dec.t, e->dec.symbols, e->dec.active, e->dec.pred_valid, e->dec.last_token, e->dec.ntok, e->dec.need_idx, e->dec.need_pos,
                 e->dec.erow, e->dec.idx, e->dec.tokens, e->dec.cnt, e->dec.stats };
    for (size_t i = 0; i < sizeof n / sizeof *n; ++i) if (n[i]) cudaFree(n[i]);
    if (e->h_win) cudaFreeHost(e->h_win);
    if (e->h_params) cudaFreeHost(e->h_params);
    if (e->h_cnt) cudaFreeHost(e->h_cnt);
    if (e->h_ntok) cudaFreeHost(e->h_ntok);
    if (e->h_tokens) cudaFreeHost(e->h_tokens);
    if (e->st) cudaStreamDestroy(e->st);
    if (e->ev0) cudaEventDestroy(e->ev0);
    if (e->ev1) cudaEventDestroy(e->ev1);
    if (e->ev_mid) cudaEventDestroy(e->ev_mid);
    for (int i = 0; i < e->ngraphs; ++i) cudaGraphExecDestroy(e->graphs[i].exec);
    free(e->enc1_layers);
    void *dt[] = { e->dec_wg1, e->dec_wg2, e->dec_b1i, e->dec_table, e->dec_r0, e->dec_r1, e->dec_pv, e->dec_pi };
    for (size_t i = 0; i < sizeof dt / sizeof *dt; ++i) if (dt[i]) cudaFree(dt[i]);
    if (e->h_span) cudaFreeHost(e->h_span);
    if (e->d_span) cudaFree(e->d_span);
    if (e->d_melq) cudaFree(e->d_melq);
    if (e->span_ev) cudaEventDestroy(e->span_ev);
    if (e->h_rs_in) cudaFreeHost(e->h_rs_in);
    if (e->h_rs_out) cudaFreeHost(e->h_rs_out);
    if (e->d_rs_in) cudaFree(e->d_rs_in);
    if (e->d_rs_out) cudaFree(e->d_rs_out);
    if (e->d_dec1) cudaFree(e->d_dec1);
    if (e->d_dec1_i) cudaFree(e->d_dec1_i);
    if (e->d_dec1_bar) cudaFree(e->d_dec1_bar);
    if (e->d_enc1_bar) cudaFree(e->d_enc1_bar);
    if (e->d_enc1_err) cudaFree(e->d_enc1_err);
    if (e->pending) for (int s = 0; s < e->B; ++s) free(e->pending[s]);
    free(e->pending);
    free(e->mel_cache);
    free(e->prompt_idx);
    free(e);
}

int nb_engine_reset(nb_engine_t *e, char *err, size_t errlen) {
    e->pending_n = 0;
    e->dev_mel = NULL;
    e->dev_mel_frames = 0;
    e->q_base = e->q_end = 0;
    e->mel_cache_n = 0;
    e->consumed = e->emitted = 0;
    e->closed = 0;
    e->cache_len = 0;
    e->pos = e->conv_left;
    e->frames_decoded = e->dec_iterations = 0;
    /* conv history rows [0, conv_left) of every layer and stream read as zeros again */
    const size_t D = (size_t)e->m->g.d_model, rowb = D * 4;
    for (int l = 0; l < e->m->g.n_layers; ++l)
        for (int s = 0; s < e->B; ++s) {
            float *base = e->din + ((size_t)l * e->B + s) * (size_t)e->cap_rows * D;
            if (cudaMemsetAsync(base, 0, (size_t)e->conv_left * rowb, e->st) != cudaSuccess) { snprintf(err, errlen, "reset failed"); return -1; }
        }
    if (nb_dec_reset(&e->dec, e->m->g.pred_hidden, e->m->g.blank_id, e->st) ||
        (e->dec_fused && nb_dec_rows_init(e->dec_r0, e->dec_r1, e->dec_b1i, e->B, 4 * e->m->g.pred_hidden, e->st))) {
        snprintf(err, errlen, "%s", nemo_gpu_last_error());
        return -1;
    }
    if (cudaStreamSynchronize(e->st) != cudaSuccess) { snprintf(err, errlen, "reset: %s", cudaGetErrorString(cudaGetLastError())); return -1; }
    return 0;
}

int nb_engine_right(const nb_engine_t *e) { return e->right; }
int nb_engine_streams(const nb_engine_t *e) { return e->B; }

int nb_engine_set_prompt(nb_engine_t *e, int s, int idx, char *err, size_t errlen) {
    if (s < 0 || s >= e->B || idx < 0 || idx >= e->m->g.num_prompts) { snprintf(err, errlen, "bad stream %d / prompt %d", s, idx); return -1; }
    const size_t PRH = (size_t)e->m->g.prompt_hidden;
    float *be = malloc(PRH * 4);
    nb_model_prompt_bias(e->m, idx, be);
    cudaError_t rc = cudaMemcpy(e->b_eff + (size_t)s * PRH, be, PRH * 4, cudaMemcpyHostToDevice);
    free(be);
    if (rc != cudaSuccess) { snprintf(err, errlen, "set prompt: %s", cudaGetErrorString(rc)); return -1; }
    e->prompt_idx[s] = idx;
    return 0;
}

int nb_engine_attach_device_mel(nb_engine_t *e, const float *d_mel, int64_t sstride_floats, size_t frames, char *err, size_t errlen) {
    if (e->consumed || e->pending_n) { snprintf(err, errlen, "attach a device mel source right after reset"); return -1; }
    e->dev_mel = d_mel;
    e->dev_mel_sstride = sstride_floats;
    e->dev_mel_frames = frames;
    e->pending_n = frames;
    return 0;
}

int nb_engine_push(nb_engine_t *e, const float *const *mel, size_t nframes, char *err, size_t errlen) {
    if (e->dev_mel) { snprintf(err, errlen, "engine reads a device mel source"); return -1; }
    if (!nframes) return 0;
    if (e->pending_n + nframes > e->pending_cap) {
        e->pending_cap = (e->pending_n + nframes) * 2;
        for (int s = 0; s < e->B; ++s) e->pending[s] = realloc(e->pending[s], e->pending_cap * 128 * sizeof(float));
    }
    for (int s = 0; s < e->B; ++s) memcpy(e->pending[s] + e->pending_n * 128, mel[s], nframes * 128 * sizeof(float));
    e->pending_n += nframes;
    return 0;
}

int nb_engine_gpu_mel(const nb_engine_t *e) { return e->use_gpu_mel; }

/* Staging span of stream s (pinned host memory, *cap floats); call nb_engine_span_wait first. */
float *nb_engine_span(nb_engine_t *e, int s, size_t *cap) {
    *cap = e->span_cap;
    return e->h_span + (size_t)s * e->span_cap;
}

/* The previous span upload has left the staging buffers. */
int nb_engine_span_wait(nb_engine_t *e) { return cudaEventSynchronize(e->span_ev) == cudaSuccess ? 0 : -1; }

/* nframes new frames of every stream from the staged spans (nb_mel_stage): upload, transform on
   the GPU into the frame queue, and queue them for the next steps. */
int nb_engine_upload_spans(nb_engine_t *e, int s0, int s1, size_t nframes, char *err, size_t errlen) {
    if (!nframes || s1 <= s0) return 0;
    if (!e->use_gpu_mel || e->dev_mel) { snprintf(err, errlen, "engine does not take sample spans"); return -1; }
    if (nframes > NB_SPAN_FRAMES || s0 < 0 || s1 > e->B) { snprintf(err, errlen, "span upload of %zu frames, streams %d..%d", nframes, s0, s1); return -1; }
    const size_t len = (nframes - 1) * NB_MEL_HOP + NB_MEL_NFFT, pitch = e->span_cap * sizeof(float);
    if (cudaMemcpy2DAsync(e->d_span + (size_t)s0 * e->span_cap, pitch, e->h_span + (size_t)s0 * e->span_cap, pitch, len * sizeof(float), (size_t)(s1 - s0),
                          cudaMemcpyHostToDevice, e->st) != cudaSuccess) {
        snprintf(err, errlen, "span upload: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    return 0;
}

int nb_engine_finish_spans(nb_engine_t *e, size_t nframes, char *err, size_t errlen) {
    if (!nframes) return 0;
    if (!e->use_gpu_mel || e->dev_mel) { snprintf(err, errlen, "engine does not take sample spans"); return -1; }
    if (nframes > NB_SPAN_FRAMES) { snprintf(err, errlen, "%zu frames in one span (at most %d)", nframes, NB_SPAN_FRAMES); return -1; }
    cudaStream_t st = e->st;
    const size_t row = 128 * sizeof(float);
    if (cudaEventRecord(e->span_ev, st) != cudaSuccess) {  /* the staging buffers are free again once this passes */
        snprintf(err, errlen, "span upload: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    if (e->q_end - e->q_base + nframes > e->qcap) {
        /* move the frames a later window can still read (from the next window's first frame on)
           to the front of the queue; the queue is sized so source and destination never overlap */
        const size_t keep_from = e->consumed - (size_t)e->mel_cache_n, keep = e->q_end - keep_from;
        if (keep_from < e->q_base || keep + nframes > e->qcap || keep_from - e->q_base < keep) {
            snprintf(err, errlen, "mel queue overflow (%zu pending frames)", keep);
            return -1;
        }
        if (keep && cudaMemcpy2DAsync(e->d_melq, e->qcap * row, e->d_melq + (keep_from - e->q_base) * 128, e->qcap * row, keep * row, (size_t)e->B,
                                      cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
            snprintf(err, errlen, "mel queue: %s", cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
        e->q_base = keep_from;
    }
    if (nb_logmel_frames(e->d_span, (int64_t)e->span_cap, e->B, (int)nframes, e->d_melq, (int64_t)e->qcap * 128, (int64_t)(e->q_end - e->q_base), st)) {
        snprintf(err, errlen, "%s", nemo_gpu_last_error());
        return -1;
    }
    e->q_end += nframes;
    e->pending_n += nframes;
    return 0;
}

/* Input at in_rate goes through the GPU resampler: with the log-mel on the GPU, for the rates
   nemo_resample takes (NEMO_GPU_RESAMPLE=0 keeps the host resampler). */
int nb_engine_gpu_resample(const nb_engine_t *e, int in_rate) {
    const char *v = getenv("NEMO_GPU_RESAMPLE");
    return e->use_gpu_mel && !e->dev_mel && in_rate != NB_MEL_SR && !(v && !strcmp(v, "0")) && nb_resample_smem_ok(in_rate, NB_MEL_SR);
}

/* Resample every stream's new input on the GPU. jobs[s] (nb_resampler_plan) must agree across
   streams on everything but the FIFO contents; on success out[s] points at job.count outputs of
   stream s in pinned memory, valid until the next call. The stream is idle on return. */
int nb_engine_resample(nb_engine_t *e, const nb_resample_job_t *jobs, const float **out, char *err, size_t errlen) {
    const int B = e->B;
    const nb_resample_job_t *j = &jobs[0];
    for (int s = 1; s < B; ++s)
        if (jobs[s].start != j->start || jobs[s].len != j->len || jobs[s].nin != j->nin || jobs[s].out0 != j->out0 || jobs[s].count != j->count ||
            jobs[s].in_rate != j->in_rate || jobs[s].out_rate != j->out_rate) {
            snprintf(err, errlen, "streams resampled to different lengths (%zu vs %zu outputs)", jobs[s].count, j->count);
            return -1;
        }
    if (!j->count) {
        for (int s = 0; s < B; ++s) out[s] = jobs[s].win;  /* no outputs: any valid pointer */
        return 0;
    }
    if (!nb_resample_smem_ok(j->in_rate, j->out_rate)) {
        snprintf(err, errlen, "input rate %d Hz is beyond the GPU resampler", j->in_rate);
        return -1;
    }
    if (j->count > (size_t)INT32_MAX) { snprintf(err, errlen, "%zu resampler outputs in one call", j->count); return -1; }
    cudaStream_t st = e->st;
    if (cudaStreamSynchronize(st) != cudaSuccess) { snprintf(err, errlen, "resampler: %s", cudaGetErrorString(cudaGetLastError())); return -1; }
    const size_t Bz = (size_t)B;
    if (j->len > e->rs_in_cap) {
        if (e->h_rs_in) cudaFreeHost(e->h_rs_in);
        if (e->d_rs_in) cudaFree(e->d_rs_in);
        e->h_rs_in = e->d_rs_in = NULL;
        e->rs_in_cap = 0;
        const size_t cap = (j->len + 4095) / 4096 * 4096 * 2;
        if (cudaMallocHost((void **)&e->h_rs_in, Bz * cap * sizeof(float)) != cudaSuccess || cudaMalloc((void **)&e->d_rs_in, Bz * cap * sizeof(float)) != cudaSuccess) {
            snprintf(err, errlen, "resampler input buffers: %s", cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
        e->rs_in_cap = cap;
    }
    if (j->count > e->rs_out_cap) {
        if (e->h_rs_out) cudaFreeHost(e->h_rs_out);
        if (e->d_rs_out) cudaFree(e->d_rs_out);
        e->h_rs_out = e->d_rs_out = NULL;
        e->rs_out_cap = 0;
        const size_t cap = (j->count + 4095) / 4096 * 4096 * 2;
        if (cudaMallocHost((void **)&e->h_rs_out, Bz * cap * sizeof(float)) != cudaSuccess || cudaMalloc((void **)&e->d_rs_out, Bz * cap * sizeof(float)) != cudaSuccess) {
            snprintf(err, errlen, "resampler output buffers: %s", cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
        e->rs_out_cap = cap;
    }
    if (j->len) {
#pragma omp parallel for schedule(static) if (B > 1)
        for (int s = 0; s < B; ++s) memcpy(e->h_rs_in + (size_t)s * e->rs_in_cap, jobs[s].win, j->len * sizeof(float));
        if (cudaMemcpy2DAsync(e->d_rs_in, e->rs_in_cap * sizeof(float), e->h_rs_in, e->rs_in_cap * sizeof(float), j->len * sizeof(float), Bz,
                              cudaMemcpyHostToDevice, st) != cudaSuccess) {
            snprintf(err, errlen, "resampler upload: %s", cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
    }
    if (nemo_resample(e->d_rs_in, (int64_t)e->rs_in_cap, j->start, (int64_t)j->len, (int64_t)j->nin, (int64_t)j->out0, (int)j->count, j->in_rate, j->out_rate,
                      e->d_rs_out, (int64_t)e->rs_out_cap, B, st)) {
        snprintf(err, errlen, "%s", nemo_gpu_last_error());
        return -1;
    }
    if (cudaMemcpy2DAsync(e->h_rs_out, e->rs_out_cap * sizeof(float), e->d_rs_out, e->rs_out_cap * sizeof(float), j->count * sizeof(float), Bz,
                          cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        snprintf(err, errlen, "resampler: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    for (int s = 0; s < B; ++s) out[s] = e->h_rs_out + (size_t)s * e->rs_out_cap;
    return 0;
}

int nb_engine_push_spans(nb_engine_t *e, size_t nframes, char *err, size_t errlen) {
    if (!nframes) return 0;
    if (nb_engine_upload_spans(e, 0, e->B, nframes, err, errlen)) return -1;
    return nb_engine_finish_spans(e, nframes, err, errlen);
}

void nb_engine_set_taps(nb_engine_t *e, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks) {
    e->tap_prompted = prompted;
    e->tap_joint = joint_enc;
    e->tap_cap = cap_rows;
    e->tap_rows = 0;
    e->tap_chunk_rows = chunk_rows;
    e->tap_chunk_cap = cap_chunks;
    e->tap_chunks = 0;
}
void nb_engine_tap_counts(const nb_engine_t *e, size_t *rows, size_t *chunks) { *rows = e->tap_rows; *chunks = e->tap_chunks; }
void nb_engine_times(const nb_engine_t *e, double *enc_ms, double *dec_ms, size_t *chunks) { *enc_ms = e->enc_ms; *dec_ms = e->dec_ms; *chunks = e->chunks; }

/* ---- device launch sequence of one encoder step ------------------------------------------ */
static nemo_gemm_args_t gemm_args(const void *A, int64_t lda, int a_fmt, int64_t a_plane, const uint16_t *W, int64_t ldw, const float *bias, void *C,
                                  int64_t ldc, int M, int N, int K, int act, int acc, float alpha) {
    nemo_gemm_args_t a;
    memset(&a, 0, sizeof a);
    a.A = A; a.lda = lda; a.a_fmt = a_fmt; a.a_plane = a_plane;
    a.W = W; a.ldw = ldw; a.bias = bias;
    a.C = C; a.ldc = ldc; a.c_fmt = NEMO_FMT_F32;
    a.M = M; a.N = N; a.K = K; a.act = act; a.accumulate = acc; a.alpha = alpha;
    return a;
}

static int launch_encoder(nb_engine_t *e, int nwin, int c) {
    const nb_model_t *m = e->m;
    const nb_config_t *g = &m->g;
    const int B = e->B, D = g->d_model, CH = g->sub_channels, FF = g->d_ff, PRH = g->prompt_hidden, JH = g->joint_hidden, NP = g->num_prompts;
    const int T1 = sub_len(nwin), F1 = 65, T2 = T1 / 2 + 1, F2 = F1 / 2 + 1, T3 = T2 / 2 + 1, F3 = F2 / 2 + 1;
    const int M = B * c;
    const float eps = g->ln_eps;
    cudaStream_t st = e->st;
    int *d_pos = e->d_params, *d_cache_len = e->d_params + 1, *d_lo = e->d_params + 2;
    const int fl = e->fmt_layer, fc = e->fmt_conv;
    /* plane offsets (elements) for buffers written as bf16 hi/lo */
    const int64_t pl_c1 = (int64_t)B * T2 * F2 * CH, pl_c3 = (int64_t)B * T3 * F3 * CH, pl_row = (int64_t)B * e->cmax;
    nemo_gemm_args_t a;

    /* subsampling (src/encoder.c:121-142); the flatten keeps only rows [lo, lo + c) (:258) */
    if (nemo_subsample_front(e->d_win, (int64_t)e->nwin_max * 128, m->conv0_w, m->conv0_b, m->conv2_w, m->conv2_b, e->c1, fc, pl_c1, B, nwin, 128, CH, st))
        return -1;
    a = gemm_args(e->c1, CH, fc, pl_c1, m->conv3_w, CH, m->conv3_b, e->c2, CH, B * T2 * F2, CH, CH, NEMO_ACT_RELU, 0, 1.0f);
    if (nemo_gemm(&a, st)) return -1;
    if (nb_dwconv2d_s2_fmt(e->c2, m->conv5_w, m->conv5_b, e->c3, fc, pl_c3, B, T2, F2, T3, F3, CH, st)) return -1;
    a = gemm_args(e->c3, CH, fc, pl_c3, m->conv6_w, CH, m->conv6_b, e->c4, CH, B * T3 * F3, CH, CH, NEMO_ACT_RELU, 0, 1.0f);
    if (nemo_gemm(&a, st)) return -1;
    if (nb_flatten_rows_fmt(e->c4, e->flat, fl, pl_row * CH * F3, d_lo, B, T3, F3, CH, c, st)) return -1;
    float *h = e->hbuf[0], *hn = e->hbuf[1];
    a = gemm_args(e->flat, CH * F3, fl, pl_row * CH * F3, m->pre_out_w, CH * F3, m->pre_out_b, h, D, M, D, CH * F3, 0, 0, 1.0f);
    if (nemo_gemm(&a, st)) return -1;

    /* 24 conformer blocks (src/encoder.c:145-188) */
    const int64_t plD = pl_row * D, plFF = pl_row * FF;
    const int64_t kv_s = (int64_t)e->cap_rows * 3 * D, din_s = (int64_t)e->cap_rows * D;
    if (e->use_enc1) {
        NbEnc1Args *q = &e->enc1_args;
        memset(q, 0, sizeof *q);
        memcpy(q->L, e->enc1_layers, (size_t)g->n_layers * sizeof *e->enc1_layers);
        q->layers = g->n_layers; q->D = D; q->FF = FF; q->H = g->n_heads; q->taps = g->conv_kernel; q->Lmax = e->Lmax; q->c = c;
        q->left = e->left;
        q->ring_bytes = nb_encoder1_ring_bytes(D, FF, e->enc1_grid, (size_t)e->enc1_optin, c, e->left + c);  /* per chunk shape */
        q->eps = eps; q->scale = 1.0f / sqrtf(128.0f);
        q->pos = d_pos; q->cache_len = d_cache_len;
        q->h = h; q->h2 = hn; q->ff = e->ff; q->att = e->att; q->image = e->enc1_image; q->fold = e->enc1_fold;
        q->xout = (uint16_t *)e->xin; q->xout_plane = plD;
        q->bar = e->d_enc1_bar; q->err = e->d_enc1_err;
        q->tail = e->enc1_tail; q->PRH = PRH; q->JH = JH; q->pw0_ld = D + NP;
        q->pw0 = m->prompt_w0; q->pw2 = m->prompt_w2; q->jw = m->joint_enc_w;
        q->pb0 = e->b_eff; q->pb2 = m->prompt_b2; q->jb = m->joint_enc_b;  /* one stream: its prompt bias row */
        q->ph = e->ph; q->prompted = e->prompted; q->joint = e->joint_enc;
        if (nb_encoder1(q, e->enc1_grid, st)) return -1;
        if (e->enc1_tail) return 0;  /* prompted and joint_enc came out of the launch */
    }
    for (int l = 0; l < (e->use_enc1 ? 0 : g->n_layers); ++l) {
        const nb_layer_t *W = &m->L[l];
        float *kv = e->kv + (size_t)l * B * kv_s, *din = e->din + (size_t)l * B * din_s;
        if (l == 0 && nemo_layernorm(h, W->ln_ff1_g, W->ln_ff1_b, e->xin, fl, plD, M, D, eps, st)) return -1;
        a = gemm_args(e->xin, D, fl, plD, W->ff1_w1, D, NULL, e->ff, FF, M, FF, D, NEMO_ACT_SILU, 0, 1.0f);
        a.c_fmt = fl; a.c_plane = plFF;
        if (nemo_gemm(&a, st)) return -1;
        a = gemm_args(e->ff, FF, fl, plFF, W->ff1_w2, FF, NULL, h, D, M, D, FF, 0, 1, 0.5f);
        if (nemo_gemm(&a, st)) return -1;
        /* attention: q|k|v appended to the per-stream cache rows [pos, pos + c) */
        if (nemo_layernorm(h, W->ln_att_g, W->ln_att_b, e->xin, fl, plD, M, D, eps, st)) return -1;
        a = gemm_args(e->xin, D, fl, plD, W->wqkv, D, NULL, kv, 3 * D, M, 3 * D, D, 0, 0, 1.0f);
        a.rpg = c; a.gstride = kv_s; a.rowoff = d_pos;
        if (nemo_gemm(&a, st)) return -1;
        if (nemo_attention_rel(kv, 3 * D, kv_s, kv + D, kv + 2 * D, 3 * D, kv_s, d_pos, d_cache_len, W->ptab, W->bias_u, W->bias_v, e->att, fl, plD,
                               (int64_t)c * D, B, c, e->Lmax, g->n_heads, 128, D, 1.0f / sqrtf(128.0f), st))
            return -1;
        a = gemm_args(e->att, D, fl, plD, W->wo, D, NULL, h, D, M, D, D, 0, 1, 1.0f);
        if (nemo_gemm(&a, st)) return -1;
        /* conv module: GLU output appended to the conv history at rows [pos, pos + c) */
        if (nemo_layernorm(h, W->ln_conv_g, W->ln_conv_b, e->xin, fl, plD, M, D, eps, st)) return -1;
        a = gemm_args(e->xin, D, fl, plD, W->pw1, D, NULL, din, D, M, 2 * D, D, NEMO_ACT_GLU, 0, 1.0f);
        a.rpg = c; a.gstride = din_s; a.rowoff = d_pos;
        if (nemo_gemm(&a, st)) return -1;
        if (nemo_dwconv_ln_silu(din, din_s, d_pos, W->dw_w, W->bn_g, W->bn_b, e->y, fl, plD, B, c, D, g->conv_kernel, eps, st)) return -1;
        a = gemm_args(e->y, D, fl, plD, W->pw2, D, NULL, h, D, M, D, D, 0, 1, 1.0f);
        if (nemo_gemm(&a, st)) return -1;
        /* FF2 half step, then the output norm fused with the next block's FF1 norm */
        if (nemo_layernorm(h, W->ln_ff2_g, W->ln_ff2_b, e->xin, fl, plD, M, D, eps, st)) return -1;
        a = gemm_args(e->xin, D, fl, plD, W->ff2_w1, D, NULL, e->ff, FF, M, FF, D, NEMO_ACT_SILU, 0, 1.0f);
        a.c_fmt = fl; a.c_plane = plFF;
        if (nemo_gemm(&a, st)) return -1;
        a = gemm_args(e->ff, FF, fl, plFF, W->ff2_w2, FF, NULL, h, D, M, D, FF, 0, 1, 0.5f);
        if (nemo_gemm(&a, st)) return -1;
        if (l + 1 < g->n_layers) {
            const nb_layer_t *Wn = &m->L[l + 1];
            if (nemo_layernorm2(h, W->ln_out_g, W->ln_out_b, Wn->ln_ff1_g, Wn->ln_ff1_b, hn, e->xin, fl, plD, M, D, eps, st)) return -1;
            float *sw = h; h = hn; hn = sw;
        } else {
            if (nemo_layernorm(h, W->ln_out_g, W->ln_out_b, e->xin, fl, plD, M, D, eps, st)) return -1;
        }
    }
    /* language prompt (per-stream one-hot folded into the bias) and joint encoder projection
       (src/encoder.c:189-194) */
    a = gemm_args(e->xin, D, fl, plD, m->prompt_w0, D + NP, e->b_eff, e->ph, PRH, M, PRH, D, NEMO_ACT_RELU, 0, 1.0f);
    a.rpg = c; a.gstride = (int64_t)c * PRH; a.bias_gstride = PRH; a.c_fmt = fl; a.c_plane = pl_row * PRH;
    if (nemo_gemm(&a, st)) return -1;
    /* post-prompt encoder output: fp32 for the caller, plus bf16 planes for the next GEMM */
    a = gemm_args(e->ph, PRH, fl, pl_row * PRH, m->prompt_w2, PRH, m->prompt_b2, e->prompted_x, D, M, D, PRH, 0, 0, 1.0f);
    if (fl != NEMO_FMT_F32) { a.c_fmt = fl; a.c_plane = plD; a.c32 = e->prompted; a.ldc32 = D; }
    if (nemo_gemm(&a, st)) return -1;
    a = gemm_args(e->prompted_x, D, fl, plD, m->joint_enc_w, D, m->joint_enc_b, e->joint_enc, JH, M, JH, D, 0, 0, 1.0f);
    if (nemo_gemm(&a, st)) return -1;
    return 0;
}

/* ---- greedy RNNT decode of the chunk's c frames for every stream (src/decoder.c:92-127) --- */
/* One greedy-decoding iteration of every stream (one frame decision each), ending with the
   read-back of the still-active count. */
static int dec_max_iterations(const nb_engine_t *e, int c) { return c * (e->m->g.max_symbols + 1) + 2; }

/* One greedy iteration over all streams (src/decoder.c:97-123). cond is the WHILE-loop handle
   when the iteration is the body of the decoder graph (the device decides whether it repeats),
   0 when the host drives the loop (the active count is then copied back each iteration). */
static NbDecStep dec_step_args(const nb_engine_t *e) {
    const nb_config_t *g = &e->m->g;
    const DecState *d = &e->dec;
    NbDecStep s;
    memset(&s, 0, sizeof s);
    s.logits = d->logits; s.ldl = logits_ld(g); s.V = g->num_classes; s.blank = g->blank_id; s.max_symbols = g->max_symbols;
    s.PH = g->pred_hidden; s.JH = g->joint_hidden; s.enc = e->joint_enc;
    s.T = e->dec_table; s.R0 = e->dec_r0; s.c0 = d->c;
    s.part_v = e->dec_pv; s.part_i = e->dec_pi; s.nparts = e->dec_np;
    s.A = (uint16_t *)d->A0; s.a_ld = g->pred_hidden; s.a_plane = d->a_plane;
    s.X = d->jx; s.x_plane = (int64_t)e->B * g->joint_hidden;
    return s;
}

/* One fused greedy iteration (see NbDecEpi): three GEMMs with decoder epilogues and the step. */
static int dec_fused_body(nb_engine_t *e, int c, unsigned long long cond) {
    const nb_model_t *m = e->m;
    const nb_config_t *g = &m->g;
    const int B = e->B, PH = g->pred_hidden, JH = g->joint_hidden;
    DecState *d = &e->dec;
    cudaStream_t st = e->st;
    char err[8];
    const size_t errlen = 0;
    (void)err; (void)errlen;
    const NbDecStep s = dec_step_args(e);
    NbDecEpi de;
    memset(&de, 0, sizeof de);
    de.mode = 1;
    de.n_split = 4 * PH;
    de.need_idx = d->need_idx;
    de.row = e->dec_r1;
    de.c = d->c + (int64_t)B * PH;
    de.next = (uint16_t *)d->hp1c; de.next_ld = PH; de.next_plane = d->h_plane;
    de.aux = e->dec_r0;
    nemo_gemm_args_t a = gemm_args(d->A0, PH, NEMO_FMT_BF16X2, d->a_plane, e->dec_wg1, PH, NULL, NULL, 0, B, 8 * PH, PH, 0, 0, 1.0f);
    a.dynM = d->cnt;
    KL(nb_gemm_dec(&a, &de, st));
    memset(&de, 0, sizeof de);
    de.mode = 2;
    de.n_split = JH;
    de.need_idx = d->need_idx; de.enc = e->joint_enc; de.erow = d->erow; de.pred = d->pred; de.X = d->jx; de.x_plane = s.x_plane;
    de.aux = e->dec_r1; de.aux_bias = e->dec_b1i;
    a = gemm_args(d->hp1c, PH, NEMO_FMT_BF16X2, d->h_plane, e->dec_wg2, PH, m->joint_pred_b, NULL, 0, B, JH + 4 * PH, PH, 0, 0, 1.0f);
    a.dynM = d->cnt;
    KL(nb_gemm_dec(&a, &de, st));
    /* joint logits reduced to (value, column) partials per 128-column tile half in the epilogue */
    memset(&de, 0, sizeof de);
    de.mode = 3;
    de.n_split = g->num_classes;
    de.part_v = e->dec_pv; de.part_i = e->dec_pi; de.part_ld = e->dec_np;
    nemo_gemm_args_t j = gemm_args(d->jx, JH, NEMO_FMT_BF16X2, s.x_plane, m->joint_out_w, JH, m->joint_out_b, NULL, 0, B, g->num_classes, JH, 0, 0,
                                   1.0f);
    KL(nb_gemm_dec(&j, &de, st));
    KL(nb_dec_step(d, &s, c, dec_max_iterations(e, c), cond, st));
    if (!cond && cudaMemcpyAsync(e->h_cnt, d->cnt, 2 * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return nb_set_error("decoder: %s", cudaGetErrorString(cudaGetLastError()));
    return 0;
}

static int dec_iteration_body(nb_engine_t *e, int c, unsigned long long cond) {
    const nb_model_t *m = e->m;
    const nb_config_t *g = &m->g;
    const int B = e->B, PH = g->pred_hidden, JH = g->joint_hidden;
    DecState *d = &e->dec;
    cudaStream_t st = e->st;
    char err[8];
    const size_t errlen = 0;
    (void)err; (void)errlen;
    if (e->dec_fused) return dec_fused_body(e, c, cond);
    {
        KL(nb_dec_plan(d, c, st));
        KL(nb_dec_gather(d, m->embed, PH, g->blank_id, st));
        nemo_gemm_args_t a = gemm_args(d->A0, 2 * PH, d->fmt, d->a_plane, m->lstm_w[0], 2 * PH, m->lstm_b[0], d->gates, 4 * PH, B, 4 * PH, 2 * PH, 0, 0, 1.0f);
        a.dynM = d->cnt;
        KL(nemo_gemm(&a, st));
        KL(nb_dec_cell(d, 0, PH, d->A1, 2 * PH, d->a_plane, st));
        a = gemm_args(d->A1, 2 * PH, d->fmt, d->a_plane, m->lstm_w[1], 2 * PH, m->lstm_b[1], d->gates, 4 * PH, B, 4 * PH, 2 * PH, 0, 0, 1.0f);
        a.dynM = d->cnt;
        KL(nemo_gemm(&a, st));
        KL(nb_dec_cell(d, 1, PH, d->hp1c, PH, d->h_plane, st));
        a = gemm_args(d->hp1c, PH, d->fmt, d->h_plane, m->joint_pred_w, PH, m->joint_pred_b, d->predc, JH, B, JH, PH, 0, 0, 1.0f);
        a.dynM = d->cnt;
        KL(nemo_gemm(&a, st));
        if (d->fmt == NEMO_FMT_BF16X2) {
            /* joint input (with the prediction scatter), joint GEMM, then the update takes each row's argmax */
            KL(nb_dec_joint_in(d, e->joint_enc, JH, d->jx, (int64_t)B * JH, st));
            nemo_gemm_args_t j = gemm_args(d->jx, JH, NEMO_FMT_BF16X2, (int64_t)B * JH, m->joint_out_w, JH, m->joint_out_b, d->logits, logits_ld(g), B,
                                           g->num_classes, JH, 0, 0, 1.0f);
            KL(nemo_gemm(&j, st));
            KL(nb_dec_update(d, c, PH, g->blank_id, g->max_symbols, dec_max_iterations(e, c), cond, d->logits, logits_ld(g), g->num_classes, st));
        } else {
            KL(nb_dec_scatter_pred(d, JH, st));
            KL(nb_joint_argmax_rows(e->joint_enc, JH, d->pred, JH, 1, m->joint_out_w, m->joint_out_b, g->num_classes, JH, B, d->erow, d->idx, NULL, st));
            KL(nb_dec_update(d, c, PH, g->blank_id, g->max_symbols, dec_max_iterations(e, c), cond, NULL, 0, 0, st));
        }
        if (!cond && cudaMemcpyAsync(e->h_cnt, d->cnt, 2 * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return nb_set_error("decoder: %s", cudaGetErrorString(cudaGetLastError()));
    }
    return 0;
}

static int dec_iteration(nb_engine_t *e, int c, int unused) {
    (void)unused;
    return dec_iteration_body(e, c, 0);
}

/* The greedy loop of a chunk as one graph: a WHILE node whose body is dec_unroll iterations;
   each iteration's last kernel sets the loop condition on the device, so no host round trip
   happens per emitted token (src/decoder.c:97-123 loops on the host). Iterations that run after
   every stream finished change nothing (no stream is listed or active). Cached per chunk length c. Returns the slot,
   or -1 on error, or -2 when the cache is full (the host loop is used instead). */
static int dec_graph(nb_engine_t *e, int c) {
    for (int i = 0; i < e->ngraphs; ++i)
        if (e->graphs[i].kind == 2 && e->graphs[i].k1 == c) return i;
    if (e->ngraphs == NB_MAX_GRAPHS) return -2;
    cudaGraph_t G = NULL;
    cudaGraphConditionalHandle h;
    if (cudaGraphCreate(&G, 0) != cudaSuccess) return nb_set_error("decoder graph: %s", cudaGetErrorString(cudaGetLastError()));
    struct cudaGraphNodeParams p;
    memset(&p, 0, sizeof p);
    cudaGraphNode_t node;
    if (cudaGraphConditionalHandleCreate(&h, G, 1, cudaGraphCondAssignDefault) != cudaSuccess) goto fail;
    p.type = cudaGraphNodeTypeConditional;
    p.conditional.handle = h;
    p.conditional.type = cudaGraphCondTypeWhile;
    p.conditional.size = 1;
    if (cudaGraphAddNode(&node, G, NULL, 0, &p) != cudaSuccess) goto fail;
    cudaGraph_t body = p.conditional.phGraph_out[0];
    if (cudaStreamBeginCaptureToGraph(e->st, body, NULL, NULL, 0, cudaStreamCaptureModeThreadLocal) != cudaSuccess) goto fail;
    nb_set_launch_counting(0);
    int rc = 0;
    for (int u = 0; u < e->dec_unroll && !rc; ++u) rc = dec_iteration_body(e, c, (unsigned long long)h);
    nb_set_launch_counting(1);
    cudaGraph_t captured = NULL;
    const cudaError_t ce = cudaStreamEndCapture(e->st, &captured);
    if (rc || ce != cudaSuccess) {
        cudaGraphDestroy(G);
        return rc ? -1 : nb_set_error("decoder graph capture: %s", cudaGetErrorString(ce));
    }
    cudaGraphExec_t exec;
    if (cudaGraphInstantiate(&exec, G, 0) != cudaSuccess) goto fail;
    const int slot = e->ngraphs++;
    e->graphs[slot].kind = 2;
    e->graphs[slot].k1 = c;
    e->graphs[slot].k2 = 0;
    e->graphs[slot].exec = exec;
    e->graphs[slot].kernels = nb_graph_kernel_nodes(body) / (uint64_t)e->dec_unroll; /* per iteration */
    cudaGraphDestroy(G);
    return slot;
fail:
    nb_set_error("decoder graph: %s", cudaGetErrorString(cudaGetLastError()));
    cudaGraphDestroy(G);
    return -1;
}

static int enc_body(nb_engine_t *e, int nwin, int c) { return launch_encoder(e, nwin, c); }

/* Slot of the graph keyed by (kind, k1, k2), capturing `body` into it when it does not exist yet
   (nothing runs). Returns the slot, -1 on error, -2 when the table is full. */
static int capture_graph(nb_engine_t *e, int kind, int k1, int k2, int (*body)(nb_engine_t *, int, int)) {
    int slot = -1;
    for (int i = 0; i < e->ngraphs; ++i)
        if (e->graphs[i].kind == kind && e->graphs[i].k1 == k1 && e->graphs[i].k2 == k2) { slot = i; break; }
    if (slot < 0) {
        if (e->ngraphs == NB_MAX_GRAPHS) return -2;
        cudaGraph_t graph;
        if (cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
            return nb_set_error("graph capture: %s", cudaGetErrorString(cudaGetLastError()));
        nb_set_launch_counting(0);
        const int rc = body(e, k1, k2);
        nb_set_launch_counting(1);
        const cudaError_t ce = cudaStreamEndCapture(e->st, &graph);
        if (rc || ce != cudaSuccess) {
            if (ce == cudaSuccess) cudaGraphDestroy(graph);
            return rc ? -1 : nb_set_error("graph capture: %s", cudaGetErrorString(ce));
        }
        cudaGraphExec_t exec;
        if (cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
            cudaGraphDestroy(graph);
            return nb_set_error("graph instantiate: %s", cudaGetErrorString(cudaGetLastError()));
        }
        slot = e->ngraphs++;
        e->graphs[slot].kind = kind;
        e->graphs[slot].k1 = k1;
        e->graphs[slot].k2 = k2;
        e->graphs[slot].exec = exec;
        e->graphs[slot].kernels = nb_graph_kernel_nodes(graph);
        cudaGraphDestroy(graph);
    }
    return slot;
}

/* Launch `body` through a captured graph keyed by (kind, k1, k2), capturing it on first use. */
static int run_graph(nb_engine_t *e, int kind, int k1, int k2, int (*body)(nb_engine_t *, int, int)) {
    if (!e->use_graphs) return body(e, k1, k2);
    const int slot = capture_graph(e, kind, k1, k2, body);
    if (slot == -2) return body(e, k1, k2);
    if (slot < 0) return -1;
    if (cudaGraphLaunch(e->graphs[slot].exec, e->st) != cudaSuccess) return nb_set_error("graph launch: %s", cudaGetErrorString(cudaGetLastError()));
    nb_count_launches(e->graphs[slot].kernels);
    return 0;
}

/* Chunk shapes (window rows, encoder rows) a stream can produce, from the bookkeeping of
   nb_engine_step (src/encoder.c:229-249) run on frame counts alone: whole chunks, then a final
   piece of 1..chunk_mel frames after 0, 1, 2 or 3 whole chunks. From the second whole chunk on
   the state repeats (16 cached rows, every whole chunk emitted), so these cover every stream
   length. Writes up to cap pairs, returns how many there are. */
static int chunk_shapes(const nb_engine_t *e, int (*out)[2], int cap) {
    int n = 0;
    for (int k = 0; k <= 3; ++k)
        for (int r = 0; r <= e->chunk_mel; ++r) {
            size_t consumed = 0, emitted = 0;
            int mel_cache_n = 0;
            for (int j = 0; j <= k; ++j) {
                const int last = j == k;
                if (last && r == 0) break;
                const int take = last ? r : e->chunk_mel;
                const int nwin = mel_cache_n + take;
                const size_t end = consumed + (size_t)take, base = (consumed - (size_t)mel_cache_n) / 8, lo = emitted - base;
                const size_t hi = last ? (size_t)sub_len(sub_len(sub_len(nwin))) : end / 8 - base;
                consumed = end;
                mel_cache_n = nwin < NB_MEL_CACHE ? nwin : NB_MEL_CACHE;
                if (hi <= lo) { emitted = base + (lo > hi ? lo : hi); continue; }
                emitted = base + hi;
                const int c = (int)(hi - lo);
                int seen = 0;
                for (int i = 0; i < n && i < cap; ++i) seen |= out[i][0] == nwin && out[i][1] == c;
                if (!seen) {
                    if (n < cap) { out[n][0] = nwin; out[n][1] = c; }
                    ++n;
                }
            }
        }
    return n;
}

/* Warm-up (src/warmup.c:23-42): capture the graphs of every chunk shape a stream at this
   engine's latency can reach, without running them, so no chunk of a later stream pays a graph
   capture. The engine's stream state is not touched. */
int nb_engine_prepare(nb_engine_t *e, char *err, size_t errlen) {
    if (!e->use_graphs) return 0;
    int shapes[NB_MAX_GRAPHS][2];
    const int n = chunk_shapes(e, shapes, NB_MAX_GRAPHS);
    int missing = 0;
    for (int i = 0; i < n && i < NB_MAX_GRAPHS; ++i) {
        int have = 0;
        for (int j = 0; j < e->ngraphs; ++j) have |= e->graphs[j].kind == 0 && e->graphs[j].k1 == shapes[i][0] && e->graphs[j].k2 == shapes[i][1];
        missing += !have;
    }
    if (n > NB_MAX_GRAPHS || missing * (e->use_dec1 ? 1 : 2) + e->ngraphs > NB_MAX_GRAPHS) {
        snprintf(err, errlen, "warm-up: %d chunk shapes exceed the graph table", n);
        return -1;
    }
    for (int i = 0; i < n; ++i) {
        const int c = shapes[i][1];
        if (c > e->cmax) { snprintf(err, errlen, "warm-up: chunk of %d rows exceeds buffer %d", c, e->cmax); return -1; }
        if (capture_graph(e, 0, shapes[i][0], c, enc_body) < 0) { snprintf(err, errlen, "warm-up: %s", nemo_gpu_last_error()); return -1; }
        if (!e->use_dec1 && dec_graph(e, c) == -1) { snprintf(err, errlen, "warm-up: %s", nemo_gpu_last_error()); return -1; }
    }
    return 0;
}

int nb_engine_graphs(const nb_engine_t *e) { return e->ngraphs; }

int nb_engine_decode_counts(nb_engine_t *e, long long out[4], char *err, size_t errlen) {
    int st[2] = { 0, 0 };
    if (cudaStreamSynchronize(e->st) != cudaSuccess || cudaMemcpy(st, e->dec.stats, sizeof st, cudaMemcpyDeviceToHost) != cudaSuccess) {
        snprintf(err, errlen, "decode counts: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    out[0] = e->frames_decoded;
    out[1] = e->use_dec1 ? -1 : st[0];
    out[2] = e->use_dec1 ? -1 : st[1];
    out[3] = e->dec_iterations;
    return 0;
}

static int run_decoder(nb_engine_t *e, int c, char *err, size_t errlen) {
    const nb_config_t *g = &e->m->g;
    DecState *d = &e->dec;
    cudaStream_t st = e->st;
    const int max_it = dec_max_iterations(e, c);
    if (e->use_dec1) {
        const nb_model_t *m = e->m;
        const size_t PH = (size_t)g->pred_hidden, JH = (size_t)g->joint_hidden;
        NbDec1Args a;
        memset(&a, 0, sizeof a);
        a.d = *d;
        a.W0 = m->lstm_w[0]; a.W1 = m->lstm_w[1]; a.Wp = m->joint_pred_w; a.Wo = m->joint_out_w; a.embed = m->embed;
        a.b0 = m->lstm_b[0]; a.b1 = m->lstm_b[1]; a.bp = m->joint_pred_b; a.bo = m->joint_out_b;
        a.enc = e->joint_enc;
        a.H0 = e->d_dec1; a.H1 = e->d_dec1 + 2 * PH; a.PRED = e->d_dec1 + 4 * PH; a.part_v = e->d_dec1 + 4 * PH + JH;
        a.part_i = e->d_dec1_i; a.err = e->d_dec1_i + (size_t)e->dec1_grid * 16; a.bar = e->d_dec1_bar;
        a.PH = g->pred_hidden; a.JH = g->joint_hidden; a.V = g->num_classes; a.blank = g->blank_id; a.max_symbols = g->max_symbols; a.c = c;
        int herr = 0;
        if (nb_decoder1(&a, e->dec1_grid, st)) { snprintf(err, errlen, "decoder: %s", nemo_gpu_last_error()); return -1; }
        if (cudaMemcpyAsync(e->h_cnt, d->cnt, 4 * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(&e->h_cnt[4], a.err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) {
            snprintf(err, errlen, "decoder: %s", cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
        herr = e->h_cnt[4];
        if (herr) { snprintf(err, errlen, "decoder: the persistent decoder gave up waiting (code %d)", herr); return -1; }
        if (c > 0 && e->h_cnt[1] != 0) { snprintf(err, errlen, "decoder did not finish the chunk in %d iterations", max_it); return -1; }
        return 0;
    }
    if (e->dec_fused) {
        const NbDecStep s = dec_step_args(e);
        KL(nb_dec_chunk_start(d, &s, c, st));
    } else {
        KL(nb_dec_chunk_init(d, c, st));
    }
    (void)g;
    if (e->use_graphs) {
        const int slot = dec_graph(e, c);
        if (slot == -1) { snprintf(err, errlen, "%s", nemo_gpu_last_error()); return -1; }
        if (slot >= 0) {
            /* no host wait here: the step's single synchronisation reads the counters */
            if (cudaGraphLaunch(e->graphs[slot].exec, st) != cudaSuccess ||
                cudaMemcpyAsync(e->h_cnt, d->cnt, 4 * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) {
                snprintf(err, errlen, "decoder: %s", cudaGetErrorString(cudaGetLastError()));
                return -1;
            }
            e->dec_pending_slot = slot;
            e->dec_pending_max_it = max_it;
            return 0;
        }
    }
    int it;
    for (it = 0; it < max_it; ++it) {
        if (run_graph(e, 1, c, 0, dec_iteration)) { snprintf(err, errlen, "decoder: %s", nemo_gpu_last_error()); return -1; }
        if (cudaStreamSynchronize(st) != cudaSuccess) {
            snprintf(err, errlen, "decoder: %s", cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
        if (e->h_cnt[1] == 0) break;
    }
    if (it == max_it) { snprintf(err, errlen, "decoder did not finish the chunk in %d iterations", max_it); return -1; }
    e->dec_iterations += it + 1;
    return 0;
}

int nb_engine_step(nb_engine_t *e, int final, int *tokens, int max_tokens, int *counts, int *frames, char *err, size_t errlen) {
    *frames = 0;
    if (e->closed) return 0;
    if (e->pending_n == 0) { if (final) e->closed = 1; return 0; }
    if ((int)e->pending_n < e->chunk_mel && !final) return 0;
    size_t take = (size_t)e->chunk_mel < e->pending_n ? (size_t)e->chunk_mel : e->pending_n;
    if (final && e->pending_n <= (size_t)e->chunk_mel) take = e->pending_n;
    const int include_boundary = final && e->pending_n == take;
    /* window = mel cache ++ take rows, per stream */
    const int nwin = e->mel_cache_n + (int)take;
    const size_t wstride = (size_t)e->nwin_max * 128;
    const size_t win_first = e->consumed - (size_t)e->mel_cache_n; /* window = frames [win_first, consumed + take) */
    const int host_queue = !e->dev_mel && !e->use_gpu_mel;
    if (host_queue) {
        for (int s = 0; s < e->B; ++s) {
            float *w = e->h_win + (size_t)s * wstride;
            memcpy(w, e->mel_cache + (size_t)s * NB_MEL_CACHE * 128, (size_t)e->mel_cache_n * 128 * sizeof(float));
            memcpy(w + (size_t)e->mel_cache_n * 128, e->pending[s], take * 128 * sizeof(float));
        }
    }
    /* bookkeeping of src/encoder.c:229-249 */
    const size_t end = e->consumed + take;
    const size_t base = (e->consumed - (size_t)e->mel_cache_n) / 8;
    const size_t lo = e->emitted - base;
    const int T3 = sub_len(sub_len(sub_len(nwin)));
    const size_t hi = include_boundary ? (size_t)T3 : end / 8 - base;
    e->consumed = end;
    const int keep = nwin < NB_MEL_CACHE ? nwin : NB_MEL_CACHE;
    if (host_queue) {
        for (int s = 0; s < e->B; ++s)
            memcpy(e->mel_cache + (size_t)s * NB_MEL_CACHE * 128, e->h_win + (size_t)s * wstride + (size_t)(nwin - keep) * 128,
                   (size_t)keep * 128 * sizeof(float));
        for (int s = 0; s < e->B; ++s) memmove(e->pending[s], e->pending[s] + take * 128, (e->pending_n - take) * 128 * sizeof(float));
    }
    e->mel_cache_n = keep;
    e->pending_n -= take;
    if (final && e->pending_n == 0) e->closed = 1;
    if (hi <= lo) { e->emitted = base + (lo > hi ? lo : hi); return 1; }
    e->emitted = base + hi;
    const int c = (int)(hi - lo);
    if (c > e->cmax) { snprintf(err, errlen, "chunk of %d rows exceeds buffer %d", c, e->cmax); return -1; }

    cudaStream_t st = e->st;
    const nb_config_t *g = &e->m->g;
    const size_t D = (size_t)g->d_model;
    cudaEventRecord(e->ev0, st);
    if (e->pos + c > e->cap_rows) {
        if (nb_compact(e->kv, e->din, g->n_layers, e->B, e->cap_rows, (int)D, e->pos - e->cache_len, e->cache_len, e->pos - e->conv_left,
                       e->cache_len - e->conv_left, e->conv_left, st)) {
            snprintf(err, errlen, "%s", nemo_gpu_last_error());
            return -1;
        }
        e->pos = e->cache_len;
    }
    e->h_params[0] = e->pos;
    e->h_params[1] = e->cache_len;
    e->h_params[2] = (int)lo;
    cudaError_t wrc;
    if (e->dev_mel)
        wrc = cudaMemcpy2DAsync(e->d_win, wstride * sizeof(float), e->dev_mel + win_first * 128, (size_t)e->dev_mel_sstride * sizeof(float),
                                (size_t)nwin * 128 * sizeof(float), (size_t)e->B, cudaMemcpyDeviceToDevice, st);
    else if (e->use_gpu_mel)
        wrc = cudaMemcpy2DAsync(e->d_win, wstride * sizeof(float), e->d_melq + (win_first - e->q_base) * 128, e->qcap * 128 * sizeof(float),
                                (size_t)nwin * 128 * sizeof(float), (size_t)e->B, cudaMemcpyDeviceToDevice, st);
    else
        wrc = cudaMemcpyAsync(e->d_win, e->h_win, (size_t)e->B * wstride * sizeof(float), cudaMemcpyHostToDevice, st);
    if (wrc != cudaSuccess || cudaMemcpyAsync(e->d_params, e->h_params, 3 * sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess) {
        snprintf(err, errlen, "upload: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    if (run_graph(e, 0, nwin, c, enc_body)) { snprintf(err, errlen, "encoder: %s", nemo_gpu_last_error()); return -1; }
    /* the decoder is queued behind the encoder without a host round trip; the device error words
       are read after the step's one synchronisation */
    if (cudaEventRecord(e->ev_mid, st) != cudaSuccess ||
        (e->use_enc1 && cudaMemcpyAsync(&e->h_cnt[5], e->d_enc1_err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)) {
        snprintf(err, errlen, "encoder: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    e->pos += c;
    const int L = e->cache_len + c;
    e->cache_len = L < e->left ? L : e->left;
    if (e->tap_prompted) {
        /* taps (tests only): the encoder's rows once it finished */
        if (cudaStreamSynchronize(st) != cudaSuccess) { snprintf(err, errlen, "encoder: %s", cudaGetErrorString(cudaGetLastError())); return -1; }
        const size_t rows = (size_t)e->B * c;
        if (e->tap_rows + rows <= e->tap_cap) {
            cudaMemcpy(e->tap_prompted + e->tap_rows * D, e->prompted, rows * D * 4, cudaMemcpyDeviceToHost);
            cudaMemcpy(e->tap_joint + e->tap_rows * (size_t)g->joint_hidden, e->joint_enc, rows * (size_t)g->joint_hidden * 4, cudaMemcpyDeviceToHost);
            e->tap_rows += rows;
        }
        if (e->tap_chunks < e->tap_chunk_cap) e->tap_chunk_rows[e->tap_chunks] = c;
        e->tap_chunks++;
    }
    if (run_decoder(e, c, err, errlen)) return -1;
    const DecState *d = &e->dec;
    if (cudaMemcpyAsync(e->h_ntok, d->ntok, (size_t)e->B * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(e->h_tokens, d->tokens, (size_t)e->B * (size_t)d->tok_cap * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaEventRecord(e->ev1, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) {
        snprintf(err, errlen, "step: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    if (nemo_gpu_check_device_errors()) { snprintf(err, errlen, "step: %s", nemo_gpu_last_error()); return -1; }
    if (e->use_enc1 && e->h_cnt[5]) {
        snprintf(err, errlen, "encoder: the persistent encoder gave up waiting (code %d)", e->h_cnt[5]);
        return -1;
    }
    e->frames_decoded += (long long)e->B * c;
    if (e->dec_pending_slot >= 0) {
        e->dec_iterations += e->h_cnt[2];
        nb_count_launches(e->graphs[e->dec_pending_slot].kernels * (uint64_t)e->h_cnt[2]);
        e->dec_pending_slot = -1;
        if (e->h_cnt[1] != 0) { snprintf(err, errlen, "decoder did not finish the chunk in %d iterations", e->dec_pending_max_it); return -1; }
    }
    float step_ms = 0.0f, enc_ms = 0.0f;
    if (cudaEventElapsedTime(&step_ms, e->ev0, e->ev1) == cudaSuccess) e->gpu_ms += step_ms;
    if (cudaEventElapsedTime(&enc_ms, e->ev0, e->ev_mid) == cudaSuccess) {
        e->enc_ms += enc_ms;
        e->dec_ms += step_ms - enc_ms;
    }
    for (int s = 0; s < e->B; ++s) {
        const int n = e->h_ntok[s] < d->tok_cap ? e->h_ntok[s] : d->tok_cap;
        for (int i = 0; i < n; ++i)
            if (counts[s] < max_tokens) tokens[(size_t)s * max_tokens + counts[s]++] = e->h_tokens[(size_t)s * d->tok_cap + i];
    }
    e->chunks++;
    *frames = c;
    return 1;
}
