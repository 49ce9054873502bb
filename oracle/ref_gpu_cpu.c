/* ORACLE — TEST INFRASTRUCTURE ONLY (see oracle.h).

   A CPU implementation of the reference's GPU interface (src/gpu.h:20-41) so that the reference's
   own host C — src/model.c, encoder.c, decoder.c, nemoasr.c, mel.c, resample.c, json.c,
   safetensors.c, tokenizer.c, warmup.c, compiled unmodified where they lie — runs on this machine.
   Buffers are zero-filled host memory (like the Metal shared-storage buffers, src/gpu.m:51-58);
   each dispatch is executed immediately by name with the restated kernels of oracle_kernels.c
   (the Metal source, src/kernels.metal, cannot be compiled here). The result is used to pin the
   restated bookkeeping in oracle_stream.c: both must produce the same numbers. */
#include "gpu.h"
#include "kernel_params.h"
#include "oracle.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

const char kernels_metal_src[] = ""; /* referenced by src/model.c:183; nothing to compile on CPU */

struct gpu { char err[256]; };
struct gpu_buf { void *p; size_t len; };

gpu_t *gpu_create(const char *src, char *err, size_t errlen) { (void)src; (void)err; (void)errlen; return calloc(1, sizeof(gpu_t)); }
void gpu_destroy(gpu_t *g) { free(g); }
const char *gpu_device_name(gpu_t *g) { (void)g; return "cpu-oracle"; }
gpu_buf_t *gpu_buf_alloc(gpu_t *g, size_t bytes) {
    (void)g;
    gpu_buf_t *b = calloc(1, sizeof *b);
    b->len = bytes ? bytes : 16;
    b->p = calloc(1, b->len);
    if (!b->p) { free(b); return NULL; }
    return b;
}
void gpu_buf_free(gpu_buf_t *b) { if (b) { free(b->p); free(b); } }
void *gpu_buf_ptr(gpu_buf_t *b) { return b->p; }
size_t gpu_buf_len(gpu_buf_t *b) { return b->len; }
int gpu_begin(gpu_t *g) { (void)g; return 0; }
int gpu_end(gpu_t *g, char *err, size_t errlen) {
    if (g->err[0]) { snprintf(err, errlen, "%s", g->err); return -1; }
    return 0;
}
double gpu_last_ms(gpu_t *g) { (void)g; return 0.0; }
const char *gpu_last_error(gpu_t *g) { return g->err; }

#define ARG(i) ((void *)(args[i].buf ? (char *)args[i].buf->p + args[i].offset : (char *)args[i].bytes))

static int run(gpu_t *g, const char *k, const gpu_arg_t *args, int nargs, uint32_t gx, uint32_t gy) {
    (void)nargs;
    if (!strcmp(k, "gemm_bf16") || !strcmp(k, "gemm_spec") || !strcmp(k, "gemm_mma")) {
        const GemmParams *p = ARG(4);
        int act = (int)p->act;
        if (!strcmp(k, "gemm_bf16") && act == 3) act = 0; /* gemm_bf16 has no GLU epilogue (kernels.metal:39-41) */
        or_gemm(ARG(0), (int)p->lda, ARG(1), (int)p->ldw, p->has_bias ? (const float *)ARG(2) : NULL, ARG(3), (int)p->ldc,
                (int)p->M, (int)p->N, (int)p->K, act, (int)p->accumulate, p->alpha);
    } else if (!strcmp(k, "layernorm")) {
        const LnParams *p = ARG(4);
        or_layernorm(ARG(0), ARG(1), ARG(2), ARG(3), (int)p->M, (int)p->D, p->eps);
    } else if (!strcmp(k, "layernorm2")) {
        const LnParams *p = ARG(7);
        or_layernorm2(ARG(0), ARG(1), ARG(2), ARG(3), ARG(4), ARG(5), ARG(6), (int)p->M, (int)p->D, p->eps);
    } else if (!strcmp(k, "attention_rel")) {
        const AttnParams *p = ARG(7);
        or_attention_rel(ARG(0), (int)p->ldq, ARG(1), ARG(2), (int)p->ldk, ARG(3), ARG(4), ARG(5), ARG(6),
                         (int)p->c, (int)p->L, (int)p->Lmax, (int)p->H, (int)p->dh, (int)p->D, p->scale);
    } else if (!strcmp(k, "dwconv_ln_silu")) {
        const DwParams *p = ARG(5);
        or_dwconv_ln_silu(ARG(0), ARG(1), ARG(2), ARG(3), ARG(4), (int)p->c, (int)p->D, (int)p->taps, p->eps);
    } else if (!strcmp(k, "conv2d_c1_s2_relu")) {
        const Conv2dParams *p = ARG(4);
        or_conv2d_c1_s2_relu(ARG(0), ARG(1), ARG(2), ARG(3), (int)p->T, (int)p->F, (int)p->T1, (int)p->F1, (int)p->C);
    } else if (!strcmp(k, "dwconv2d_s2")) {
        const Conv2dParams *p = ARG(4);
        or_dwconv2d_s2(ARG(0), ARG(1), ARG(2), ARG(3), (int)p->T, (int)p->F, (int)p->T1, (int)p->F1, (int)p->C);
    } else if (!strcmp(k, "flatten_cf")) {
        const FlatParams *p = ARG(2);
        or_flatten_cf(ARG(0), ARG(1), (int)p->T, (int)p->F, (int)p->C);
    } else if (!strcmp(k, "copy_f32")) {
        const CountParams *p = ARG(2);
        memmove(ARG(1), ARG(0), (size_t)p->n * sizeof(float));
    } else if (!strcmp(k, "fill_f32")) {
        const FillParams *p = ARG(1);
        float *d = ARG(0);
        for (uint32_t i = 0; i < p->n; ++i) d[i] = p->value;
    } else if (!strcmp(k, "lstm_cell")) {
        const LstmParams *p = ARG(4);
        or_lstm_cell(ARG(0), ARG(1), ARG(2), ARG(3), (int)p->H);
    } else if (!strcmp(k, "joint_partial")) {
        /* The whole row's argmax goes into partial slot 0; the other slots hold (-inf, INT_MAX),
           which argmax_reduce (kernels.metal:522-550) never prefers. */
        const JointParams *p = ARG(6);
        const uint32_t G = gx * GEMM_SIMDS, rows = gy;
        float *pv = ARG(4);
        int *pi = ARG(5);
        for (uint32_t r = 0; r < rows; ++r) {
            int idx;
            float val;
            const float *enc = (const float *)ARG(0) + (size_t)(p->enc_row + r) * p->enc_ld;
            or_joint_argmax(enc, (int)p->enc_ld, ARG(1), ARG(2), ARG(3), (int)p->V, (int)p->H, 1, &idx, &val, NULL);
            for (uint32_t i = 0; i < G; ++i) { pv[r * G + i] = i ? -INFINITY : val; pi[r * G + i] = i ? 0x7fffffff : idx; }
        }
    } else if (!strcmp(k, "argmax_reduce")) {
        const CountParams *p = ARG(3);
        const float *pv = ARG(0);
        const int *pi = ARG(1);
        int *out = ARG(2);
        for (uint32_t r = 0; r < gx; ++r) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (uint32_t i = 0; i < p->n; ++i) {
                const float v = pv[r * p->n + i];
                const int ix = pi[r * p->n + i];
                if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
            }
            out[2 * r] = bi;
            memcpy(&out[2 * r + 1], &bv, sizeof bv);
        }
    } else {
        snprintf(g->err, sizeof g->err, "no kernel %s", k);
        return -1;
    }
    return 0;
}

int gpu_dispatch(gpu_t *g, const char *kernel, const gpu_arg_t *args, int nargs,
                 uint32_t gx, uint32_t gy, uint32_t gz, uint32_t tx, uint32_t ty, uint32_t tz) {
    (void)gz; (void)tx; (void)ty; (void)tz;
    return run(g, kernel, args, nargs, gx, gy);
}
int gpu_dispatch_groups(gpu_t *g, const char *kernel, const gpu_arg_t *args, int nargs,
                        uint32_t groups_x, uint32_t groups_y, uint32_t groups_z, uint32_t tx, uint32_t ty, uint32_t tz) {
    (void)groups_z; (void)tx; (void)ty; (void)tz;
    return run(g, kernel, args, nargs, groups_x, groups_y);
}
int gpu_dispatch_groups_fc(gpu_t *g, const char *kernel, const uint32_t *fc, int nfc, const gpu_arg_t *args, int nargs,
                           uint32_t groups_x, uint32_t groups_y, uint32_t groups_z, uint32_t tx, uint32_t ty, uint32_t tz) {
    (void)fc; (void)nfc; (void)groups_z; (void)tx; (void)ty; (void)tz;
    return run(g, kernel, args, nargs, groups_x, groups_y);
}
