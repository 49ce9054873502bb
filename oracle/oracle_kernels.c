/* ORACLE — TEST INFRASTRUCTURE ONLY (see oracle.h). CPU restatement of src/kernels.metal.
   fp32 arithmetic throughout, bf16 weights widened exactly (value << 16). Sums use a fixed
   8-lane partial-sum order so results do not depend on the OpenMP thread count. */
#include "oracle.h"
#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf2f(uint16_t v) {
    union { uint32_t u; float f; } x;
    x.u = (uint32_t)v << 16;
    return x.f;
}
/* kernels.metal:6-7 */
static inline float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }
static inline float silu_f(float v) { return v / (1.0f + expf(-v)); }

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* sum_k a[k] * bf16(w[k]) with 8 fixed partial sums */
static float dot_bf16(const float *a, const uint16_t *w, int K) {
    float p[8] = { 0, 0, 0, 0, 0, 0, 0, 0 };
    int k = 0;
    for (; k + 8 <= K; k += 8)
        for (int j = 0; j < 8; ++j) p[j] += a[k + j] * bf2f(w[k + j]);
    for (; k < K; ++k) p[k & 7] += a[k] * bf2f(w[k]);
    return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
}
static float dot_f32(const float *a, const float *b, int K) {
    float p[8] = { 0, 0, 0, 0, 0, 0, 0, 0 };
    int k = 0;
    for (; k + 8 <= K; k += 8)
        for (int j = 0; j < 8; ++j) p[j] += a[k + j] * b[k + j];
    for (; k < K; ++k) p[k & 7] += a[k] * b[k];
    return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
}

/* gemm_bf16 / gemm_spec / gemm_mma (kernels.metal:12-48, 58-118, 132-208): all three compute
   C[m][n] (= or +=) alpha * act(sum_k A[m][k] * W[n][k] + bias[n]); epilogue order bias -> act
   -> *alpha -> store/accumulate (:39-44, :106-114, :193-201). GLU (act 3) pairs column n with
   n + N/2 and writes a * sigmoid(b) * alpha into N/2 columns (:96-104, :181-191). */
void or_gemm(const float *A, int lda, const uint16_t *W, int ldw, const float *bias, float *C, int ldc,
             int M, int N, int K, int act, int accumulate, float alpha) {
    const int glu = act == 3;
    const int nout = glu ? N / 2 : N;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < nout; ++n) {
        const uint16_t *wa = W + (size_t)n * ldw;
        const uint16_t *wb = glu ? W + (size_t)(n + N / 2) * ldw : NULL;
        for (int m = 0; m < M; ++m) {
            const float *a = A + (size_t)m * lda;
            float v;
            if (glu) {
                const float va = dot_bf16(a, wa, K) + (bias ? bias[n] : 0.0f);
                const float vb = dot_bf16(a, wb, K) + (bias ? bias[n + N / 2] : 0.0f);
                v = va * sigmoid_f(vb) * alpha;
            } else {
                v = dot_bf16(a, wa, K) + (bias ? bias[n] : 0.0f);
                if (act == 1) v = silu_f(v);
                else if (act == 2) v = v > 0.0f ? v : 0.0f;
                v *= alpha;
            }
            float *c = C + (size_t)m * ldc + n;
            *c = accumulate ? *c + v : v;
        }
    }
}

/* layernorm (kernels.metal:258-288): two-pass mean / variance, y = (x-mean)*inv*g + b,
   inv = 1/sqrt(var/D + eps). */
static void ln_row(const float *x, const float *g, const float *b, float *y, int D, float eps) {
    float s = 0.0f;
    for (int i = 0; i < D; ++i) s += x[i];
    const float mean = s / (float)D;
    float v = 0.0f;
    for (int i = 0; i < D; ++i) { const float d = x[i] - mean; v += d * d; }
    const float inv = 1.0f / sqrtf(v / (float)D + eps);
    for (int i = 0; i < D; ++i) y[i] = (x[i] - mean) * inv * g[i] + b[i];
}
void or_layernorm(const float *X, const float *g, const float *b, float *Y, int M, int D, float eps) {
    for (int m = 0; m < M; ++m) ln_row(X + (size_t)m * D, g, b, Y + (size_t)m * D, D, eps);
}
/* layernorm2 (kernels.metal:212-255): Y1 = LN(X; g1,b1), Y2 = LN(Y1; g2,b2). */
void or_layernorm2(const float *X, const float *g1, const float *b1, const float *g2, const float *b2,
                   float *Y1, float *Y2, int M, int D, float eps) {
    for (int m = 0; m < M; ++m) {
        ln_row(X + (size_t)m * D, g1, b1, Y1 + (size_t)m * D, D, eps);
        ln_row(Y1 + (size_t)m * D, g2, b2, Y2 + (size_t)m * D, D, eps);
    }
}

/* attention_rel (kernels.metal:293-348). For head h and query i (of c), keys j < L:
   s_j = ((q+u).k_j + (q+v).P[prow]) * scale with prow = (Lmax - L) + (c - 1 - i + j)
   (:317); softmax over all L keys, no mask (:327-345); O[i][h*dh+d] = sum_j p_j V[j][h*dh+d]. */
void or_attention_rel(const float *Q, int ldq, const float *K, const float *V, int ldk, const float *P,
                      const float *bias_u, const float *bias_v, float *O, int c, int L, int Lmax, int H, int dh, int D, float scale) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h) {
        for (int i = 0; i < c; ++i) {
            const int off = h * dh;
            float qu[1024], qv[1024], s[256];
            for (int d = 0; d < dh; ++d) {
                const float q = Q[(size_t)i * ldq + off + d];
                qu[d] = q + bias_u[off + d];
                qv[d] = q + bias_v[off + d];
            }
            float mx = -INFINITY;
            for (int j = 0; j < L; ++j) {
                const int prow = (Lmax - L) + (c - 1 - i + j);
                const float a = dot_f32(qu, K + (size_t)j * ldk + off, dh) + dot_f32(qv, P + (size_t)prow * D + off, dh);
                s[j] = a * scale;
                if (s[j] > mx) mx = s[j];
            }
            float sum = 0.0f;
            for (int j = 0; j < L; ++j) { s[j] = expf(s[j] - mx); sum += s[j]; }
            for (int j = 0; j < L; ++j) s[j] = s[j] / sum;
            for (int d = 0; d < dh; ++d) {
                float acc = 0.0f;
                for (int j = 0; j < L; ++j) acc += s[j] * V[(size_t)j * ldk + off + d];
                O[(size_t)i * D + off + d] = acc;
            }
        }
    }
}

/* dwconv_ln_silu (kernels.metal:361-409): y[t][ch] = SiLU(LN_ch(sum_tap W[ch][tap] *
   din[t+tap][ch])) where din row 0 is taps-1 rows before the first output row. */
void or_dwconv_ln_silu(const float *din, const float *W, const float *g, const float *b, float *Y, int c, int D, int taps, float eps) {
    float v[8192];
    for (int t = 0; t < c; ++t) {
        for (int ch = 0; ch < D; ++ch) {
            float acc = 0.0f;
            for (int tap = 0; tap < taps; ++tap) acc += W[(size_t)ch * taps + tap] * din[(size_t)(t + tap) * D + ch];
            v[ch] = acc;
        }
        float s = 0.0f;
        for (int ch = 0; ch < D; ++ch) s += v[ch];
        const float mean = s / (float)D;
        float var = 0.0f;
        for (int ch = 0; ch < D; ++ch) { const float d = v[ch] - mean; var += d * d; }
        const float inv = 1.0f / sqrtf(var / (float)D + eps);
        for (int ch = 0; ch < D; ++ch) Y[(size_t)t * D + ch] = silu_f((v[ch] - mean) * inv * g[ch] + b[ch]);
    }
}

/* conv2d_c1_s2_relu (kernels.metal:413-432): 1 -> C channels, 3x3 stride 2, causal padding
   (input index 2*o + k - 2, zero outside), ReLU. X [T][F] -> Y [T1][F1][C]. */
void or_conv2d_c1_s2_relu(const float *X, const float *W, const float *bias, float *Y, int T, int F, int T1, int F1, int C) {
#pragma omp parallel for schedule(static)
    for (int t1 = 0; t1 < T1; ++t1)
        for (int f1 = 0; f1 < F1; ++f1)
            for (int o = 0; o < C; ++o) {
                float acc = bias[o];
                for (int kh = 0; kh < 3; ++kh) {
                    const int ti = 2 * t1 + kh - 2;
                    if (ti < 0 || ti >= T) continue;
                    for (int kw = 0; kw < 3; ++kw) {
                        const int fi = 2 * f1 + kw - 2;
                        if (fi < 0 || fi >= F) continue;
                        acc += W[o * 9 + kh * 3 + kw] * X[(size_t)ti * F + fi];
                    }
                }
                Y[((size_t)t1 * F1 + f1) * C + o] = acc > 0.0f ? acc : 0.0f;
            }
}

/* dwconv2d_s2 (kernels.metal:435-454): depthwise 3x3 stride 2, same padding, no activation. */
void or_dwconv2d_s2(const float *X, const float *W, const float *bias, float *Y, int T, int F, int T1, int F1, int C) {
#pragma omp parallel for schedule(static)
    for (int t1 = 0; t1 < T1; ++t1)
        for (int f1 = 0; f1 < F1; ++f1)
            for (int ch = 0; ch < C; ++ch) {
                float acc = bias[ch];
                for (int kh = 0; kh < 3; ++kh) {
                    const int ti = 2 * t1 + kh - 2;
                    if (ti < 0 || ti >= T) continue;
                    for (int kw = 0; kw < 3; ++kw) {
                        const int fi = 2 * f1 + kw - 2;
                        if (fi < 0 || fi >= F) continue;
                        acc += W[ch * 9 + kh * 3 + kw] * X[((size_t)ti * F + fi) * C + ch];
                    }
                }
                Y[((size_t)t1 * F1 + f1) * C + ch] = acc;
            }
}

/* flatten_cf (kernels.metal:457-462): [T][F][C] -> [T][C*F], channel-major. */
void or_flatten_cf(const float *X, float *Y, int T, int F, int C) {
    for (int t = 0; t < T; ++t)
        for (int f = 0; f < F; ++f)
            for (int c = 0; c < C; ++c) Y[(size_t)t * C * F + (size_t)c * F + f] = X[((size_t)t * F + f) * C + c];
}

/* lstm_cell (kernels.metal:475-486): gates in i, f, g, o order. */
void or_lstm_cell(const float *gates, const float *c_in, float *c_out, float *h_out, int H) {
    for (int i = 0; i < H; ++i) {
        const float ig = sigmoid_f(gates[i]);
        const float fg = sigmoid_f(gates[H + i]);
        const float gg = tanhf(gates[2 * H + i]);
        const float og = sigmoid_f(gates[3 * H + i]);
        const float c = fg * c_in[i] + ig * gg;
        c_out[i] = c;
        h_out[i] = og * tanhf(c);
    }
}

/* joint_partial + argmax_reduce (kernels.metal:490-550): logits = W . relu(enc + pred) + b,
   argmax with ties going to the lowest index. */
void or_joint_argmax(const float *enc, int enc_ld, const float *pred, const uint16_t *W, const float *bias,
                     int V, int H, int rows, int *out_idx, float *out_val, float *out_margin) {
    for (int r = 0; r < rows; ++r) {
        float x[4096];
        const float *e = enc + (size_t)r * enc_ld;
        for (int i = 0; i < H; ++i) { const float v = e[i] + pred[i]; x[i] = v > 0.0f ? v : 0.0f; }
        float bv = -INFINITY, sv = -INFINITY;
        int bi = 0x7fffffff;
        for (int n = 0; n < V; ++n) {
            const float acc = dot_bf16(x, W + (size_t)n * H, H) + bias[n];
            if (acc > bv || (acc == bv && n < bi)) { sv = bv; bv = acc; bi = n; }
            else if (acc > sv) sv = acc;
        }
        out_idx[r] = bi;
        out_val[r] = bv;
        if (out_margin) out_margin[r] = bv - sv;
    }
}
