// LayerNorms, the conv-module depthwise conv + LN + SiLU, and the subsampling convolutions.
#include "common.cuh"

namespace {

constexpr int LNT = 256;   // threads per row
constexpr int LN_MAXV = 16; // D <= 4096

// src/kernels.metal:258-288: mean, then variance of (x - mean), inv = 1/sqrt(var/D + eps).
__device__ __forceinline__ void ln_vals(float (&v)[LN_MAXV], int D, const float *g, const float *b, float eps, float *red) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; if (i < D) s += v[k]; }
    const float mean = nb::block_sum<LNT>(s, red) / (float)D;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; if (i < D) { const float d = v[k] - mean; q += d * d; } }
    const float var = nb::block_sum<LNT>(q, red);
    const float inv = 1.0f / sqrtf(var / (float)D + eps);
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; if (i < D) v[k] = (v[k] - mean) * inv * g[i] + b[i]; }
}

__global__ void __launch_bounds__(LNT) layernorm_kernel(const float *__restrict__ X, const float *__restrict__ g, const float *__restrict__ b,
                                                        void *Y, int y_fmt, int64_t y_plane, int D, float eps) {
    __shared__ float red[LNT / 32];
    nb::pdl_wait();
    const int64_t row = blockIdx.x;
    float v[LN_MAXV];
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; v[k] = i < D ? X[row * D + i] : 0.0f; }
    ln_vals(v, D, g, b, eps, red);
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; if (i < D) nb::store_act(Y, y_fmt, y_plane, row * D + i, v[k]); }
}

// src/kernels.metal:212-255
__global__ void __launch_bounds__(LNT) layernorm2_kernel(const float *__restrict__ X, const float *__restrict__ g1, const float *__restrict__ b1,
                                                         const float *__restrict__ g2, const float *__restrict__ b2, float *Y1, void *Y2,
                                                         int y2_fmt, int64_t y2_plane, int D, float eps) {
    __shared__ float red[LNT / 32];
    nb::pdl_wait();
    const int64_t row = blockIdx.x;
    float v[LN_MAXV];
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; v[k] = i < D ? X[row * D + i] : 0.0f; }
    ln_vals(v, D, g1, b1, eps, red);
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; if (i < D) Y1[row * D + i] = v[k]; }
    ln_vals(v, D, g2, b2, eps, red);
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) { const int i = threadIdx.x + k * LNT; if (i < D) nb::store_act(Y2, y2_fmt, y2_plane, row * D + i, v[k]); }
}

// src/kernels.metal:361-409: causal depthwise conv over taps rows (history already in din),
// LayerNorm over channels, SiLU. One block per (stream, output row).
__global__ void __launch_bounds__(LNT) dwconv_ln_silu_kernel(const float *__restrict__ din, int64_t din_sstride, const int *pos_p,
                                                             const float *__restrict__ W, const float *__restrict__ g, const float *__restrict__ b,
                                                             void *Y, int y_fmt, int64_t y_plane, int c, int D, int taps, float eps) {
    __shared__ float red[LNT / 32];
    nb::pdl_wait();
    const int s = blockIdx.y, t = blockIdx.x;
    const float *x = din + (int64_t)s * din_sstride + (int64_t)(*pos_p - (taps - 1) + t) * D;
    float v[LN_MAXV];
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) {
        const int ch = threadIdx.x + k * LNT;
        float acc = 0.0f;
        if (ch < D)
            for (int tap = 0; tap < taps; ++tap) acc += W[ch * taps + tap] * x[(int64_t)tap * D + ch];
        v[k] = acc;
    }
    ln_vals(v, D, g, b, eps, red);
    const int64_t row = (int64_t)s * c + t;
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) {
        const int ch = threadIdx.x + k * LNT;
        if (ch < D) nb::store_act(Y, y_fmt, y_plane, row * D + ch, nb::silu_f(v[k]));
    }
}

// src/kernels.metal:413-432: 1 -> C channels, 3x3 stride 2, input index 2*o + k - 2, ReLU.
// One thread per output (channel fastest, so stores coalesce).
__global__ void conv2d_c1_s2_relu_kernel(const float *__restrict__ X, int64_t x_sstride, const float *__restrict__ W, const float *__restrict__ bias,
                                         float *Y, int T, int F, int T1, int F1, int C, int64_t total) {
    nb::pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int o = (int)(i % C);
        int64_t r = i / C;
        const int f1 = (int)(r % F1);
        r /= F1;
        const int t1 = (int)(r % T1);
        const int s = (int)(r / T1);
        const float *x = X + (int64_t)s * x_sstride;
        float acc = bias[o];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            const int ti = 2 * t1 + kh - 2;
            if (ti < 0 || ti >= T) continue;
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                const int fi = 2 * f1 + kw - 2;
                if (fi < 0 || fi >= F) continue;
                acc += W[o * 9 + kh * 3 + kw] * x[(int64_t)ti * F + fi];
            }
        }
        Y[i] = fmaxf(acc, 0.0f);
    }
}

// src/kernels.metal:435-454: depthwise 3x3 stride 2, same padding, no activation.
__global__ void dwconv2d_s2_kernel(const float *__restrict__ X, const float *__restrict__ W, const float *__restrict__ bias, void *Y,
                                   int y_fmt, int64_t y_plane, int T, int F, int T1, int F1, int C, int64_t total) {
    nb::pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int ch = (int)(i % C);
        int64_t r = i / C;
        const int f1 = (int)(r % F1);
        r /= F1;
        const int t1 = (int)(r % T1);
        const int s = (int)(r / T1);
        const float *x = X + (int64_t)s * T * F * C;
        float acc = bias[ch];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            const int ti = 2 * t1 + kh - 2;
            if (ti < 0 || ti >= T) continue;
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                const int fi = 2 * f1 + kw - 2;
                if (fi < 0 || fi >= F) continue;
                acc += W[ch * 9 + kh * 3 + kw] * x[((int64_t)ti * F + fi) * C + ch];
            }
        }
        nb::store_act(Y, y_fmt, y_plane, i, acc);
    }
}

// The first two subsampling stages fused: conv2d_c1_s2_relu (src/kernels.metal:413-432) then
// dwconv2d_s2 (src/kernels.metal:435-454), without materialising the first stage's output.
// Output (t2, f2) needs first-stage outputs t1 = 2*t2-2+kh, f1 = 2*f2-2+kw (zero when outside
// [0,T1) x [0,F1): the depthwise conv's padding), which need input rows 2*t1-2..2*t1 and columns
// 2*f1-2..2*f1: a 7x7 input patch starting at (4*t2-6, 4*f2-6). One warp per output position;
// the patch sits in shared memory; lanes take channels ch = lane, lane+32, ...
__global__ void __launch_bounds__(256) subsample_front_kernel(const float *__restrict__ X, int64_t x_sstride, const float *__restrict__ W0,
                                                              const float *__restrict__ b0, const float *__restrict__ W2, const float *__restrict__ b2,
                                                              void *Y, int y_fmt, int64_t y_plane, int T, int F, int T1, int F1, int T2, int F2, int C,
                                                              int64_t positions) {
    __shared__ float patch[8][49];
    nb::pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t pidx = (int64_t)blockIdx.x * 8 + warp;
    if (pidx >= positions) return;
    const int f2 = (int)(pidx % F2);
    const int64_t r = pidx / F2;
    const int t2 = (int)(r % T2), s = (int)(r / T2);
    const float *x = X + (int64_t)s * x_sstride;
    const int tx0 = 4 * t2 - 6, fx0 = 4 * f2 - 6;
    for (int e = lane; e < 49; e += 32) {
        const int ti = tx0 + e / 7, fi = fx0 + e % 7;
        patch[warp][e] = (ti >= 0 && ti < T && fi >= 0 && fi < F) ? x[(int64_t)ti * F + fi] : 0.0f;
    }
    __syncwarp();
    const float *pt = patch[warp];
    for (int ch = lane; ch < C; ch += 32) {
        float w0[9], w2[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) { w0[k] = W0[ch * 9 + k]; w2[k] = W2[ch * 9 + k]; }
        const float bb0 = b0[ch];
        float acc = b2[ch];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            const int t1 = 2 * t2 - 2 + kh;
            if (t1 < 0 || t1 >= T1) continue;
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                const int f1 = 2 * f2 - 2 + kw;
                if (f1 < 0 || f1 >= F1) continue;
                // first-stage output at (t1, f1): input rows 2*t1-2+a, columns 2*f1-2+b, i.e.
                // patch rows 2*kh + a and columns 2*kw + b
                float c0 = bb0;
#pragma unroll
                for (int a = 0; a < 3; ++a)
#pragma unroll
                    for (int b = 0; b < 3; ++b) c0 += w0[a * 3 + b] * pt[(2 * kh + a) * 7 + 2 * kw + b];
                acc += w2[kh * 3 + kw] * fmaxf(c0, 0.0f);
            }
        }
        nb::store_act(Y, y_fmt, y_plane, pidx * C + ch, acc);
    }
}

// flatten_cf (src/kernels.metal:457-462) of rows [lo, lo + c) only: Y[s*c + i][ch*F + f] =
// X[s][lo + i][f][ch]. Thread per output element (f fastest within a channel).
__global__ void flatten_rows_kernel(const float *__restrict__ X, void *Y, int y_fmt, int64_t y_plane, const int *lo_p, int T, int F, int C, int c,
                                    int64_t total) {
    nb::pdl_wait();
    const int lo = *lo_p;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int col = (int)(i % ((int64_t)C * F));
        const int64_t row = i / ((int64_t)C * F);
        const int ch = col / F, f = col - ch * F;
        const int s = (int)(row / c), r = (int)(row - (int64_t)s * c);
        nb::store_act(Y, y_fmt, y_plane, i, X[(((int64_t)s * T + lo + r) * F + f) * C + ch]);
    }
}

}  // namespace

static int grid_for(int64_t total) {
    int64_t g = (total + 255) / 256;
    return (int)(g < 148 * 16 ? g : 148 * 16);
}

extern "C" int nemo_layernorm(const float *X, const float *g, const float *b, void *Y, int y_fmt, int64_t y_plane, int M, int D, float eps, void *stream) {
    if (D > LNT * LN_MAXV) return nb_set_error("nemo_layernorm: D=%d too large", D);
    if (M <= 0) return 0;
    layernorm_kernel<<<M, LNT, 0, (cudaStream_t)stream>>>(X, g, b, Y, y_fmt, y_plane, D, eps);
    return nb_check_launch("layernorm_kernel");
}

extern "C" int nemo_layernorm2(const float *X, const float *g1, const float *b1, const float *g2, const float *b2, float *Y1, void *Y2,
                               int y2_fmt, int64_t y2_plane, int M, int D, float eps, void *stream) {
    if (D > LNT * LN_MAXV) return nb_set_error("nemo_layernorm2: D=%d too large", D);
    if (M <= 0) return 0;
    layernorm2_kernel<<<M, LNT, 0, (cudaStream_t)stream>>>(X, g1, b1, g2, b2, Y1, Y2, y2_fmt, y2_plane, D, eps);
    return nb_check_launch("layernorm2_kernel");
}

extern "C" int nemo_dwconv_ln_silu(const float *din, int64_t din_sstride, const int *pos, const float *W, const float *g, const float *b, void *Y,
                                   int y_fmt, int64_t y_plane, int streams, int c, int D, int taps, float eps, void *stream) {
    if (D > LNT * LN_MAXV) return nb_set_error("nemo_dwconv_ln_silu: D=%d too large", D);
    if (streams <= 0 || c <= 0) return 0;
    dwconv_ln_silu_kernel<<<dim3(c, streams), LNT, 0, (cudaStream_t)stream>>>(din, din_sstride, pos, W, g, b, Y, y_fmt, y_plane, c, D, taps, eps);
    return nb_check_launch("dwconv_ln_silu_kernel");
}

extern "C" int nemo_conv2d_c1_s2_relu(const float *X, int64_t x_sstride, const float *W, const float *bias, float *Y, int streams, int T, int F,
                                      int T1, int F1, int C, void *stream) {
    const int64_t total = (int64_t)streams * T1 * F1 * C;
    if (total <= 0) return 0;
    conv2d_c1_s2_relu_kernel<<<grid_for(total), 256, 0, (cudaStream_t)stream>>>(X, x_sstride, W, bias, Y, T, F, T1, F1, C, total);
    return nb_check_launch("conv2d_c1_s2_relu_kernel");
}

extern "C" int nb_dwconv2d_s2_fmt(const float *X, const float *W, const float *bias, void *Y, int y_fmt, int64_t y_plane, int streams, int T, int F,
                                  int T1, int F1, int C, void *stream) {
    const int64_t total = (int64_t)streams * T1 * F1 * C;
    if (total <= 0) return 0;
    dwconv2d_s2_kernel<<<grid_for(total), 256, 0, (cudaStream_t)stream>>>(X, W, bias, Y, y_fmt, y_plane, T, F, T1, F1, C, total);
    return nb_check_launch("dwconv2d_s2_kernel");
}

extern "C" int nemo_dwconv2d_s2(const float *X, const float *W, const float *bias, float *Y, int streams, int T, int F, int T1, int F1, int C, void *stream) {
    return nb_dwconv2d_s2_fmt(X, W, bias, Y, NEMO_FMT_F32, 0, streams, T, F, T1, F1, C, stream);
}

extern "C" int nemo_subsample_front(const float *X, int64_t x_sstride, const float *W0, const float *b0, const float *W2, const float *b2, void *Y,
                                    int y_fmt, int64_t y_plane, int streams, int T, int F, int C, void *stream) {
    const int T1 = T / 2 + 1, F1 = F / 2 + 1, T2 = T1 / 2 + 1, F2 = F1 / 2 + 1;
    const int64_t positions = (int64_t)streams * T2 * F2;
    if (positions <= 0) return 0;
    subsample_front_kernel<<<(unsigned)((positions + 7) / 8), 256, 0, (cudaStream_t)stream>>>(X, x_sstride, W0, b0, W2, b2, Y, y_fmt, y_plane, T, F, T1,
                                                                                              F1, T2, F2, C, positions);
    return nb_check_launch("subsample_front_kernel");
}

extern "C" int nb_flatten_rows_fmt(const float *X, void *Y, int y_fmt, int64_t y_plane, const int *lo, int streams, int T, int F, int C, int c, void *stream) {
    const int64_t total = (int64_t)streams * c * C * F;
    if (total <= 0) return 0;
    flatten_rows_kernel<<<grid_for(total), 256, 0, (cudaStream_t)stream>>>(X, Y, y_fmt, y_plane, lo, T, F, C, c, total);
    return nb_check_launch("flatten_rows_kernel");
}

extern "C" int nemo_flatten_rows(const float *X, float *Y, const int *lo, int streams, int T, int F, int C, int c, void *stream) {
    return nb_flatten_rows_fmt(X, Y, NEMO_FMT_F32, 0, lo, streams, T, F, C, c, stream);
}
