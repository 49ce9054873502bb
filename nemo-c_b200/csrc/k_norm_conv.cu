// LayerNorms, the conv-module depthwise conv + LN + SiLU, and the subsampling convolutions.
#include <cuda_bf16.h>
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

// The same by output rows: one block per (stream, output row t1), threads over channels (weights
// in registers), looping over the row's columns; no per-element index arithmetic.
__global__ void __launch_bounds__(256) dwconv2d_s2_rows_kernel(const float *__restrict__ X, const float *__restrict__ W, const float *__restrict__ bias,
                                                               void *Y, int y_fmt, int64_t y_plane, int T, int F, int T1, int F1, int C) {
    nb::pdl_wait();
    const int s = blockIdx.x / T1, t1 = blockIdx.x - s * T1;
    const float *x = X + (int64_t)s * T * F * C;
    for (int ch = threadIdx.x; ch < C; ch += blockDim.x) {
        float w[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = __ldg(W + ch * 9 + k);
        const float b = __ldg(bias + ch);
        for (int f1 = 0; f1 < F1; ++f1) {
            float acc = b;
#pragma unroll
            for (int kh = 0; kh < 3; ++kh) {
                const int ti = 2 * t1 + kh - 2;
                if (ti < 0 || ti >= T) continue;
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    const int fi = 2 * f1 + kw - 2;
                    if (fi < 0 || fi >= F) continue;
                    acc += w[kh * 3 + kw] * x[((int64_t)ti * F + fi) * C + ch];
                }
            }
            nb::store_act(Y, y_fmt, y_plane, (((int64_t)s * T1 + t1) * F1 + f1) * C + ch, acc);
        }
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

// The same two stages computed by tiles: a block owns TR consecutive second-stage rows t2 of one
// stream and 32 channels. It stages the input rows those rows read (4 * TR + 3 rows, zero outside
// the input) in shared memory, computes every first-stage output they need once (2 * TR + 1 rows
// t1 x F1 columns x 32 channels, zero for t1 outside [0, T1): the depthwise conv's padding) into
// shared memory, and then the depthwise outputs from there. Each first-stage value is computed
// once per block instead of once per depthwise tap that reads it. Lanes are channels: input
// reads are broadcasts, first-stage reads and output stores are 32 consecutive channels.
constexpr int FT_TR = 4;         // second-stage rows per block

__device__ __forceinline__ void front_split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - __low2float(h), x1 - __high2float(h));
    hi = *(const uint32_t *)&h;
    lo = *(const uint32_t *)&l;
}
__device__ __forceinline__ void front_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
constexpr int FT_IN_W = 136;     // staged input columns: fi = -2 .. 133 (F <= 128 + 2 * (F1 - F / 2 - 1) checked on the host)

// First-stage rows in shared memory are F1 + 3 columns wide: f1 = -2 .. F1 (the depthwise conv's
// zero padding stored, so its taps need no bounds checks).
__host__ __device__ __forceinline__ size_t front_tile_smem(int F1) {
    return ((size_t)(4 * FT_TR + 3) * FT_IN_W + (size_t)(2 * FT_TR + 1) * (F1 + 3) * 32) * sizeof(float);
}

// FC: mel bins fixed at compile time (0: F at run time); BF: output as bf16 hi / lo planes.
template <int FC, bool BF>
__global__ void __launch_bounds__(256) subsample_front_tile_kernel(const float *__restrict__ X, int64_t x_sstride, const float *__restrict__ W0,
                                                                   const float *__restrict__ b0, const float *__restrict__ W2,
                                                                   const float *__restrict__ b2, void *Y, int64_t y_plane, int T, int Frt, int T1,
                                                                   int T2, int C) {
    extern __shared__ float fsm[];
    const int F = FC ? FC : Frt, F1 = F / 2 + 1, F2 = F1 / 2 + 1, CW = F1 + 3;
    float *xin = fsm, *c1 = fsm + (4 * FT_TR + 3) * FT_IN_W;  // c1[r][f1 + 2][32]
    nb::pdl_wait();
    const int tiles_t = (T2 + FT_TR - 1) / FT_TR;
    const int s = blockIdx.x / tiles_t, t2_0 = (blockIdx.x % tiles_t) * FT_TR;
    const int cb = blockIdx.y * 32, lane = threadIdx.x & 31, grp = threadIdx.x >> 5, ch = cb + lane;
    const float *x = X + (int64_t)s * x_sstride;
    // input rows ti = 4 * t2_0 - 6 + i, columns fi = j - 2
    const int ti0 = 4 * t2_0 - 6;
    constexpr int NIN = (4 * FT_TR + 3) * FT_IN_W, NPT = (NIN + 255) / 256;  // 256 threads
    float v[NPT];  // every load of the staging issued before the first store
#pragma unroll
    for (int q = 0; q < NPT; ++q) {
        const int e = threadIdx.x + q * 256, i = e / FT_IN_W, j = e - i * FT_IN_W, ti = ti0 + i, fi = j - 2;
        v[q] = (e < NIN && ti >= 0 && ti < T && fi >= 0 && fi < F) ? x[(int64_t)ti * F + fi] : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < NPT; ++q)
        if (threadIdx.x + q * 256 < NIN) xin[threadIdx.x + q * 256] = v[q];
    // the padding columns f1 = -2, -1, F1 of every first-stage row
    for (int e = threadIdx.x; e < (2 * FT_TR + 1) * 3 * 32; e += 256) {
        const int r = e / 96, q = (e / 32) % 3, l = e % 32;
        c1[(r * CW + (q < 2 ? q : F1 + 2)) * 32 + l] = 0.0f;
    }
    float w2[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) w2[k] = __ldg(W2 + ch * 9 + k);
    const float bb2 = __ldg(b2 + ch);
    // first-stage weights as the MMA's B operand (k = tap, n = channel), split into bf16 hi + lo:
    // b0 = (taps 2t, 2t + 1; channel g), b1 = (taps 2t + 8, 2t + 9; channel g) per 8-channel tile
    const int g = lane >> 2, t = lane & 3;
    uint32_t wbh[4][2], wbl[4][2];
    float bias0[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
        const float *wr = W0 + (cb + nt * 8 + g) * 9;
        const float k0a = __ldg(wr + 2 * t), k0b = __ldg(wr + 2 * t + 1);
        const float k1a = t == 0 ? __ldg(wr + 8) : 0.0f;
        front_split2(k0a, k0b, wbh[nt][0], wbl[nt][0]);
        front_split2(k1a, 0.0f, wbh[nt][1], wbl[nt][1]);
        bias0[nt][0] = __ldg(b0 + cb + nt * 8 + 2 * t);
        bias0[nt][1] = __ldg(b0 + cb + nt * 8 + 2 * t + 1);
    }
    __syncthreads();
    // first stage on the tensor cores: for positions p = r * F1 + f1 (t1 = 2 * t2_0 - 2 + r) the
    // 3 x 3 input patch (taps k = 3a + b, padded to 16) times the block's 32 channels, mma.sync
    // m16n8k16 on bf16 hi / lo splits of both operands (four products, fp32 accumulation); then
    // bias and ReLU, and zero for t1 outside [0, T1)
    const int P = (2 * FT_TR + 1) * F1;
    for (int mt = grp; mt * 16 < P; mt += 8) {
        uint32_t ah[4], al[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int pp = mt * 16 + g + 8 * (e & 1), k = 2 * t + 8 * (e >> 1);
            float v0 = 0.0f, v1 = 0.0f;
            if (pp < P) {
                const int r = pp / F1, f1 = pp - r * F1;
                const float *xr = xin + 2 * r * FT_IN_W + 2 * f1;
                if (k < 9) v0 = xr[(k / 3) * FT_IN_W + k % 3];
                if (k + 1 < 9) v1 = xr[((k + 1) / 3) * FT_IN_W + (k + 1) % 3];
            }
            front_split2(v0, v1, ah[e], al[e]);
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            float d[4] = { 0.f, 0.f, 0.f, 0.f };
            front_mma(d, al, wbl[nt][0], wbl[nt][1]);
            front_mma(d, al, wbh[nt][0], wbh[nt][1]);
            front_mma(d, ah, wbl[nt][0], wbl[nt][1]);
            front_mma(d, ah, wbh[nt][0], wbh[nt][1]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int pp = mt * 16 + g + 8 * h;
                if (pp >= P) continue;
                const int r = pp / F1, t1 = 2 * t2_0 - 2 + r;
                const bool okt = t1 >= 0 && t1 < T1;
                const int n = nt * 8 + 2 * t, idx = (r * CW + (pp - r * F1) + 2) * 32 + n;
                c1[idx] = okt ? fmaxf(d[2 * h] + bias0[nt][0], 0.0f) : 0.0f;
                c1[idx + 1] = okt ? fmaxf(d[2 * h + 1] + bias0[nt][1], 0.0f) : 0.0f;
            }
        }
    }
    __syncthreads();
    // depthwise stride-2 stage over the staged first-stage outputs
    for (int tr = 0; tr < FT_TR; ++tr) {
        const int t2 = t2_0 + tr;
        if (t2 >= T2) break;
        for (int f2 = grp; f2 < F2; f2 += 8) {
            float acc = bb2;
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) acc += w2[kh * 3 + kw] * c1[((2 * tr + kh) * CW + 2 * f2 + kw) * 32 + lane];  // f1 = 2 f2 - 2 + kw
            nb::store_act(Y, BF ? NEMO_FMT_BF16X2 : NEMO_FMT_F32, y_plane, (((int64_t)s * T2 + t2) * F2 + f2) * C + ch, acc);
        }
    }
}

// flatten_cf (src/kernels.metal:457-462) of rows [lo, lo + c) only: Y[s*c + i][ch*F + f] =
// X[s][lo + i][f][ch]. Thread per output element (f fastest within a channel).
// The same by rows: one block per output row (stream s, row r); the [F][C] source row is read
// coalesced into shared memory and written out in [C][F] order.
__global__ void __launch_bounds__(256) flatten_rows_smem_kernel(const float *__restrict__ X, void *Y, int y_fmt, int64_t y_plane, const int *lo_p, int T,
                                                                int F, int C, int c) {
    extern __shared__ float frow[];  // [F][C]
    nb::pdl_wait();
    const int lo = *lo_p;
    const int s = blockIdx.x / c, r = blockIdx.x - s * c, n = F * C;
    const float *src = X + ((int64_t)s * T + lo + r) * n;
    for (int e = threadIdx.x; e < n; e += blockDim.x) frow[e] = src[e];
    __syncthreads();
    const int64_t row = (int64_t)blockIdx.x * n;
    for (int e = threadIdx.x; e < n; e += blockDim.x) {
        const int ch = e / F, f = e - ch * F;
        nb::store_act(Y, y_fmt, y_plane, row + e, frow[f * C + ch]);
    }
}

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

// ---- warp-per-row variants (D <= 1024, D % 128 == 0): one wave for thousands of rows, shuffle-only
// reductions. Lane l holds columns 4 (l + 32 j) .. +3 for j < D / 128 (float4 loads).
constexpr int WROWS = 8;  // rows (warps) per block

template <int NV>
__device__ __forceinline__ void ln_warp(float4 (&v)[NV], int nv, int D, const float *__restrict__ g, const float *__restrict__ b, float eps) {
    const int lane = threadIdx.x & 31;
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) if (j < nv) s += v[j].x + v[j].y + v[j].z + v[j].w;
    const float mean = nb::warp_sum(s) / (float)D;
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
        if (j < nv) {
            const float a = v[j].x - mean, bb = v[j].y - mean, cc = v[j].z - mean, d = v[j].w - mean;
            q += a * a + bb * bb + cc * cc + d * d;
        }
    const float inv = 1.0f / sqrtf(nb::warp_sum(q) / (float)D + eps);
#pragma unroll
    for (int j = 0; j < NV; ++j)
        if (j < nv) {
            const int k = 4 * (lane + 32 * j);
            const float4 gg = __ldg((const float4 *)(g + k)), bv = __ldg((const float4 *)(b + k));
            v[j].x = (v[j].x - mean) * inv * gg.x + bv.x;
            v[j].y = (v[j].y - mean) * inv * gg.y + bv.y;
            v[j].z = (v[j].z - mean) * inv * gg.z + bv.z;
            v[j].w = (v[j].w - mean) * inv * gg.w + bv.w;
        }
}

__device__ __forceinline__ void store4(void *Y, int fmt, int64_t plane, int64_t idx, const float4 v) {
    if (fmt == NEMO_FMT_F32) {
        *(float4 *)((float *)Y + idx) = v;
    } else {
        const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
        const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - __low2float(h0), v.y - __high2float(h0));
        const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - __low2float(h1), v.w - __high2float(h1));
        uint16_t *y = (uint16_t *)Y + idx;
        *(uint2 *)y = make_uint2(*(const uint32_t *)&h0, *(const uint32_t *)&h1);
        *(uint2 *)(y + plane) = make_uint2(*(const uint32_t *)&l0, *(const uint32_t *)&l1);
    }
}

// Y = LN(X; g, b) (src/kernels.metal:258-288); with g2: Y1 = that, Y = LN(Y1; g2, b2) (:212-255).
__global__ void __launch_bounds__(WROWS * 32) layernorm_warp_kernel(const float *__restrict__ X, const float *__restrict__ g, const float *__restrict__ b,
                                                                    const float *__restrict__ g2, const float *__restrict__ b2, float *Y1, void *Y,
                                                                    int y_fmt, int64_t y_plane, int M, int D, float eps) {
    nb::pdl_wait();
    const int row = blockIdx.x * WROWS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    const int nv = D / 128;
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) if (j < nv) v[j] = *(const float4 *)(X + (int64_t)row * D + 4 * (lane + 32 * j));
    ln_warp<8>(v, nv, D, g, b, eps);
    if (g2) {
#pragma unroll
        for (int j = 0; j < 8; ++j) if (j < nv) *(float4 *)(Y1 + (int64_t)row * D + 4 * (lane + 32 * j)) = v[j];
        ln_warp<8>(v, nv, D, g2, b2, eps);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) if (j < nv) store4(Y, y_fmt, y_plane, (int64_t)row * D + 4 * (lane + 32 * j), v[j]);
}

// Two-pass LayerNorm of one 1024-wide row over a 128-thread block: thread t holds dims 4t .. 4t + 3
// (v0) and 512 + 4t .. + 3 (v1); the four warps' partial sums meet in shared memory.
__device__ __forceinline__ void ln_block1024x2(float4 &v0, float4 &v1, float4 g0, float4 g1, float4 b0, float4 b1, float eps, float (&red)[2][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float s = nb::warp_sum((v0.x + v0.y + v0.z + v0.w) + (v1.x + v1.y + v1.z + v1.w));
    if (lane == 0) red[0][warp] = s;
    __syncthreads();
    const float mean = (red[0][0] + red[0][1] + red[0][2] + red[0][3]) / 1024.0f;
    const float a0 = v0.x - mean, a1 = v0.y - mean, a2 = v0.z - mean, a3 = v0.w - mean;
    const float c0 = v1.x - mean, c1 = v1.y - mean, c2 = v1.z - mean, c3 = v1.w - mean;
    const float q = nb::warp_sum((a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3) + (c0 * c0 + c1 * c1 + c2 * c2 + c3 * c3));
    if (lane == 0) red[1][warp] = q;
    __syncthreads();
    const float inv = 1.0f / sqrtf((red[1][0] + red[1][1] + red[1][2] + red[1][3]) / 1024.0f + eps);
    v0 = make_float4(a0 * inv * g0.x + b0.x, a1 * inv * g0.y + b0.y, a2 * inv * g0.z + b0.z, a3 * inv * g0.w + b0.w);
    v1 = make_float4(c0 * inv * g1.x + b1.x, c1 * inv * g1.y + b1.y, c2 * inv * g1.z + b1.z, c3 * inv * g1.w + b1.w);
}

// LayerNorm (and the paired second LayerNorm of layernorm2) for D = 1024, one 128-thread block per
// row: every row of a 1792-row batch resident at once (16 blocks per SM), two barriers per LayerNorm
// among four warps. (One 256-thread block per row took 1.5 rounds of the SMs and 0.15 ms more per
// config #4 step over its 96 launches.)
__global__ void __launch_bounds__(128) layernorm_row128_kernel(const float *__restrict__ X, const float *__restrict__ g, const float *__restrict__ b,
                                                               const float *__restrict__ g2, const float *__restrict__ b2, float *Y1, void *Y, int y_fmt,
                                                               int64_t y_plane, float eps) {
    __shared__ float red[2][4];
    nb::pdl_wait();
    const int t4 = 4 * threadIdx.x;
    const int64_t base = (int64_t)blockIdx.x * 1024 + t4;
    float4 v0 = *(const float4 *)(X + base), v1 = *(const float4 *)(X + base + 512);
    const float4 ga = __ldg((const float4 *)(g + t4)), gb = __ldg((const float4 *)(g + t4 + 512));
    const float4 ba = __ldg((const float4 *)(b + t4)), bb = __ldg((const float4 *)(b + t4 + 512));
    ln_block1024x2(v0, v1, ga, gb, ba, bb, eps, red);
    if (g2) {
        *(float4 *)(Y1 + base) = v0;
        *(float4 *)(Y1 + base + 512) = v1;
        const float4 g2a = __ldg((const float4 *)(g2 + t4)), g2b = __ldg((const float4 *)(g2 + t4 + 512));
        const float4 b2a = __ldg((const float4 *)(b2 + t4)), b2b = __ldg((const float4 *)(b2 + t4 + 512));
        ln_block1024x2(v0, v1, g2a, g2b, b2a, b2b, eps, red);  // red is free again: every warp read it before the last barrier
    }
    store4(Y, y_fmt, y_plane, base, v0);
    store4(Y, y_fmt, y_plane, base + 512, v1);
}


// Causal depthwise conv + LN + SiLU (src/kernels.metal:361-409), one warp per (stream, row).
__global__ void __launch_bounds__(WROWS * 32) dwconv_ln_silu_warp_kernel(const float *__restrict__ din, int64_t din_sstride, const int *pos_p,
                                                                         const float *__restrict__ W, const float *__restrict__ g,
                                                                         const float *__restrict__ b, void *Y, int y_fmt, int64_t y_plane, int streams,
                                                                         int c, int D, int taps, float eps) {
    nb::pdl_wait();
    const int item = blockIdx.x * WROWS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (item >= streams * c) return;
    const int s = item / c, t = item - s * c;
    const float *x = din + (int64_t)s * din_sstride + (int64_t)(*pos_p - (taps - 1) + t) * D;
    const int nv = D / 128;
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (j < nv) {
            const int ch = 4 * (lane + 32 * j);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (taps == 9) {
                // the 4 channels' 36 taps are contiguous ([ch][9]) and 16-byte aligned: 9 vector loads
                float w[36];
#pragma unroll
                for (int q = 0; q < 9; ++q) {
                    const float4 t4 = __ldg((const float4 *)(W + ch * 9) + q);
                    w[4 * q] = t4.x; w[4 * q + 1] = t4.y; w[4 * q + 2] = t4.z; w[4 * q + 3] = t4.w;
                }
#pragma unroll
                for (int tap = 0; tap < 9; ++tap) {
                    const float4 xv = *(const float4 *)(x + (int64_t)tap * D + ch);
                    acc.x += w[tap] * xv.x;
                    acc.y += w[9 + tap] * xv.y;
                    acc.z += w[18 + tap] * xv.z;
                    acc.w += w[27 + tap] * xv.w;
                }
            } else {
                for (int tap = 0; tap < taps; ++tap) {
                    const float4 xv = *(const float4 *)(x + (int64_t)tap * D + ch);
                    acc.x += W[(ch + 0) * taps + tap] * xv.x;
                    acc.y += W[(ch + 1) * taps + tap] * xv.y;
                    acc.z += W[(ch + 2) * taps + tap] * xv.z;
                    acc.w += W[(ch + 3) * taps + tap] * xv.w;
                }
            }
            v[j] = acc;
        }
    ln_warp<8>(v, nv, D, g, b, eps);
    const int64_t row = (int64_t)s * c + t;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (j < nv) {
            float4 o = v[j];
            o.x = nb::silu_f(o.x); o.y = nb::silu_f(o.y); o.z = nb::silu_f(o.z); o.w = nb::silu_f(o.w);
            store4(Y, y_fmt, y_plane, row * D + 4 * (lane + 32 * j), o);
        }
}

}  // namespace

// warp-per-row kernels need D a multiple of 128 up to 1024, 16-byte aligned rows and planes
static bool warp_rows_ok(const void *X, const void *Y, int y_fmt, int64_t y_plane, int D) {
    return D % 128 == 0 && D <= 1024 && !((uintptr_t)X & 15) && !((uintptr_t)Y & 15) && (y_fmt == NEMO_FMT_F32 || y_plane % 8 == 0);
}

static int grid_for(int64_t total) {
    int64_t g = (total + 255) / 256;
    return (int)(g < 148 * 16 ? g : 148 * 16);
}

extern "C" int nemo_layernorm(const float *X, const float *g, const float *b, void *Y, int y_fmt, int64_t y_plane, int M, int D, float eps, void *stream) {
    if (D > LNT * LN_MAXV) return nb_set_error("nemo_layernorm: D=%d too large", D);
    if (M <= 0) return 0;
    if (D == 1024 && warp_rows_ok(X, Y, y_fmt, y_plane, D)) {
        nb::launch(layernorm_row128_kernel, M, 128, 0, (cudaStream_t)stream, X, g, b, nullptr, nullptr, nullptr, Y, y_fmt, y_plane, eps);
        return nb_check_launch("layernorm_row128_kernel");
    }
    if (warp_rows_ok(X, Y, y_fmt, y_plane, D)) {
        nb::launch(layernorm_warp_kernel, (M + WROWS - 1) / WROWS, WROWS * 32, 0, (cudaStream_t)stream, X, g, b, nullptr, nullptr, nullptr, Y, y_fmt, y_plane, M, D,
                                                                                              eps);
        return nb_check_launch("layernorm_warp_kernel");
    }
    nb::launch(layernorm_kernel, M, LNT, 0, (cudaStream_t)stream, X, g, b, Y, y_fmt, y_plane, D, eps);
    return nb_check_launch("layernorm_kernel");
}

extern "C" int nemo_layernorm2(const float *X, const float *g1, const float *b1, const float *g2, const float *b2, float *Y1, void *Y2,
                               int y2_fmt, int64_t y2_plane, int M, int D, float eps, void *stream) {
    if (D > LNT * LN_MAXV) return nb_set_error("nemo_layernorm2: D=%d too large", D);
    if (M <= 0) return 0;
    if (D == 1024 && warp_rows_ok(X, Y2, y2_fmt, y2_plane, D) && !((uintptr_t)Y1 & 15)) {
        nb::launch(layernorm_row128_kernel, M, 128, 0, (cudaStream_t)stream, X, g1, b1, g2, b2, Y1, Y2, y2_fmt, y2_plane, eps);
        return nb_check_launch("layernorm_row128_kernel");
    }
    if (warp_rows_ok(X, Y2, y2_fmt, y2_plane, D) && !((uintptr_t)Y1 & 15)) {
        nb::launch(layernorm_warp_kernel, (M + WROWS - 1) / WROWS, WROWS * 32, 0, (cudaStream_t)stream, X, g1, b1, g2, b2, Y1, Y2, y2_fmt, y2_plane, M, D, eps);
        return nb_check_launch("layernorm_warp_kernel");
    }
    nb::launch(layernorm2_kernel, M, LNT, 0, (cudaStream_t)stream, X, g1, b1, g2, b2, Y1, Y2, y2_fmt, y2_plane, D, eps);
    return nb_check_launch("layernorm2_kernel");
}

// The same for D = 1024 and 9 taps with one block (8 warps) per output row: warp j owns channels
// [128 j, 128 j + 128), so each thread has only its 4 channels' 9 weight and 9 input vectors to
// load (all in flight at once), and the two-pass LayerNorm reduces across the warps in shared
// memory. Eight times the warps of the warp-per-row kernel for the same rows.
__global__ void __launch_bounds__(256) dwconv_ln_silu_row_kernel(const float *__restrict__ din, int64_t din_sstride, const int *pos_p,
                                                                 const float *__restrict__ W, const float *__restrict__ g, const float *__restrict__ b,
                                                                 void *Y, int y_fmt, int64_t y_plane, int c, float eps) {
    constexpr int D = 1024, TAPS = 9;
    __shared__ float red[2][8];
    nb::pdl_wait();
    const int item = blockIdx.x, s = item / c, t = item - s * c;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, ch = 4 * (lane + 32 * warp);
    const float *x = din + (int64_t)s * din_sstride + (int64_t)(*pos_p - (TAPS - 1) + t) * D;
    float4 wv[TAPS], xv[TAPS];
#pragma unroll
    for (int q = 0; q < TAPS; ++q) wv[q] = __ldg((const float4 *)(W + ch * TAPS) + q);  // the 4 channels' 36 taps, [ch][9]
#pragma unroll
    for (int tap = 0; tap < TAPS; ++tap) xv[tap] = *(const float4 *)(x + (int64_t)tap * D + ch);
    const float4 gg = __ldg((const float4 *)(g + ch)), bv = __ldg((const float4 *)(b + ch));
    const float *w = (const float *)wv;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int tap = 0; tap < TAPS; ++tap) {
        acc.x += w[tap] * xv[tap].x;
        acc.y += w[9 + tap] * xv[tap].y;
        acc.z += w[18 + tap] * xv[tap].z;
        acc.w += w[27 + tap] * xv[tap].w;
    }
    float sum = nb::warp_sum(acc.x + acc.y + acc.z + acc.w);
    if (lane == 0) red[0][warp] = sum;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[0][i];
    const float mean = tot / (float)D;
    const float a0 = acc.x - mean, a1 = acc.y - mean, a2 = acc.z - mean, a3 = acc.w - mean;
    float q = nb::warp_sum(a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3);
    if (lane == 0) red[1][warp] = q;
    __syncthreads();
    float qt = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) qt += red[1][i];
    const float inv = 1.0f / sqrtf(qt / (float)D + eps);
    float4 o;
    o.x = nb::silu_f(a0 * inv * gg.x + bv.x);
    o.y = nb::silu_f(a1 * inv * gg.y + bv.y);
    o.z = nb::silu_f(a2 * inv * gg.z + bv.z);
    o.w = nb::silu_f(a3 * inv * gg.w + bv.w);
    store4(Y, y_fmt, y_plane, (int64_t)item * D + ch, o);
}

// The same for all c <= 8 rows of a stream at once: one block per stream, thread = four channels.
// The stream's c + 8 input rows are read once (the row kernel reads 9 rows for each output row,
// ~9x the L2 traffic), the taps once per block; both LayerNorm passes reduce all rows together
// (two CTA barriers per block instead of two per row).
constexpr int DW_CM = 8;  // rows per stream at most
__global__ void __launch_bounds__(256) dwconv_ln_silu_stream_kernel(const float *__restrict__ din, int64_t din_sstride, const int *pos_p,
                                                                    const float *__restrict__ W, const float *__restrict__ g, const float *__restrict__ b,
                                                                    void *Y, int y_fmt, int64_t y_plane, int c, float eps) {
    constexpr int D = 1024, TAPS = 9, R = DW_CM + TAPS - 1;
    __shared__ float red[2][8][DW_CM];
    nb::pdl_wait();
    const int s = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, ch = 4 * threadIdx.x;
    const float *x = din + (int64_t)s * din_sstride + (int64_t)(*pos_p - (TAPS - 1)) * D + ch;
    float4 xv[R], wv[TAPS];
#pragma unroll
    for (int r = 0; r < R; ++r) xv[r] = r < c + TAPS - 1 ? *(const float4 *)(x + (int64_t)r * D) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < TAPS; ++q) wv[q] = __ldg((const float4 *)(W + ch * TAPS) + q);  // the 4 channels' 36 taps, [ch][9]
    const float4 gg = __ldg((const float4 *)(g + ch)), bv = __ldg((const float4 *)(b + ch));
    const float *w = (const float *)wv;
    float4 acc[DW_CM];
#pragma unroll
    for (int t = 0; t < DW_CM; ++t) {
        acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int tap = 0; tap < TAPS; ++tap) {  // output row t reads input rows t .. t + 8
            acc[t].x += w[tap] * xv[t + tap].x;
            acc[t].y += w[9 + tap] * xv[t + tap].y;
            acc[t].z += w[18 + tap] * xv[t + tap].z;
            acc[t].w += w[27 + tap] * xv[t + tap].w;
        }
        const float sum = nb::warp_sum((acc[t].x + acc[t].y) + (acc[t].z + acc[t].w));
        if (lane == 0) red[0][warp][t] = sum;
    }
    __syncthreads();
    float q[DW_CM];
#pragma unroll
    for (int t = 0; t < DW_CM; ++t) {
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) tot += red[0][i][t];
        const float mean = tot / (float)D;
        acc[t].x -= mean; acc[t].y -= mean; acc[t].z -= mean; acc[t].w -= mean;
        q[t] = nb::warp_sum(acc[t].x * acc[t].x + acc[t].y * acc[t].y + acc[t].z * acc[t].z + acc[t].w * acc[t].w);
        if (lane == 0) red[1][warp][t] = q[t];
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < DW_CM; ++t) {
        if (t >= c) break;
        float qt = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) qt += red[1][i][t];
        const float inv = 1.0f / sqrtf(qt / (float)D + eps);
        float4 o;
        o.x = nb::silu_f(acc[t].x * inv * gg.x + bv.x);
        o.y = nb::silu_f(acc[t].y * inv * gg.y + bv.y);
        o.z = nb::silu_f(acc[t].z * inv * gg.z + bv.z);
        o.w = nb::silu_f(acc[t].w * inv * gg.w + bv.w);
        store4(Y, y_fmt, y_plane, ((int64_t)s * c + t) * D + ch, o);
    }
}

extern "C" int nemo_dwconv_ln_silu(const float *din, int64_t din_sstride, const int *pos, const float *W, const float *g, const float *b, void *Y,
                                   int y_fmt, int64_t y_plane, int streams, int c, int D, int taps, float eps, void *stream) {
    if (D > LNT * LN_MAXV) return nb_set_error("nemo_dwconv_ln_silu: D=%d too large", D);
    if (streams <= 0 || c <= 0) return 0;
    if (D == 1024 && taps == 9 && c <= DW_CM && warp_rows_ok(din, Y, y_fmt, y_plane, D) && din_sstride % 4 == 0 && !((uintptr_t)W & 15)) {
        nb::launch(dwconv_ln_silu_stream_kernel, streams, 256, 0, (cudaStream_t)stream, din, din_sstride, pos, W, g, b, Y, y_fmt, y_plane, c, eps);
        return nb_check_launch("dwconv_ln_silu_stream_kernel");
    }
    if (D == 1024 && taps == 9 && warp_rows_ok(din, Y, y_fmt, y_plane, D) && din_sstride % 4 == 0 && !((uintptr_t)W & 15)) {
        nb::launch(dwconv_ln_silu_row_kernel, streams * c, 256, 0, (cudaStream_t)stream, din, din_sstride, pos, W, g, b, Y, y_fmt, y_plane, c, eps);
        return nb_check_launch("dwconv_ln_silu_row_kernel");
    }
    if (warp_rows_ok(din, Y, y_fmt, y_plane, D) && din_sstride % 4 == 0 && !((uintptr_t)W & 15)) {
        const int items = streams * c;
        nb::launch(dwconv_ln_silu_warp_kernel, (items + WROWS - 1) / WROWS, WROWS * 32, 0, (cudaStream_t)stream, din, din_sstride, pos, W, g, b, Y, y_fmt, y_plane,
                                                                                                       streams, c, D, taps, eps);
        return nb_check_launch("dwconv_ln_silu_warp_kernel");
    }
    nb::launch(dwconv_ln_silu_kernel, dim3(c, streams), LNT, 0, (cudaStream_t)stream, din, din_sstride, pos, W, g, b, Y, y_fmt, y_plane, c, D, taps, eps);
    return nb_check_launch("dwconv_ln_silu_kernel");
}

extern "C" int nemo_conv2d_c1_s2_relu(const float *X, int64_t x_sstride, const float *W, const float *bias, float *Y, int streams, int T, int F,
                                      int T1, int F1, int C, void *stream) {
    const int64_t total = (int64_t)streams * T1 * F1 * C;
    if (total <= 0) return 0;
    nb::launch(conv2d_c1_s2_relu_kernel, grid_for(total), 256, 0, (cudaStream_t)stream, X, x_sstride, W, bias, Y, T, F, T1, F1, C, total);
    return nb_check_launch("conv2d_c1_s2_relu_kernel");
}

extern "C" int nb_dwconv2d_s2_fmt(const float *X, const float *W, const float *bias, void *Y, int y_fmt, int64_t y_plane, int streams, int T, int F,
                                  int T1, int F1, int C, void *stream) {
    const int64_t total = (int64_t)streams * T1 * F1 * C;
    if (total <= 0) return 0;
    // by rows when there are enough rows to fill the GPU (batches); a single stream's few rows go
    // to the element-parallel kernel
    if ((int64_t)streams * T1 >= 148 && (int64_t)streams * T1 <= 0x7fffffff) {
        nb::launch(dwconv2d_s2_rows_kernel, (unsigned)(streams * T1), 256, 0, (cudaStream_t)stream, X, W, bias, Y, y_fmt, y_plane, T, F, T1, F1, C);
        return nb_check_launch("dwconv2d_s2_rows_kernel");
    }
    nb::launch(dwconv2d_s2_kernel, grid_for(total), 256, 0, (cudaStream_t)stream, X, W, bias, Y, y_fmt, y_plane, T, F, T1, F1, C, total);
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
    if (C % 32 == 0 && 2 * F1 + 1 <= FT_IN_W - 2) {
        const size_t smem = front_tile_smem(F1);
        const bool bf = y_fmt == NEMO_FMT_BF16X2;
        void (*k)(const float *, int64_t, const float *, const float *, const float *, const float *, void *, int64_t, int, int, int, int, int) =
            F == 128 ? (bf ? subsample_front_tile_kernel<128, true> : subsample_front_tile_kernel<128, false>)
                     : (bf ? subsample_front_tile_kernel<0, true> : subsample_front_tile_kernel<0, false>);
        if (nb_smem_attr((const void *)k, smem)) return nb_set_error("nemo_subsample_front: %s", nemo_gpu_last_error());
        const dim3 grid((unsigned)(streams * ((T2 + FT_TR - 1) / FT_TR)), (unsigned)(C / 32));
        nb::launch(k, grid, 256, smem, (cudaStream_t)stream, X, x_sstride, W0, b0, W2, b2, Y, y_plane, T, F, T1, T2, C);
        return nb_check_launch("subsample_front_tile_kernel");
    }
    nb::launch(subsample_front_kernel, (unsigned)((positions + 7) / 8), 256, 0, (cudaStream_t)stream, X, x_sstride, W0, b0, W2, b2, Y, y_fmt, y_plane, T, F, T1,
                                                                                              F1, T2, F2, C, positions);
    return nb_check_launch("subsample_front_kernel");
}

extern "C" int nb_flatten_rows_fmt(const float *X, void *Y, int y_fmt, int64_t y_plane, const int *lo, int streams, int T, int F, int C, int c, void *stream) {
    const int64_t total = (int64_t)streams * c * C * F;
    if (total <= 0) return 0;
    if ((size_t)F * C * sizeof(float) <= 48 * 1024 && (int64_t)streams * c >= 148 && (int64_t)streams * c <= 0x7fffffff) {
        nb::launch(flatten_rows_smem_kernel, (unsigned)(streams * c), 256, (size_t)F * C * sizeof(float), (cudaStream_t)stream, X, Y, y_fmt, y_plane, lo, T,
                   F, C, c);
        return nb_check_launch("flatten_rows_smem_kernel");
    }
    nb::launch(flatten_rows_kernel, grid_for(total), 256, 0, (cudaStream_t)stream, X, Y, y_fmt, y_plane, lo, T, F, C, c, total);
    return nb_check_launch("flatten_rows_kernel");
}

extern "C" int nemo_flatten_rows(const float *X, float *Y, const int *lo, int streams, int T, int F, int C, int c, void *stream) {
    return nb_flatten_rows_fmt(X, Y, NEMO_FMT_F32, 0, lo, streams, T, F, C, c, stream);
}
