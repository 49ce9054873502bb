// Log-mel frames on the GPU: the transform of src/mel.c:115-173 (Hann(400) window centred in a
// 512-point frame, double-precision radix-2 FFT, power spectrum, 128 Slaney filters, log) for
// many frames of many streams at once. The host keeps the streaming bookkeeping (pre-emphasis,
// which frames are complete, reflection at the stream edges) and hands over, per stream, the
// sample span the new frames read; frame f of a stream covers span[f * 160 .. f * 160 + 512).
// One CTA per (frame, stream). The butterflies run in the same order and precision as the host
// transform; the filterbank sums skip the filters' zero taps (which add exactly +0).
#include "common.cuh"
#include "engine_dev.h"
#include "nb.h"

namespace {

constexpr int NFFT = NB_MEL_NFFT, NFREQ = NB_MEL_NFREQ, NMEL = NB_MEL_NMEL, HOP = NB_MEL_HOP;
constexpr int THREADS = NFFT / 2;  // one butterfly per thread and stage
constexpr float LOG_GUARD = 5.960464477539063e-08f;

__global__ void __launch_bounds__(THREADS) logmel_kernel(const float *__restrict__ span, int64_t span_stride, const float *__restrict__ window,
                                                         const float *__restrict__ fb, const int2 *__restrict__ fb_rng, const double *__restrict__ wr,
                                                         const double *__restrict__ wi, float *out, int64_t out_stride, int64_t out_row0) {
    __shared__ double re[NFFT], im[NFFT];
    __shared__ float pw[NFREQ];
    nb::pdl_wait();
    const int f = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
    const float *x = span + (int64_t)s * span_stride + (int64_t)f * HOP;
    // windowed samples, stored in bit-reversed order (the iterative FFT's input order)
    for (int k = tid; k < NFFT; k += THREADS) {
        const int r = (int)(__brev((unsigned)k) >> (32 - 9));
        re[r] = (double)(x[k] * window[k]);
        im[r] = 0.0;
    }
    __syncthreads();
    for (int width = 2; width <= NFFT; width <<= 1) {
        const int half = width >> 1, tstep = NFFT / width;
        const int k = tid % half, p = (tid / half) * width + k, q = p + half;
        const double c = wr[k * tstep], sn = wi[k * tstep];
        const double xr = re[q] * c - im[q] * sn, xi = re[q] * sn + im[q] * c;
        const double ar = re[p], ai = im[p];
        re[p] = ar + xr;
        im[p] = ai + xi;
        re[q] = ar - xr;
        im[q] = ai - xi;
        __syncthreads();
    }
    for (int k = tid; k < NFREQ; k += THREADS) pw[k] = (float)(re[k] * re[k] + im[k] * im[k]);
    __syncthreads();
    if (tid < NMEL) {
        const int2 rg = fb_rng[tid];
        const float *fr = fb + tid * NFREQ;
        float acc = 0.0f;
        for (int k = rg.x; k < rg.y; ++k) acc += fr[k] * pw[k];
        out[(int64_t)s * out_stride + (out_row0 + f) * NMEL + tid] = logf(acc + LOG_GUARD);
    }
}

struct Tables {
    float *window, *fb;
    int2 *rng;
    double *wr, *wi;
};
Tables g_tab[64];  // per device

int tables(Tables **t) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nb_set_error("log-mel: no usable device");
    Tables &T = g_tab[dev];
    if (!T.window) {
        nb_mel_t *m = nb_mel_create();
        const float *win, *fb;
        const double *wr, *wi;
        nb_mel_tables(m, &win, &fb, &wr, &wi);
        int2 rng[NMEL];
        for (int b = 0; b < NMEL; ++b) {
            int lo = NFREQ, hi = 0;
            for (int k = 0; k < NFREQ; ++k)
                if (fb[b * NFREQ + k] != 0.0f) { lo = lo < k ? lo : k; hi = k + 1; }
            rng[b] = make_int2(lo < hi ? lo : 0, lo < hi ? hi : 0);
        }
        Tables n = {};
        const bool ok = cudaMalloc(&n.window, NFFT * sizeof(float)) == cudaSuccess && cudaMalloc(&n.fb, NMEL * NFREQ * sizeof(float)) == cudaSuccess &&
                        cudaMalloc(&n.rng, NMEL * sizeof(int2)) == cudaSuccess && cudaMalloc(&n.wr, NFFT / 2 * sizeof(double)) == cudaSuccess &&
                        cudaMalloc(&n.wi, NFFT / 2 * sizeof(double)) == cudaSuccess &&
                        cudaMemcpy(n.window, win, NFFT * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess &&
                        cudaMemcpy(n.fb, fb, NMEL * NFREQ * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess &&
                        cudaMemcpy(n.rng, rng, NMEL * sizeof(int2), cudaMemcpyHostToDevice) == cudaSuccess &&
                        cudaMemcpy(n.wr, wr, NFFT / 2 * sizeof(double), cudaMemcpyHostToDevice) == cudaSuccess &&
                        cudaMemcpy(n.wi, wi, NFFT / 2 * sizeof(double), cudaMemcpyHostToDevice) == cudaSuccess;
        nb_mel_destroy(m);
        if (!ok) return nb_set_error("log-mel: cannot upload the transform tables");
        T = n;
    }
    *t = &T;
    return 0;
}

}  // namespace

// Frames of `streams` sample spans (device, span_stride floats apart) into rows out_row0 ..
// out_row0 + nframes - 1 of each stream's [rows][128] block (out_stride floats apart).
extern "C" int nb_logmel_frames(const float *span, int64_t span_stride, int streams, int nframes, float *out, int64_t out_stride, int64_t out_row0,
                                void *stream) {
    if (nframes <= 0 || streams <= 0) return 0;
    Tables *T;
    if (tables(&T)) return -1;
    nb::launch(logmel_kernel, dim3(nframes, streams), THREADS, 0, (cudaStream_t)stream, span, span_stride, T->window, T->fb, T->rng, T->wr, T->wi, out, out_stride,
                                                                               out_row0);
    return nb_check_launch("logmel_kernel");
}

extern "C" int nemo_logmel_frames(const float *span, int64_t span_stride, int streams, int nframes, float *out, int64_t out_stride, void *stream) {
    return nb_logmel_frames(span, span_stride, streams, nframes, out, out_stride, 0, stream);
}
