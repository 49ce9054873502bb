// Sample-rate conversion on the GPU: the windowed-sinc resampler of src/resample.c:34-82
// (Blackman-windowed sinc with 16 zero crossings, cutoff at the lower Nyquist, weights
// normalised by their sum, input taken as zero outside [0, nin)) for many streams at once.
// The host keeps the streaming bookkeeping (each stream's input FIFO, how many outputs the input
// seen so far allows); this kernel does the sums. Output j of every stream sits at the same
// input position t = j * ratio, so a block computes the tap weights of its 32 outputs once, in
// shared memory, and applies them to up to 64 streams. Weights, sums and the final division run
// in double precision in the host's order (ascending input index), so an output differs from
// the host's only by the last bits of the double cos/sin.
#include "common.cuh"
#include "engine_dev.h"
#include "nb.h"

namespace {

constexpr int OPB = 32;        // outputs per block (one per lane)
constexpr int WARPS = 8;
constexpr int SPB = 64;        // streams per block
constexpr double ZERO_CROSSINGS = 16.0;
constexpr size_t SMEM_LIMIT = 160 * 1024;

struct Rate {
    double ratio, half, fc2;
};

Rate rate_of(int in_rate, int out_rate) {
    Rate r;
    r.ratio = (double)in_rate / (double)out_rate;
    r.half = ZERO_CROSSINGS * fmax(r.ratio, 1.0);
    r.fc2 = fmin(1.0, 1.0 / r.ratio);
    return r;
}

// taps an output can span: ceil(t - half) .. floor(t + half)
int max_taps(double half) { return (int)floor(2.0 * half) + 2; }
// odd row pitch (in doubles) so the lanes' rows start on different banks
int tap_pitch(double half) { return max_taps(half) | 1; }
size_t smem_bytes(double half) { return (size_t)OPB * tap_pitch(half) * sizeof(double) + OPB * (2 * sizeof(double) + sizeof(long long)); }

__device__ __forceinline__ double taper(double u, double half, double fc2) {
    const double x = u / half;
    if (x <= -1.0 || x >= 1.0) return 0.0;
    const double blackman = 0.42 + 0.5 * cos(M_PI * x) + 0.08 * cos(2.0 * M_PI * x);
    const double a = M_PI * fc2 * u;
    return fc2 * (fabs(a) < 1e-9 ? 1.0 : sin(a) / a) * blackman;
}

__global__ void __launch_bounds__(OPB * WARPS) resample_kernel(const float *__restrict__ in, int64_t in_ld, int64_t in_start, int64_t in_len,
                                                               int64_t nin, int64_t out0, int count, Rate r, int tp, float *out, int64_t out_ld,
                                                               int streams) {
    extern __shared__ double smem[];
    double *w = smem;                                   // [OPB][tp] tap weights
    double *wsum = w + (size_t)OPB * tp;                // [OPB]
    long long *first = (long long *)(wsum + OPB);       // [OPB] input index of tap 0
    int *ntap = (int *)(first + OPB);                   // [OPB]
    nb::pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int j0 = blockIdx.x * OPB;
    const int nout = min(OPB, count - j0);
    if (tid < nout) {
        const double t = (double)(out0 + j0 + tid) * r.ratio;
        const long long a = (long long)ceil(t - r.half), b = (long long)floor(t + r.half);
        first[tid] = a;
        ntap[tid] = (int)min(b - a + 1, (long long)tp);  // b - a <= 2 * half + 1 < tp; the clamp only guards the rows
    }
    __syncthreads();
    for (int idx = tid; idx < nout * tp; idx += OPB * WARPS) {
        const int o = idx / tp, k = idx - o * tp;
        const double t = (double)(out0 + j0 + o) * r.ratio;
        w[idx] = k < ntap[o] ? taper((double)(first[o] + k) - t, r.half, r.fc2) : 0.0;
    }
    __syncthreads();
    if (tid < nout) {
        double s = 0.0;
        for (int k = 0; k < ntap[tid]; ++k) s += w[tid * tp + k];
        wsum[tid] = s;
    }
    __syncthreads();
    if (lane >= nout) return;
    const double *wo = w + lane * tp;
    const long long a = first[lane];
    const int n = ntap[lane];
    // taps whose input index lies in [0, nin) and inside the staged window
    const long long lo = max(max(a, 0LL), (long long)in_start), hi = min(min(a + n, (long long)nin), (long long)(in_start + in_len));
    const double sum = wsum[lane];
    const int s_end = min(streams, (int)(blockIdx.y + 1) * SPB);
    for (int s = blockIdx.y * SPB + warp; s < s_end; s += WARPS) {
        const float *x = in + (int64_t)s * in_ld;
        double acc = 0.0;
        for (long long i = lo; i < hi; ++i) acc += wo[i - a] * (double)x[i - in_start];
        out[(int64_t)s * out_ld + j0 + lane] = (float)(sum > 0 ? acc / sum : 0.0);
    }
}

}  // namespace

extern "C" int nb_resample_smem_ok(int in_rate, int out_rate) {
    return in_rate > 0 && out_rate > 0 && smem_bytes(rate_of(in_rate, out_rate).half) <= SMEM_LIMIT;
}

extern "C" int nemo_resample(const float *in, int64_t in_ld, int64_t in_start, int64_t in_len, int64_t nin, int64_t out0, int count, int in_rate,
                             int out_rate, float *out, int64_t out_ld, int streams, void *stream) {
    if (count <= 0 || streams <= 0) return 0;
    if (in_rate <= 0 || out_rate <= 0) return nb_set_error("nemo_resample: rates %d -> %d", in_rate, out_rate);
    if (in_start < 0 || in_len < 0 || in_ld < in_len || out_ld < count || out0 < 0 || nin < in_start + in_len)
        return nb_set_error("nemo_resample: window [%lld, +%lld) (ld %lld) of %lld samples, %d outputs (ld %lld)", (long long)in_start,
                            (long long)in_len, (long long)in_ld, (long long)nin, count, (long long)out_ld);
    const Rate r = rate_of(in_rate, out_rate);
    const size_t smem = smem_bytes(r.half);
    if (smem > SMEM_LIMIT) return nb_set_error("nemo_resample: %d -> %d Hz needs %zu B of shared memory", in_rate, out_rate, smem);
    if (nb_smem_attr((const void *)resample_kernel, smem)) return nb_set_error("nemo_resample: %s", nemo_gpu_last_error());
    const dim3 grid((count + OPB - 1) / OPB, (streams + SPB - 1) / SPB);
    nb::launch(resample_kernel, grid, OPB * WARPS, smem, (cudaStream_t)stream, in, in_ld, in_start, in_len, nin, out0, count, r, tap_pitch(r.half),
               out, out_ld, streams);
    return nb_check_launch("resample_kernel");
}
