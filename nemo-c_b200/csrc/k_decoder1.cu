// Persistent single-stream greedy RNNT decoder: the whole greedy loop of one chunk
// (src/decoder.c:92-127) for ONE stream in one launch of one CTA per SM.
//
// Why: with one stream every greedy step is a chain of small dependent products (two LSTM
// layers, the prediction projection, the joint), ~11 launches per emitted token. Here each CTA
// keeps its slice of every decoder weight matrix in shared memory for the whole chunk (the
// gate rows i, f, g, o of its hidden units in both LSTM layers, its rows of the prediction
// projection and of the vocabulary projection, ~118 KB), so a step streams no weights at all:
//   L0    gates of this CTA's units = b + W0 [embed(last) | h0], then the cell    -> h0' slice
//   L1    same for layer 1 with [h0' | h1]                                       -> h1' slice
//   PRED  pred slice = bp + Wp h1'
//   JOINT logits of this CTA's vocabulary rows for every remaining frame of the chunk (the
//         prediction only changes on an emission, so the frames up to the first non-blank are
//         decided with one evaluation, as src/decoder.c:97-103 does with up to 16 frames),
//         reduced to a per-CTA (value, lowest index) per frame
// with a grid barrier after each. Every CTA then reduces the per-CTA maxima itself (ties to the
// lowest index, src/kernels.metal:521-550) and takes the same decision: the greedy state lives
// in every CTA, no barrier is needed for it. On an emission the provisional LSTM state becomes
// the committed one by swapping the roles of two buffers.
//
// Every wait is bounded; a CTA that gives up raises a global abort flag all waits watch.
#include "common.cuh"
#include "engine_dev.h"
#include "sm100.cuh"
#include "gridsync.cuh"

namespace {

constexpr int THREADS = 256;
constexpr int NWARPS = THREADS / 32;
constexpr int MAXU = 8;      // hidden units per CTA (4 gate rows each)
constexpr int MAXP = 8;      // prediction rows per CTA
constexpr int MAXV = 8;      // vocabulary rows per CTA
constexpr int MAXF = 16;     // frames per chunk
constexpr int MAXCTA = 256;  // CTAs of the grid at most (the decision reads 8 per lane)
constexpr long long WAIT_LIMIT = 2000000000LL;

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(sm100::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void slice(int n, int &lo, int &hi) {
    lo = (int)(((long long)blockIdx.x * n) / gridDim.x);
    hi = (int)(((long long)(blockIdx.x + 1) * n) / gridDim.x);
}

struct __align__(16) Shared {
    float x[2048];                 // input vector of the current product
    float gates[4 * MAXU];
    float pred[1024];              // full prediction vector (joint input)
    float pv[NWARPS][MAXF];        // per-warp best value per frame
    int pi[NWARPS][MAXF];          // per-warp best index per frame
    uint64_t wbar;
    int abort;
};

// Grid barrier over all CTAs (monotonic arrival counter, global abort word; gridsync.cuh).
__device__ bool grid_sync(const NbDec1Args &a, Shared &S, unsigned &epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
        ++epoch;
        if (!nb::grid_arrive_wait(a.bar, epoch * gridDim.x, a.err, 1, WAIT_LIMIT)) S.abort = 1;
    }
    __syncthreads();
    return !S.abort;
}

// dst[k] = src[k] for k < n <= 4 * THREADS (a vector another CTA wrote, read from L2): every load
// of the thread is issued before the first store, so the copy costs one L2 round trip.
__device__ __forceinline__ void copy_vec(float *dst, const float *src, int n) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int k = threadIdx.x + q * THREADS;
        v[q] = k < n ? __ldcg(src + k) : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int k = threadIdx.x + q * THREADS;
        if (k < n) dst[k] = v[q];
    }
}

// out[r] = sum_k W[r][k] x[k] for the nr rows of a bf16 [nr][K] block in shared memory (row r
// handled by warp r % 8, lanes over k in float4 steps); x in shared memory.
__device__ __forceinline__ void rows_dot(const uint16_t *W, int nr, int K, const float *x, float *out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < nr; r += NWARPS) {
        const uint2 *w = (const uint2 *)(W + (size_t)r * K);
        float acc = 0.0f;
        for (int k = lane; k < K / 4; k += 32) {
            const uint2 q = w[k];
            const float4 xx = *(const float4 *)(x + 4 * k);
            acc += xx.x * nb::bf16lo(q.x) + xx.y * nb::bf16hi(q.x) + xx.z * nb::bf16lo(q.y) + xx.w * nb::bf16hi(q.y);
        }
        acc = nb::warp_sum(acc);
        if (lane == 0) out[r] = acc;
    }
}

__global__ void __launch_bounds__(THREADS, 1) decoder1_kernel(const __grid_constant__ NbDec1Args a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Shared &S = *(Shared *)smem_raw;
    const int PH = a.PH, JH = a.JH, V = a.V, c = a.c;
    // shared layout sized by the largest slices of the grid (every CTA uses the same offsets)
    const int Um = (PH + gridDim.x - 1) / gridDim.x, Pm = (JH + gridDim.x - 1) / gridDim.x, Vm = (V + gridDim.x - 1) / gridDim.x;
    uint16_t *W0s = (uint16_t *)(smem_raw + sizeof(Shared));   // [4U][2PH] gate rows of layer 0
    uint16_t *W1s = W0s + (size_t)4 * Um * 2 * PH;             // layer 1
    uint16_t *Wps = W1s + (size_t)4 * Um * 2 * PH;             // [P][PH]
    uint16_t *Wos = Wps + (size_t)Pm * PH;                     // [Vr][JH]
    float *encs = (float *)(Wos + (size_t)Vm * JH);            // [c][JH] joint encoder rows of the chunk
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int u0, u1, p0, p1, v0, v1;
    slice(PH, u0, u1);
    slice(JH, p0, p1);
    slice(V, v0, v1);
    const int U = u1 - u0, P = p1 - p0, Vr = v1 - v0;

    // ---- this CTA's weight rows and the chunk's encoder rows, once per launch ----
    if (tid == 0) {
        sm100::mbar_init(&S.wbar, 1);
        S.abort = 0;
        sm100::fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t bytes = (uint32_t)(2 * 4 * U * 2 * PH * 2 + P * PH * 2 + Vr * JH * 2 + c * JH * 4);
        if (lane == 0) sm100::mbar_arrive_expect_tx(&S.wbar, bytes);
        __syncwarp();
        for (int j = lane; j < 4 * U; j += 32) {
            const int row = (j / U) * PH + u0 + j % U;  // gate j / U of unit u0 + j % U
            bulk_g2s(W0s + (size_t)j * 2 * PH, a.W0 + (size_t)row * 2 * PH, (uint32_t)(2 * PH * 2), &S.wbar);
            bulk_g2s(W1s + (size_t)j * 2 * PH, a.W1 + (size_t)row * 2 * PH, (uint32_t)(2 * PH * 2), &S.wbar);
        }
        for (int j = lane; j < P; j += 32) bulk_g2s(Wps + (size_t)j * PH, a.Wp + (size_t)(p0 + j) * PH, (uint32_t)(PH * 2), &S.wbar);
        for (int j = lane; j < Vr; j += 32) bulk_g2s(Wos + (size_t)j * JH, a.Wo + (size_t)(v0 + j) * JH, (uint32_t)(JH * 2), &S.wbar);
        for (int j = lane; j < c; j += 32) bulk_g2s(encs + (size_t)j * JH, a.enc + (size_t)j * JH, (uint32_t)(JH * 4), &S.wbar);
    }

    // ---- greedy state (identical in every CTA) ----
    const DecState &d = a.d;
    int t = 0, symbols = 0, last = d.last_token[0], pred_valid = d.pred_valid[0], ntok = 0;
    int cur = 0;  // committed half of H0 / H1; the other half holds the provisional state
    // cell states of this CTA's units (thread tid < U owns unit u0 + tid): committed and provisional
    float cc0 = 0.0f, cc1 = 0.0f, cp0 = 0.0f, cp1 = 0.0f;
    if (tid < U) {
        const int j = u0 + tid;
        a.H0[j] = d.h[j];
        a.H1[j] = d.h[PH + j];
        cc0 = d.c[j];
        cc1 = d.c[PH + j];
        if (pred_valid) {
            a.H0[PH + j] = d.hp[j];
            a.H1[PH + j] = d.hp[PH + j];
            cp0 = d.cp[j];
            cp1 = d.cp[PH + j];
        }
    }
    if (pred_valid)
        for (int j = p0 + tid; j < p1; j += THREADS) a.PRED[j] = d.pred[j];
    // the biases this thread adds, held in registers for the whole launch: gates i, f, g, o of unit
    // u0 + tid in both layers (tid < U), prediction row p0 + tid (tid < P), vocabulary row v0 + warp
    float b0r[4] = { 0.f, 0.f, 0.f, 0.f }, b1r[4] = { 0.f, 0.f, 0.f, 0.f }, bpr = 0.0f, bor = 0.0f;
    if (tid < U)
#pragma unroll
        for (int gt = 0; gt < 4; ++gt) { b0r[gt] = a.b0[gt * PH + u0 + tid]; b1r[gt] = a.b1[gt * PH + u0 + tid]; }
    if (tid < P) bpr = a.bp[p0 + tid];
    if (warp < Vr) bor = a.bo[v0 + warp];
    unsigned epoch = 0;
    bool ok = grid_sync(a, S, epoch);
    if (ok && tid == 0 && !sm100::mbar_wait(&S.wbar, 0, WAIT_LIMIT)) { S.abort = 1; atomicExch(&a.bar[1], 1u); atomicCAS(a.err, 0, 2); }
    __syncthreads();
    ok = ok && !S.abort;

    const int max_it = c * (a.max_symbols + 1) + 2;
    for (int it = 0; ok && t < c && it < max_it; ++it) {
        if (!pred_valid) {
            // ---- L0: x = [embed(last) | h0 committed] ----
            float *H0c = a.H0 + cur * PH, *H0p = a.H0 + (1 - cur) * PH;
            float *H1c = a.H1 + cur * PH, *H1p = a.H1 + (1 - cur) * PH;
            {
                // the embedding row (all loads in flight at once) and the committed h0
                uint16_t ev[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int k = tid + q * THREADS;
                    ev[q] = (k < PH && last != a.blank) ? a.embed[(size_t)last * PH + k] : (uint16_t)0;
                }
                copy_vec(S.x + PH, H0c, PH);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int k = tid + q * THREADS;
                    if (k < PH) S.x[k] = nb::bf2f(ev[q]);
                }
            }
            __syncthreads();
            rows_dot(W0s, 4 * U, 2 * PH, S.x, S.gates);
            __syncthreads();
            if (tid < U) {
                const int j = u0 + tid;
                const float ig = nb::sigmoid_f(S.gates[tid] + b0r[0]), fg = nb::sigmoid_f(S.gates[U + tid] + b0r[1]);
                const float gg = tanhf(S.gates[2 * U + tid] + b0r[2]), og = nb::sigmoid_f(S.gates[3 * U + tid] + b0r[3]);
                cp0 = fg * cc0 + ig * gg;
                H0p[j] = og * tanhf(cp0);
            }
            if (!(ok = grid_sync(a, S, epoch))) break;
            // ---- L1: x = [h0' | h1 committed] ----
            copy_vec(S.x, H0p, PH);
            copy_vec(S.x + PH, H1c, PH);
            __syncthreads();
            rows_dot(W1s, 4 * U, 2 * PH, S.x, S.gates);
            __syncthreads();
            if (tid < U) {
                const int j = u0 + tid;
                const float ig = nb::sigmoid_f(S.gates[tid] + b1r[0]), fg = nb::sigmoid_f(S.gates[U + tid] + b1r[1]);
                const float gg = tanhf(S.gates[2 * U + tid] + b1r[2]), og = nb::sigmoid_f(S.gates[3 * U + tid] + b1r[3]);
                cp1 = fg * cc1 + ig * gg;
                H1p[j] = og * tanhf(cp1);
            }
            if (!(ok = grid_sync(a, S, epoch))) break;
            // ---- PRED: pred = bp + Wp h1' ----
            copy_vec(S.x, H1p, PH);
            __syncthreads();
            rows_dot(Wps, P, PH, S.x, S.gates);
            __syncthreads();
            if (tid < P) a.PRED[p0 + tid] = S.gates[tid] + bpr;
            if (!(ok = grid_sync(a, S, epoch))) break;
            pred_valid = 1;
        }
        // ---- JOINT: this CTA's vocabulary rows for every remaining frame ----
        copy_vec(S.pred, a.PRED, JH);
        __syncthreads();
        const int nf = c - t;
        {
            float bv[MAXF];
            int bi[MAXF];
#pragma unroll
            for (int f = 0; f < MAXF; ++f) { bv[f] = -INFINITY; bi[f] = 0x7fffffff; }
            for (int r = warp; r < Vr; r += NWARPS) {  // rows ascend per warp: strict > keeps the lowest index
                const uint2 *w = (const uint2 *)(Wos + (size_t)r * JH);
#pragma unroll
                for (int f = 0; f < MAXF; ++f) {
                    if (f >= nf) break;
                    const float *e = encs + (size_t)(t + f) * JH;
                    float acc = 0.0f;
                    for (int k = lane; k < JH / 4; k += 32) {
                        const uint2 q = w[k];
                        const float4 ee = *(const float4 *)(e + 4 * k), pp = *(const float4 *)(S.pred + 4 * k);
                        acc += fmaxf(ee.x + pp.x, 0.0f) * nb::bf16lo(q.x) + fmaxf(ee.y + pp.y, 0.0f) * nb::bf16hi(q.x) +
                               fmaxf(ee.z + pp.z, 0.0f) * nb::bf16lo(q.y) + fmaxf(ee.w + pp.w, 0.0f) * nb::bf16hi(q.y);
                    }
                    acc = nb::warp_sum(acc) + (r == warp ? bor : a.bo[v0 + r]);
                    if (acc > bv[f]) { bv[f] = acc; bi[f] = v0 + r; }
                }
            }
            if (lane == 0)
#pragma unroll
                for (int f = 0; f < MAXF; ++f) { S.pv[warp][f] = bv[f]; S.pi[warp][f] = bi[f]; }
        }
        __syncthreads();
        if (tid < nf) {
            float best = -INFINITY;
            int bidx = 0x7fffffff;
            for (int w = 0; w < NWARPS; ++w) {
                const float v = S.pv[w][tid];
                const int i = S.pi[w][tid];
                if (v > best || (v == best && i < bidx)) { best = v; bidx = i; }
            }
            a.part_v[(size_t)tid * gridDim.x + blockIdx.x] = best;  // frame-major: one frame's maxima are contiguous
            a.part_i[(size_t)tid * gridDim.x + blockIdx.x] = bidx;
        }
        if (!(ok = grid_sync(a, S, epoch))) break;
        // ---- decision (every CTA): argmax per frame over the CTAs, first non-blank frame ----
        // warp w reduces frames w, w + 8: lane l reads the maxima of CTAs l, l + 32, ... (all its
        // loads in flight at once), then a warp-wide max, ties to the lowest index
        for (int fr = warp; fr < nf; fr += NWARPS) {
            float pv[MAXCTA / 32];
            int pix[MAXCTA / 32];
#pragma unroll
            for (int q = 0; q < MAXCTA / 32; ++q) {
                const int b = lane + 32 * q;
                pv[q] = -INFINITY;
                pix[q] = 0x7fffffff;
                if (b < (int)gridDim.x) {
                    pv[q] = __ldcg(a.part_v + (size_t)fr * gridDim.x + b);
                    pix[q] = __ldcg(a.part_i + (size_t)fr * gridDim.x + b);
                }
            }
            float best = -INFINITY;
            int bidx = 0x7fffffff;
#pragma unroll
            for (int q = 0; q < MAXCTA / 32; ++q)
                if (pv[q] > best || (pv[q] == best && pix[q] < bidx)) { best = pv[q]; bidx = pix[q]; }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
                if (ov > best || (ov == best && oi < bidx)) { best = ov; bidx = oi; }
            }
            if (lane == 0) S.pi[0][fr] = bidx;
        }
        __syncthreads();
        int f = 0;
        while (f < nf && S.pi[0][f] == a.blank) ++f;
        if (f == nf) {
            t = c;  // every remaining frame is blank
        } else {
            const int k = S.pi[0][f];
            if (f > 0) symbols = 0;  // blanks advanced the frame
            t += f;
            if (blockIdx.x == 0 && tid == 0) {
                if (ntok < d.tok_cap) d.tokens[ntok] = k;
            }
            ++ntok;
            last = k;
            cur = 1 - cur;  // provisional state becomes the committed one
            cc0 = cp0;
            cc1 = cp1;
            pred_valid = 0;
            if (++symbols >= a.max_symbols) { symbols = 0; ++t; }
        }
        __syncthreads();  // S.pi is rewritten by the next joint
    }
    // ---- write the greedy state back (committed and provisional LSTM state, prediction) ----
    if (ok) {
        if (tid < U) {
            const int j = u0 + tid;
            d.h[j] = a.H0[cur * PH + j];
            d.h[PH + j] = a.H1[cur * PH + j];
            d.c[j] = cc0;
            d.c[PH + j] = cc1;
            if (pred_valid) {
                d.hp[j] = a.H0[(1 - cur) * PH + j];
                d.hp[PH + j] = a.H1[(1 - cur) * PH + j];
                d.cp[j] = cp0;
                d.cp[PH + j] = cp1;
            }
        }
        if (pred_valid)
            for (int j = p0 + tid; j < p1; j += THREADS) d.pred[j] = a.PRED[j];
        if (blockIdx.x == 0 && tid == 0) {
            d.t[0] = t;
            d.symbols[0] = symbols;
            d.active[0] = t < c;
            d.last_token[0] = last;
            d.pred_valid[0] = pred_valid;
            d.ntok[0] = ntok;
            d.cnt[1] = t < c;  // streams still active (nonzero: the loop bound was hit)
        }
    }
    // the weight copies must have landed before the CTA exits (bounded)
    if (tid == 0) sm100::mbar_wait(&S.wbar, 0, WAIT_LIMIT);
    __syncthreads();
}

}  // namespace

extern "C" size_t nb_decoder1_smem(int PH, int JH, int V, int grid, int c) {
    const size_t Um = (PH + grid - 1) / grid, Pm = (JH + grid - 1) / grid, Vm = (V + grid - 1) / grid;
    return sizeof(Shared) + 2 * 4 * Um * 2 * PH * 2 + Pm * PH * 2 + Vm * JH * 2 + (size_t)c * JH * 4;
}

// Whether the persistent decoder fits this model on `grid` CTAs.
extern "C" int nb_decoder1_fits(int PH, int JH, int V, int grid, int cmax, size_t smem_optin) {
    const int U = (PH + grid - 1) / grid, P = (JH + grid - 1) / grid, Vr = (V + grid - 1) / grid;
    if (grid > MAXCTA || U > MAXU || P > MAXP || Vr > MAXV || cmax > MAXF || 2 * PH > 2048 || JH > 1024 || PH % 4 || JH % 4) return 0;
    return nb_decoder1_smem(PH, JH, V, grid, cmax) <= smem_optin;
}

extern "C" int nb_decoder1(const NbDec1Args *args, int grid, void *stream) {
    const NbDec1Args &a = *args;
    if (a.c < 0 || a.c > MAXF) return nb_set_error("persistent decoder: %d frames per chunk (0..%d)", a.c, MAXF);
    if (a.c == 0) return 0;
    if (grid > MAXCTA) return nb_set_error("persistent decoder: %d CTAs above %d", grid, MAXCTA);
    const size_t smem = nb_decoder1_smem(a.PH, a.JH, a.V, grid, a.c);
    if (nb_smem_attr((const void *)decoder1_kernel, nb_decoder1_smem(a.PH, a.JH, a.V, grid, MAXF)))
        return nb_set_error("persistent decoder: %s", nemo_gpu_last_error());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaMemsetAsync(a.bar, 0, 2 * sizeof(unsigned), (cudaStream_t)stream) != cudaSuccess)
        return nb_set_error("persistent decoder: %s", cudaGetErrorString(cudaGetLastError()));
    if (cudaLaunchKernelEx(&cfg, decoder1_kernel, a) != cudaSuccess) return nb_set_error("persistent decoder: %s", cudaGetErrorString(cudaGetLastError()));
    return nb_check_launch("decoder1_kernel");
}
