// Persistent single-stream encoder: every conformer block of one chunk (src/encoder.c:145-188)
// for ONE stream (c <= 16 rows) in one launch of one CTA per SM.
//
// Why: with a handful of rows the chunk is a chain of ~220 small dependent steps, each of which
// streams a few MB of bf16 weights (1.18 GB per chunk). Launched one by one, every step pays a
// launch, a pipeline fill and a split-K reduction. Here each CTA owns a fixed slice of output
// columns of every projection, so a projection needs no cross-CTA reduction, and a producer warp
// streams the CTA's weight rows of the NEXT projections into a ring of shared-memory slots
// (bulk copies) while the compute warps are still waiting on the grid barrier of the current
// one: the weight stream does not wait on the dependency chain.
//
// Stages of block l (grid barrier after each):
//   FF1a  ff = SiLU(LN_ff1(x) W1^T)            x = h (l = 0) or LN_out_{l-1}(h)
//   FF1b  h  = x + 0.5 ff W2^T
//   QKV   kv[pos + r] = LN_att(h) Wqkv^T        (cache rows, src/encoder.c:160)
//   ATT   att = rel-pos attention over the cache window, one CTA per (head, row)
//   WO    h += att Wo^T
//   PW1   din[pos + r] = GLU(LN_conv(h) Wpw1^T); then each CTA runs the causal depthwise conv of
//         its own channels (they depend on its own din columns only) into xdw
//   PW2   h += SiLU(LN_bn(xdw)) Wpw2^T
//   FF2a  ff = SiLU(LN_ff2(h) W1^T)
//   FF2b  h += 0.5 ff W2^T
// and after the last block xout = LN_out(h) as bf16 hi/lo planes for the prompt projection.
//
// Projections run on the tensor cores with mma.sync m16n8k16 (weights as the 16-row operand,
// activation rows as the 8-column operand, bf16 hi/lo activation planes as in the batched path),
// K split over the 8 compute warps and reduced through shared memory. Every wait is bounded:
// on a timeout the CTA records an error, raises a global abort flag that every other wait also
// watches, lets its producer drain its copies in flight, and returns.
#include <cuda_bf16.h>
#include "common.cuh"
#include "engine_dev.h"
#include "sm100.cuh"
#include "gridsync.cuh"

namespace {

constexpr int CWARPS = 8;
constexpr int CTHREADS = CWARPS * 32;
constexpr int THREADS = CTHREADS;
constexpr int MAXC = 16;
constexpr int KC = 512;                 // activation k-chunk staged in shared memory
constexpr int ACT_PITCH = KC * 2 + 16;  // bytes per staged activation row (+16: ldmatrix bank spread)
constexpr int ACT_PLANE = MAXC * ACT_PITCH;
constexpr int NSLOT = 3;
constexpr int MAXL = 72;              // attention window rows (56 history + 16 new)
constexpr int NSTAGE = 8;               // projections per block
constexpr long long WAIT_LIMIT = 2000000000LL;  // clock cycles (~1 s)

struct Smem {
    // weight slots live at the front of dynamic shared memory; this struct follows them
    __align__(16) uint8_t act[2 * ACT_PLANE];        // bf16 hi / lo activation planes of one k-chunk
    float red[CWARPS][2][2][128];                     // per-warp partial accumulators
    float outv[32][MAXC];                             // reduced outputs [weight row][activation row]
    float st[MAXC][4];                                // row statistics: mean1, inv1, mean2, inv2
    float rs[CWARPS][16];                             // per-warp partial row sums
    float hs[MAXC][32];                               // this CTA's columns of the residual stream
    float glu[32][MAXC];                              // conv-module GLU outputs of this CTA's channels
    float sc[MAXL];                                   // attention scores / probabilities
    float vpart[2][128];                              // attention value halves
    uint64_t full[NSLOT], vbar;
    int abort;
};
// attention keeps the value rows of its window in the activation tile + reduction area
static_assert(offsetof(Smem, red) + sizeof(float) * CWARPS * 2 * 2 * 128 >= MAXL * 512, "value rows do not fit");

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(sm100::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float sigm(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

__device__ __forceinline__ void cbar() { sm100::named_barrier(1, CTHREADS); }

// Weight operand of projection s of block l.
__device__ __forceinline__ void stage_w(const NbEnc1Args &a, int l, int s, const uint16_t *&W, int &N, int &K, bool &glu) {
    const NbEnc1Layer &w = a.L[l];
    const int D = a.D, FF = a.FF;
    glu = false;
    switch (s) {
    case 0: W = w.ff1_w1; N = FF; K = D; break;
    case 1: W = w.ff1_w2; N = D; K = FF; break;
    case 2: W = w.wqkv; N = 3 * D; K = D; break;
    case 3: W = w.wo; N = D; K = D; break;
    case 4: W = w.pw1; N = 2 * D; K = D; glu = true; break;
    case 5: W = w.pw2; N = D; K = D; break;
    case 6: W = w.ff2_w1; N = FF; K = D; break;
    default: W = w.ff2_w2; N = D; K = FF; break;
    }
}

// This CTA's output columns [lo, hi) of an N-output projection.
__device__ __forceinline__ void slice(int nout, int &lo, int &hi) {
    lo = (int)(((long long)blockIdx.x * nout) / gridDim.x);
    hi = (int)(((long long)(blockIdx.x + 1) * nout) / gridDim.x);
}

// Grid-wide barrier of the compute threads (arrival counter plus a global abort word every
// waiter watches; gridsync.cuh). Returns false when the launch is being abandoned.
__device__ bool grid_sync(const NbEnc1Args &a, Smem &S, unsigned &epoch) {
    cbar();
    if (threadIdx.x == 0) {
        ++epoch;
        if (!nb::grid_arrive_wait(a.bar, epoch * gridDim.x, a.err, 1, WAIT_LIMIT)) S.abort = 1;
    }
    cbar();
    return !S.abort;
}

// Row statistics of the c rows of X ([c][D] fp32) for LayerNorm (src/kernels.metal:258-288:
// mean, then the mean of squared deviations): st[r] = {mean, inv}. With (g2, b2) the rows are
// normalised with (g1, b1) first and the statistics of that result go to st[r][2..3].
__device__ void row_stats(Smem &S, const float *X, int c, int D, float eps, const float *g1, const float *b1, bool twice) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < c; r += CWARPS) {
        float v[32];
        const int per = D / 32;  // values per lane (D <= 1024)
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = j < per ? X[(int64_t)r * D + j * 32 + lane] : 0.0f;
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) s += v[j];
        const float mean = nb::warp_sum(s) / (float)D;
        float q = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) if (j < per) { const float d = v[j] - mean; q += d * d; }
        const float inv = 1.0f / sqrtf(nb::warp_sum(q) / (float)D + eps);
        float m2 = 0.0f, inv2 = 0.0f;
        if (twice) {
            float s2 = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) if (j < per) { const int k = j * 32 + lane; v[j] = (v[j] - mean) * inv * g1[k] + b1[k]; s2 += v[j]; }
            m2 = nb::warp_sum(s2) / (float)D;
            float q2 = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) if (j < per) { const float d = v[j] - m2; q2 += d * d; }
            inv2 = 1.0f / sqrtf(nb::warp_sum(q2) / (float)D + eps);
        }
        if (lane == 0) { S.st[r][0] = mean; S.st[r][1] = inv; S.st[r][2] = m2; S.st[r][3] = inv2; }
    }
}

enum { P_PLAIN = 0, P_LN = 1, P_LN2 = 2, P_DWLN = 3 };

// One k-chunk of the activation rows in registers: element e = threadIdx.x + u * CTHREADS is
// row e / (kc / 4), columns 4 (e % (kc / 4)) .. +3. A chunk holds at most 8 x CTHREADS float4
// (c <= 8 rows of 1024 columns or c <= 16 rows of 512), so all its loads go out at once.
struct ActRegs { float4 x[8]; };

__device__ __forceinline__ void act_load(ActRegs &R, const float *X, int ldx, int c, int k0, int kc) {
    const int sh = __ffs(kc / 4) - 1, total = c << sh;  // kc / 4 is a power of two
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int e = threadIdx.x + u * CTHREADS;
        if (e < total) {
            const int r = e >> sh, k = (e - (r << sh)) * 4;
            R.x[u] = *(const float4 *)(X + (int64_t)r * ldx + k0 + k);
        }
    }
}

// Normalise (mode) and store the chunk as bf16 hi/lo planes, rows apitch bytes apart.
// pre: when non-null, the normalisation vectors of this thread's columns (g1, b1, g2, b2), loaded
// together with the chunk (fused layout: thread t holds columns 4t .. 4t+3 of every row).
__device__ __forceinline__ void act_store(const ActRegs &R, Smem &S, int mode, int c, int k0, int kc, int apitch, const float *g1, const float *b1,
                                          const float *g2, const float *b2, const float4 (&pre)[4], bool use_pre) {
    const int sh = __ffs(kc / 4) - 1, total = c << sh;
    const int plane = ACT_PLANE;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int e = threadIdx.x + u * CTHREADS;
        if (e < total) {
            const int r = e >> sh, k = (e - (r << sh)) * 4;
            float v[4] = { R.x[u].x, R.x[u].y, R.x[u].z, R.x[u].w };
            if (mode != P_PLAIN) {
                const float m1 = S.st[r][0], i1 = S.st[r][1];
                const float4 ga = use_pre ? pre[0] : __ldg((const float4 *)(g1 + k0 + k)), ba = use_pre ? pre[1] : __ldg((const float4 *)(b1 + k0 + k));
                const float gg[4] = { ga.x, ga.y, ga.z, ga.w }, bb[4] = { ba.x, ba.y, ba.z, ba.w };
                float g2v[4] = { 0.f, 0.f, 0.f, 0.f }, b2v[4] = { 0.f, 0.f, 0.f, 0.f };
                if (mode == P_LN2) {
                    const float4 gc = use_pre ? pre[2] : __ldg((const float4 *)(g2 + k0 + k)), bc = use_pre ? pre[3] : __ldg((const float4 *)(b2 + k0 + k));
                    g2v[0] = gc.x; g2v[1] = gc.y; g2v[2] = gc.z; g2v[3] = gc.w;
                    b2v[0] = bc.x; b2v[1] = bc.y; b2v[2] = bc.z; b2v[3] = bc.w;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float y = (v[j] - m1) * i1 * gg[j] + bb[j];
                    if (mode == P_LN2) y = (y - S.st[r][2]) * S.st[r][3] * g2v[j] + b2v[j];
                    else if (mode == P_DWLN) y = y * sigm(y);
                    v[j] = y;
                }
            }
            const __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
            const __nv_bfloat162 l0 = __floats2bfloat162_rn(v[0] - __low2float(h0), v[1] - __high2float(h0));
            const __nv_bfloat162 l1 = __floats2bfloat162_rn(v[2] - __low2float(h1), v[3] - __high2float(h1));
            uint8_t *hp = S.act + r * apitch + k * 2, *lp = hp + plane;
            *(uint2 *)hp = make_uint2(*(const uint32_t *)&h0, *(const uint32_t *)&h1);
            *(uint2 *)lp = make_uint2(*(const uint32_t *)&l0, *(const uint32_t *)&l1);
        }
    }
}

// Sums over the CTA of two values per row u < 8 (every compute thread gets the totals).
__device__ __forceinline__ void rows_sum8x2(float (&v)[8], float (&w2)[8], Smem &S) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const float t = nb::warp_sum(v[u]), t2 = nb::warp_sum(w2[u]);
        if (lane == 0) { S.rs[warp][u] = t; S.rs[warp][8 + u] = t2; }
    }
    cbar();
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        float t = 0.0f, t2 = 0.0f;
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) { t += S.rs[w][u]; t2 += S.rs[w][8 + u]; }
        v[u] = t;
        w2[u] = t2;
    }
    cbar();
}

// LayerNorm statistics straight from a chunk that holds whole rows (kc == K == 4 * CTHREADS:
// thread t has columns 4t .. 4t+3 of every row u in x[u]), from the sums of x and x^2 in one
// reduction: mean = S1 / D, variance = S2 / D - mean^2 (the Metal kernel subtracts the mean
// first; the two agree to fp32 rounding for normalised activations).
__device__ __forceinline__ void stats_regs(const ActRegs &R, Smem &S, int c, int D, float eps, bool twice, const float4 ga, const float4 ba) {
    float s1[8], s2[8], mean[8], inv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const float4 x = R.x[u];
        s1[u] = u < c ? x.x + x.y + x.z + x.w : 0.0f;
        s2[u] = u < c ? x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w : 0.0f;
    }
    rows_sum8x2(s1, s2, S);
    const float invD = 1.0f / (float)D;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        mean[u] = s1[u] * invD;
        inv[u] = rsqrtf(fmaxf(s2[u] * invD - mean[u] * mean[u], 0.0f) + eps);
    }
    float m2[8], inv2[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) m2[u] = inv2[u] = 0.0f;
    if (twice) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float y0 = (R.x[u].x - mean[u]) * inv[u] * ga.x + ba.x, y1 = (R.x[u].y - mean[u]) * inv[u] * ga.y + ba.y;
            const float y2 = (R.x[u].z - mean[u]) * inv[u] * ga.z + ba.z, y3 = (R.x[u].w - mean[u]) * inv[u] * ga.w + ba.w;
            s1[u] = u < c ? y0 + y1 + y2 + y3 : 0.0f;
            s2[u] = u < c ? y0 * y0 + y1 * y1 + y2 * y2 + y3 * y3 : 0.0f;
        }
        rows_sum8x2(s1, s2, S);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            m2[u] = s1[u] * invD;
            inv2[u] = rsqrtf(fmaxf(s2[u] * invD - m2[u] * m2[u], 0.0f) + eps);
        }
    }
    if (threadIdx.x < c) {
        const int u = threadIdx.x;
        S.st[u][0] = mean[u]; S.st[u][1] = inv[u]; S.st[u][2] = m2[u]; S.st[u][3] = inv2[u];
    }
}

// The staging group of a warp: act_store gives thread t the columns 4 (t % (kc / 4)) .. +3 of
// its rows, so the 32 threads of a warp stage 128 consecutive columns, shared with the other
// warps of its group (kc / 4 threads per row span: groups of 256 / (kc / 4) warps... 1, 2 or 4).
// The group stages those columns for all rows and multiplies them, so it only syncs with itself.
__device__ __forceinline__ void group_sync(int kc) {
    const int gw = CTHREADS / (kc / 4);          // warps sharing a column range
    if (gw <= 1) { __syncwarp(); return; }
    const int span = (kc / 4) / 32;              // column ranges (groups)
    const int grp = (threadIdx.x >> 5) % span;
    sm100::named_barrier(2 + grp, gw * 32);
}

// One k-step (16 columns at kk of the staged chunk): ah / al[g][nt] += W rows of granule g times
// the hi / lo activation rows of tile nt.
__device__ __forceinline__ void mma_kstep(uint32_t act, uint32_t wb, int pitch, int nrows, int k0, int kk, int ng, int nnt, int apitch,
                                          float (&ah)[2][2][4], float (&al)[2][2][4]) {
    const int lane = threadIdx.x & 31, mi = lane >> 3, rr = lane & 7;
    uint32_t b[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
        if (nt < nnt) ldsm_x4(act + (mi >> 1) * ACT_PLANE + (nt * 8 + rr) * apitch + (kk + (mi & 1) * 8) * 2, b[nt][0], b[nt][1], b[nt][2], b[nt][3]);
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        if (g >= ng) break;
        const int row = min(g * 16 + (mi & 1) * 8 + rr, nrows - 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(wb + row * pitch + (k0 + kk + (mi >> 1) * 8) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
            if (nt < nnt) {
                mma16816(ah[g][nt], a0, a1, a2, a3, b[nt][0], b[nt][1]);  // hi plane
                mma16816(al[g][nt], a0, a1, a2, a3, b[nt][2], b[nt][3]);  // lo plane
            }
    }
}

// This warp's k-steps of the staged chunk: the 8 k-steps of its group's 128 columns, split
// between the group's warps; consecutive k-steps alternate between two accumulator sets so the
// MMA dependency chains are half as long.
__device__ __forceinline__ void mma_chunk(const Smem &S, const uint8_t *slot, int pitch, int nrows, int k0, int kc, int ng, int nnt, int apitch,
                                          float (&acc_h)[2][2][4], float (&acc_l)[2][2][4], float (&acc_h2)[2][2][4], float (&acc_l2)[2][2][4]) {
    const int warp = threadIdx.x >> 5;
    const int span = (kc / 4) / 32, gw = CWARPS / span;  // column ranges, warps per range
    const int grp = warp % span, member = warp / span;
    const int per = 8 / gw;                             // k-steps of this warp: 8, 4 or 2
    const uint32_t act = sm100::smem_u32(S.act), wb = sm100::smem_u32(slot);
    for (int q = 0; q < per; q += 2) {
        const int kk = (grp * 8 + member * per + q) * 16;
        mma_kstep(act, wb, pitch, nrows, k0, kk, ng, nnt, apitch, acc_h, acc_l);
        mma_kstep(act, wb, pitch, nrows, k0, kk + 16, ng, nnt, apitch, acc_h2, acc_l2);
    }
}

// Warp 0 requests this CTA's weight rows of projection i (block i / 8, projection i % 8) into
// ring slot i % NSLOT: one bulk copy per row, completion counted on full[slot]. Called once the
// CTA's last reads of the slot (projection i - NSLOT) are behind a CTA barrier.
__device__ __forceinline__ void issue_weights(const NbEnc1Args &a, Smem &S, uint8_t *slots, int i, int total) {
    if ((threadIdx.x >> 5) != 0 || i >= total) return;
    const int lane = threadIdx.x & 31, slot = i % NSLOT;
    const uint16_t *W;
    int N, K;
    bool glu;
    stage_w(a, i / NSTAGE, i % NSTAGE, W, N, K, glu);
    int lo, hi;
    slice(glu ? N / 2 : N, lo, hi);
    const int R = hi - lo, nrows = glu ? 2 * R : R, pitch = K * 2 + 16;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier reads of the slot before the copy's writes
    if (lane == 0) sm100::mbar_arrive_expect_tx(&S.full[slot], (uint32_t)(nrows * K * 2));
    __syncwarp();
    uint8_t *dst = slots + (size_t)slot * a.slot_bytes;
    for (int j = lane; j < nrows; j += 32) {
        const int wrow = j < R ? lo + j : N / 2 + lo + (j - R);
        bulk_g2s(dst + (size_t)j * pitch, W + (int64_t)wrow * K, (uint32_t)(K * 2), &S.full[slot]);
    }
}

// Relative-position attention of one (head, query row) (src/kernels.metal:293-348). Right after
// the barrier the item requests everything it needs at once: the value rows go to shared memory
// by bulk copy (they are needed last), the query, key and position rows to registers.
__device__ __forceinline__ bool attention_item(const NbEnc1Args &a, Smem &S, const NbEnc1Layer &w, int hd, int r, int pos, int cache_len,
                                               unsigned &vphase) {
    const int D = a.D, c = a.c, L = cache_len + c, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ld = 3 * (int64_t)D;
    const int off = hd * 128;
    const float *Kb = w.kv + (int64_t)(pos - cache_len) * ld + D + off;
    const float *Vb = Kb + D;
    const float *Pb = w.ptab + (int64_t)(a.Lmax - L + c - 1 - r) * D + off;
    float *Vs = (float *)S.act;  // [L][128]: the activation tile and reduction area are idle here
    if (warp == 0) {
        if (lane == 0) sm100::mbar_arrive_expect_tx(&S.vbar, (uint32_t)(L * 512));
        __syncwarp();
        for (int j = lane; j < L; j += 32) bulk_g2s(Vs + j * 128, Vb + (int64_t)j * ld, 512u, &S.vbar);
    }
    // query (lane's 4 dims) and this warp's keys j = warp + 8 i (i < 9 covers L <= 72)
    const float4 q4 = *(const float4 *)(w.kv + (int64_t)(pos + r) * ld + off + 4 * lane);
    const float4 u4 = __ldg((const float4 *)(w.bias_u + off + 4 * lane)), v4 = __ldg((const float4 *)(w.bias_v + off + 4 * lane));
    const float4 qu = make_float4(q4.x + u4.x, q4.y + u4.y, q4.z + u4.z, q4.w + u4.w);
    const float4 qv = make_float4(q4.x + v4.x, q4.y + v4.y, q4.z + v4.z, q4.w + v4.w);
#pragma unroll
    for (int i0 = 0; i0 < 9; i0 += 5) {  // keys in two batches of loads (register budget)
        float4 k4[5], p4[5];
#pragma unroll
        for (int i = 0; i < 5; ++i) {
            const int j = warp + CWARPS * (i0 + i);
            if (i0 + i < 9 && j < L) {
                k4[i] = *(const float4 *)(Kb + (int64_t)j * ld + 4 * lane);
                p4[i] = __ldg((const float4 *)(Pb + (int64_t)j * D + 4 * lane));
            }
        }
#pragma unroll
        for (int i = 0; i < 5; ++i) {
            const int j = warp + CWARPS * (i0 + i);
            if (i0 + i < 9 && j < L) {
                float sc = qu.x * k4[i].x + qu.y * k4[i].y + qu.z * k4[i].z + qu.w * k4[i].w;
                float tp = qv.x * p4[i].x + qv.y * p4[i].y + qv.z * p4[i].z + qv.w * p4[i].w;
                sc = nb::warp_sum(sc);
                tp = nb::warp_sum(tp);
                if (lane == 0) S.sc[j] = (sc + tp) * a.scale;
            }
        }
    }
    cbar();
    if (warp == 0) {
        float sv[3], mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < 3; ++t) { const int j = lane + 32 * t; sv[t] = j < L ? S.sc[j] : -INFINITY; mx = fmaxf(mx, sv[t]); }
        mx = nb::warp_max(mx);
        float sum = 0.0f;
#pragma unroll
        for (int t = 0; t < 3; ++t) { const int j = lane + 32 * t; sv[t] = j < L ? expf(sv[t] - mx) : 0.0f; sum += sv[t]; }
        sum = nb::warp_sum(sum);
#pragma unroll
        for (int t = 0; t < 3; ++t) { const int j = lane + 32 * t; if (j < L) S.sc[j] = sv[t] / sum; }
    }
    // the value rows
    if (tid == 0 && !sm100::mbar_wait(&S.vbar, vphase & 1, WAIT_LIMIT)) {
        S.abort = 1;
        atomicExch(&a.bar[1], 1u);
        atomicCAS(a.err, 0, 4);
    }
    ++vphase;
    cbar();
    if (S.abort) return false;
    const int d = tid & 127, half = tid >> 7;
    float acc = 0.0f;
    for (int j = half; j < L; j += 2) acc += S.sc[j] * Vs[j * 128 + d];
    S.vpart[half][d] = acc;
    cbar();
    if (tid < 128) a.att[(int64_t)r * D + off + tid] = S.vpart[0][tid] + S.vpart[1][tid];
    cbar();  // the value rows are read before the area is reused
    return true;
}

__global__ void __launch_bounds__(THREADS, 1) encoder1_kernel(const __grid_constant__ NbEnc1Args a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *slots = smem_raw;
    Smem &S = *(Smem *)(smem_raw + NSLOT * a.slot_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = a.D, c = a.c;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; ++s) sm100::mbar_init(&S.full[s], 1);
        sm100::mbar_init(&S.vbar, 1);
        S.abort = 0;
        sm100::fence_mbar_init();
    }
    // activation rows past c stay zero for the whole launch (the MMAs read 8 or 16 rows)
    for (int i = threadIdx.x; i < 2 * ACT_PLANE / 16; i += THREADS) ((uint4 *)S.act)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    const int total = a.layers * NSTAGE;

    {
        // ---- compute warps ----
        unsigned epoch = 0, vphase = 0;
        const int pos = *a.pos, cache_len = *a.cache_len;
        for (int i = 0; i < NSLOT; ++i) issue_weights(a, S, slots, i, total);
        int issued = min(NSLOT, total);  // projections whose weight copies were requested
        const int nnt = (c + 7) / 8;
        int dlo, dhi;
        slice(D, dlo, dhi);  // this CTA's columns of every D-wide output: its slice of h
        const int dR = dhi - dlo;
        // the CTA's columns of the residual stream live in shared memory between stages
        for (int e = threadIdx.x; e < dR * c; e += CTHREADS) S.hs[e / dR][e % dR] = a.h[(int64_t)(e / dR) * D + dlo + e % dR];
        int gi = 0;  // projection index (ring position)
        for (int l = 0; l < a.layers && !S.abort; ++l) {
            const NbEnc1Layer &w = a.L[l];
            const NbEnc1Layer *prev = l > 0 ? &a.L[l - 1] : nullptr;
            for (int s = 0; s < NSTAGE; ++s, ++gi) {
                if (s == 3) {
                    // attention over the cache window (the QKV stage's barrier made the rows visible)
                    const int items = a.H * c;
                    for (int it = blockIdx.x; it < items; it += gridDim.x)
                        if (!attention_item(a, S, w, it % a.H, it / a.H, pos, cache_len, vphase)) break;
                    if (!grid_sync(a, S, epoch)) break;
                }
                const uint16_t *W;
                int N, K;
                bool glu;
                stage_w(a, l, s, W, N, K, glu);
                int lo, hi;
                slice(glu ? N / 2 : N, lo, hi);
                const int R = hi - lo, nrows = glu ? 2 * R : R, pitch = K * 2 + 16, ng = (nrows + 15) / 16;
                // activation source and normalisation of this projection
                int mode = P_PLAIN, ldx = D;
                const float *X = a.h, *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
                switch (s) {
                case 0:
                    if (prev) { mode = P_LN2; g1 = prev->ln_out_g; b1 = prev->ln_out_b; g2 = w.ln_ff1_g; b2 = w.ln_ff1_b; }
                    else { mode = P_LN; g1 = w.ln_ff1_g; b1 = w.ln_ff1_b; }
                    break;
                case 1: case 7: X = a.ff; ldx = a.FF; break;
                case 2: mode = P_LN; g1 = w.ln_att_g; b1 = w.ln_att_b; break;
                case 3: X = a.att; break;
                case 4: mode = P_LN; g1 = w.ln_conv_g; b1 = w.ln_conv_b; break;
                case 5: mode = P_DWLN; X = a.att; g1 = w.bn_g; b1 = w.bn_b; break;  // att holds the depthwise-conv output
                default: mode = P_LN; g1 = w.ln_ff2_g; b1 = w.ln_ff2_b; break;
                }
                // activation chunks: c <= 8 rows of up to 1024 columns, or 16 rows of 512
                const int kcmax = nnt == 1 ? 2 * KC : KC, apitch = kcmax * 2 + 16;
                const int kc = K < kcmax ? K : kcmax;
                const bool fused = mode != P_PLAIN && kc == K && K == 4 * CTHREADS;
                // one burst of loads: the first chunk, this thread's normalisation vectors, and what
                // the epilogue needs (output-LN vectors of its column; depthwise taps and history)
                ActRegs AR;
                act_load(AR, X, ldx, c, 0, kc);
                float4 pre[4];
                pre[0] = pre[1] = pre[2] = pre[3] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (fused) {
                    const int k = 4 * threadIdx.x;
                    pre[0] = __ldg((const float4 *)(g1 + k));
                    pre[1] = __ldg((const float4 *)(b1 + k));
                    if (mode == P_LN2) { pre[2] = __ldg((const float4 *)(g2 + k)); pre[3] = __ldg((const float4 *)(b2 + k)); }
                }
                const int e0 = threadIdx.x;             // epilogue item of this thread (R * c <= CTHREADS)
                const int en = R > 0 ? e0 % R : 0, er = R > 0 ? e0 / R : 0;
                const bool eact = R > 0 && e0 < R * c;
                float og = 1.0f, ob = 0.0f, dw[9], hist[8];
                if (eact && s == 1 && prev) { og = __ldg(prev->ln_out_g + lo + en); ob = __ldg(prev->ln_out_b + lo + en); }
                if (eact && s == 4) {
                    const int ch = lo + en;
#pragma unroll
                    for (int t = 0; t < 9; ++t) dw[t] = t < a.taps ? __ldg(w.dw_w + ch * a.taps + t) : 0.0f;
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const int row = pos - (a.taps - 1) + er + t;  // history rows precede pos
                        hist[t] = (t < a.taps - 1 && row < pos) ? w.din[(int64_t)row * D + ch] : 0.0f;
                    }
                }
                if (mode != P_PLAIN) {
                    if (fused) stats_regs(AR, S, c, D, a.eps, mode == P_LN2, pre[0], pre[1]);
                    else row_stats(S, X, c, D, a.eps, g1, b1, mode == P_LN2);
                }
                // wait for this projection's weight rows (one thread; the others at the barrier)
                const int slot = gi % NSLOT;
                if (threadIdx.x == 0 && !sm100::mbar_wait(&S.full[slot], (gi / NSLOT) & 1, WAIT_LIMIT)) {
                    S.abort = 1;
                    atomicExch(&a.bar[1], 1u);
                    atomicCAS(a.err, 0, 3);
                }
                cbar();
                if (S.abort) break;
                const uint8_t *ws = slots + (size_t)slot * a.slot_bytes;
                float acc[2][2][4], acl[2][2][4], acc2[2][2][4], acl2[2][2][4];
#pragma unroll
                for (int g = 0; g < 2; ++g)
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[g][nt][q] = acl[g][nt][q] = acc2[g][nt][q] = acl2[g][nt][q] = 0.0f;
                for (int k0 = 0; k0 < K; k0 += kc) {
                    act_store(AR, S, mode, c, k0, kc, apitch, g1, b1, g2, b2, pre, fused);
                    group_sync(kc);
                    if (k0 + kc < K) act_load(AR, X, ldx, c, k0 + kc, kc);  // next chunk in flight during the MMAs
                    if (nrows > 0) mma_chunk(S, ws, pitch, nrows, k0, kc, ng, nnt, apitch, acc, acl, acc2, acl2);
                    group_sync(kc);
                }
#pragma unroll
                for (int g = 0; g < 2; ++g)
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[g][nt][q] += acl[g][nt][q] + (acc2[g][nt][q] + acl2[g][nt][q]);
                // reduce the warps' partial sums: outv[weight row][activation row]
#pragma unroll
                for (int g = 0; g < 2; ++g)
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int q = 0; q < 4; ++q) S.red[warp][g][nt][lane * 4 + q] = acc[g][nt][q];
                cbar();
                // every warp is done with the slot: request the projection NSLOT ahead into it
                issue_weights(a, S, slots, gi + NSLOT, total);
                issued = min(gi + NSLOT + 1, total);
                for (int e = threadIdx.x; e < 2 * 2 * 128; e += CTHREADS) {
                    const int g = e >> 8, nt = (e >> 7) & 1, v = e & 127, ln = v >> 2, q = v & 3;
                    float sum = 0.0f;
#pragma unroll
                    for (int ww = 0; ww < CWARPS; ++ww) sum += S.red[ww][g][nt][v];
                    const int n = g * 16 + (ln >> 2) + (q >= 2 ? 8 : 0), r = nt * 8 + (ln & 3) * 2 + (q & 1);
                    S.outv[n][r] = sum;
                }
                cbar();
                // epilogue: output (column lo + e % R, row e / R); the stages that use prefetched
                // per-item values (1 and 4) have R * c <= CTHREADS, so there e == e0
                for (int e = threadIdx.x; R > 0 && e < R * c; e += CTHREADS) {
                    const int n = e % R, r = e / R, col = lo + n;
                    const float v = S.outv[n][r];
                    switch (s) {
                    case 0: case 6: a.ff[(int64_t)r * a.FF + col] = v * sigm(v); break;
                    case 1: {
                        float base = S.hs[r][n];
                        if (prev) base = (base - S.st[r][0]) * S.st[r][1] * og + ob;
                        const float hv = base + 0.5f * v;
                        S.hs[r][n] = hv;
                        a.h[(int64_t)r * D + col] = hv;
                        break;
                    }
                    case 2: w.kv[(int64_t)(pos + r) * 3 * D + col] = v; break;
                    case 3: case 5: { const float hv = S.hs[r][n] + v; S.hs[r][n] = hv; a.h[(int64_t)r * D + col] = hv; break; }
                    case 4: {
                        const float gv = v * sigm(S.outv[R + n][r]);
                        w.din[(int64_t)(pos + r) * D + col] = gv;
                        S.glu[n][r] = gv;
                        break;
                    }
                    default: { const float hv = S.hs[r][n] + 0.5f * v; S.hs[r][n] = hv; a.h[(int64_t)r * D + col] = hv; break; }
                    }
                }
                if (s == 4) {
                    // causal depthwise conv of this CTA's channels (src/kernels.metal:361-380) over
                    // rows pos - (taps - 1) .. pos + c - 1: history from registers, new rows from glu
                    cbar();
                    if (eact) {
                        float x = 0.0f;
#pragma unroll
                        for (int t = 0; t < 9; ++t) {
                            if (t >= a.taps) break;
                            const int rr = er - (a.taps - 1) + t;  // row relative to pos
                            x += dw[t] * (rr < 0 ? hist[t] : S.glu[en][rr]);
                        }
                        a.att[(int64_t)er * D + lo + en] = x;
                    }
                }
                if (!grid_sync(a, S, epoch)) break;
            }
        }
        // output LayerNorm of the last block, as bf16 hi/lo planes for the prompt projection
        if (!S.abort) {
            const NbEnc1Layer &w = a.L[a.layers - 1];
            row_stats(S, a.h, c, D, a.eps, nullptr, nullptr, false);
            cbar();
            for (int e = threadIdx.x; e < dR * c; e += CTHREADS) {
                const int n = e % dR, r = e / dR, col = dlo + n;
                const float y = (S.hs[r][n] - S.st[r][0]) * S.st[r][1] * w.ln_out_g[col] + w.ln_out_b[col];
                const uint16_t hb = nb::f2bf(y);
                a.xout[(int64_t)r * D + col] = hb;
                a.xout[(int64_t)r * D + col + a.xout_plane] = nb::f2bf(y - nb::bf2f(hb));
            }
        }
        // copies requested but not consumed (the launch was abandoned): wait for them (bounded)
        if (threadIdx.x == 0)
            for (int j = gi; j < issued; ++j) sm100::mbar_wait(&S.full[j % NSLOT], (j / NSLOT) & 1, WAIT_LIMIT);
    }
    __syncthreads();
}

}  // namespace

extern "C" size_t nb_encoder1_smem(int slot_bytes) { return (size_t)NSLOT * slot_bytes + sizeof(Smem); }

// Largest weight slice (rows x padded row bytes) any CTA loads for a model of width D / FF on a
// grid of `grid` CTAs.
extern "C" int nb_encoder1_slot_bytes(int D, int FF, int grid) {
    const int outs[NSTAGE] = { FF, D, 3 * D, D, D, D, FF, D }, Ks[NSTAGE] = { D, FF, D, D, D, D, D, FF }, rows_per[NSTAGE] = { 1, 1, 1, 1, 2, 1, 1, 1 };
    int best = 0;
    for (int s = 0; s < NSTAGE; ++s) {
        const int R = (outs[s] + grid - 1) / grid;
        const int b = R * rows_per[s] * (Ks[s] * 2 + 16);
        if (b > best) best = b;
    }
    return (best + 127) & ~127;
}

extern "C" int nb_encoder1(const NbEnc1Args *args, int grid, void *stream) {
    const NbEnc1Args &a = *args;
    if (a.c < 1 || a.c > MAXC) return nb_set_error("persistent encoder: %d rows per chunk (1..%d)", a.c, MAXC);
    if (a.D % 128 || a.D > 1024 || a.FF % 16 || (a.D < KC ? KC % a.D : a.D % KC) || (a.FF < KC ? KC % a.FF : a.FF % KC))
        return nb_set_error("persistent encoder: unsupported widths D=%d FF=%d", a.D, a.FF);
    if (a.H * 128 != a.D) return nb_set_error("persistent encoder: heads of 128 expected");
    if (a.Lmax > MAXL) return nb_set_error("persistent encoder: attention window %d above %d rows", a.Lmax, MAXL);
    if (a.taps < 1 || a.taps > 9) return nb_set_error("persistent encoder: depthwise kernel of %d taps (1..9)", a.taps);
    const size_t smem = nb_encoder1_smem(a.slot_bytes);
    if (nb_smem_attr((const void *)encoder1_kernel, smem)) return nb_set_error("persistent encoder: %s", nemo_gpu_last_error());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (the grid barriers need it)
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaMemsetAsync(a.bar, 0, 2 * sizeof(unsigned), (cudaStream_t)stream) != cudaSuccess)
        return nb_set_error("persistent encoder: %s", cudaGetErrorString(cudaGetLastError()));
    if (cudaLaunchKernelEx(&cfg, encoder1_kernel, a) != cudaSuccess) return nb_set_error("persistent encoder: %s", cudaGetErrorString(cudaGetLastError()));
    return nb_check_launch("encoder1_kernel");
}
