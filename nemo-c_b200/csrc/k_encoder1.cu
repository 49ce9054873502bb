// Persistent single-stream encoder: every conformer block of one chunk (src/encoder.c:145-188)
// for ONE stream (c <= 16 rows) in one launch of one CTA per SM.
//
// Why: with a handful of rows the chunk is a chain of ~220 small dependent steps, each of which
// streams a few MB of bf16 weights (1.18 GB per chunk). Launched one by one, every step pays a
// launch, a pipeline fill and a split-K reduction. Here the weight stream runs ahead of the
// dependency chain: one warp of each CTA requests the CTA's weight rows of the coming projections
// into a ring of shared memory as far ahead as the ring holds, one bulk copy per projection out
// of a copy of the weights laid out per CTA at set-up (the weight image), so each stage
// of the chain costs one grid barrier, one gather of its input rows from L2 and a few hundred
// cycles of math.
//
// Stages of block l (a grid barrier after each); x = h (l = 0) or LN_out_{l-1}(h):
//   FF1a  ff = SiLU(LN_ff1(x) W1^T)                  CTA b: a slice of the FF hidden columns
//   FF1b  h' = x + 0.5 ff W2^T                       CTA (kr, g): output columns of group g over
//                                                    the kr-th 1024-wide range of the hidden;
//                                                    the ranges' partial sums meet in h' through
//                                                    red.add (h' zeroed one stage ahead)
//   QKV   kv[pos + r] = LN_att(h') Wqkv^T            (cache rows, src/encoder.c:160)
//   ATT   att = rel-pos attention over the cache window, one CTA per (head, row)
//   WO    h' += att Wo^T
//   PW1   din[pos + r] = GLU(LN_conv(h') Wpw1^T); each CTA then runs the causal depthwise conv
//         of its own channels (they need its own din columns only) into y
//   PW2   h' += SiLU(LN_bn(y)) Wpw2^T
//   FF2a  ff = SiLU(LN_ff2(h') W1^T)
//   FF2b  h = h' + 0.5 ff W2^T                       (as FF1b, back into the block's input buffer)
// and after the last block xout = LN_out(h) as bf16 hi/lo planes for the prompt projection.
//
// Every stage's input is at most 1024 columns wide: each thread gathers four columns of every
// row with one 16-byte L2 load per row, reduces the LayerNorm statistics in registers,
// normalises, and stores bf16 hi/lo planes in shared memory. Projections run on the tensor cores
// with mma.sync m16n8k16 (weights as the 16-row operand, activation rows as the 8-column
// operand, hi and lo planes as two products), K split over the 8 compute warps and reduced
// through shared memory. Every wait is bounded: on a timeout the CTA records an error, raises a
// global abort flag that every other wait also watches, waits (bounded) for its copies in flight,
// and returns.
#include <cuda_bf16.h>
#include "common.cuh"
#include "engine_dev.h"
#include "sm100.cuh"
#include "gridsync.cuh"

namespace {

constexpr int CWARPS = 8;
constexpr int CTHREADS = CWARPS * 32;
constexpr int THREADS = CTHREADS;
constexpr int ISSUE_WARP = CWARPS - 1;
constexpr int MWARPS = CWARPS - 1;       // warps that run a stage's MMAs (all but the issue warp)
constexpr int MAXC = 16;
constexpr int KRW = 1024;                // widest k-range of one stage
constexpr int APITCH = KRW * 2 + 16;     // bytes per staged activation row (+16: ldmatrix bank spread)
constexpr int NB = 8;                    // projections in flight in the weight ring at most
constexpr int MAXL = 72;                 // attention window rows (56 history + 16 new)
constexpr int MAXR = 32;                 // weight rows of one CTA in one projection
constexpr int NSTAGE = 8;                // projections per block
constexpr int NTAIL = 3;                 // projections of the encoder's tail (prompt and joint encoder)
constexpr int NALL = NSTAGE + NTAIL;     // projection types
constexpr long long WAIT_LIMIT = 2000000000LL;  // clock cycles (~1 s)

struct Smem {
    float red[CWARPS][2][2][128];  // per-warp partial accumulators
    float outv[MAXR][MAXC];        // reduced outputs [weight row][activation row]
    float st[MAXC][8];             // per row: LN_out mean, inv of the block input (FF1a, read by FF1b);
                                   // the stage's folded statistics mu1, inv1, mu2, inv2
    float rs[2][CWARPS][2 * MAXC]; // per-warp row sums (two buffers)
    float fs[CWARPS][128];         // per-warp row sums of a folded LayerNorm
    float glu[16][MAXC];           // conv-module GLU outputs of this CTA's channels
    float cdw[16][9];              // depthwise taps of this CTA's channels (flat: channel * taps + tap)
    float chist[8][16];            // conv history rows [h][channel]
    float sc[MAXL];                // attention scores / probabilities
    float vpart[2][128];           // attention value halves
    uint64_t full[NB];
    int ring_off[NB];              // byte offset of projection i's rows in the ring (slot i % NB)
    int g_lo[NALL], g_hi[NALL], g_kr[NALL], g_krw[NALL], g_rows[NALL], g_pitch[NALL], g_bytes[NALL];
    long long g_img[NALL];         // byte offset of this CTA's block of projection s in block 0 of the image
                                   // (for the tail: in the tail, which follows the blocks)
    long long g_layer;             // image bytes of one block
    int consumed;                  // projections taken by the compute warps (set when they stop)
    int issued;                    // projections requested so far
    int abort;
};
// Bytes of the activation area for chunks of up to c rows and attention windows of up to Lw rows:
// the bf16 hi and lo planes of the NR-row tile (NR rows each, the lo plane NR * APITCH bytes
// after the hi plane), or the attention stage's value rows, whichever is larger.
// (The 8-row form serves chunks of up to 8 rows with attention windows of up to 64 rows.)
__host__ __device__ inline int act_rows(int c, int Lw) { return c <= 8 && Lw <= 64 ? 8 : 16; }
__host__ __device__ inline int act_bytes(int c, int Lw) {
    const int tile = 2 * act_rows(c, Lw) * APITCH, vals = Lw * 512;
    return ((tile > vals ? tile : vals) + 127) / 128 * 128;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(sm100::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar))
                 : "memory");
}
// The same for weight rows, which are read once per chunk: marked first to leave L2, so the 1.2 GB
// weight stream does not push out the activations and the small per-layer tensors.
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
                     sm100::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar)), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Bring [p, p + bytes) into L2 (bytes and p multiples of 16).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    // register operands only (not volatile): the compiler may schedule it among the fragment loads
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void red_add(float *p, float v) { asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory"); }

__device__ __forceinline__ float sigm(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

__device__ __forceinline__ void cbar() { sm100::named_barrier(1, CTHREADS); }

// Where CTA `cta` works in projection s of block l: its weight rows [lo, hi) (plus the gate rows
// N/2 + [lo, hi) for GLU) over columns [kr * krw, (kr + 1) * krw) of K. A projection whose K is
// wider than KRW is split two ways: KT / KRW k-ranges x (grid / ranges) column groups.
struct Geo {
    const uint16_t *W;
    int N, K, ldw, krw, kr, lo, hi;  // ldw: elements between weight rows
    bool glu;
};

__device__ __forceinline__ void slice(int n, int parts, int part, int &lo, int &hi) {
    lo = (int)(((long long)part * n) / parts);
    hi = (int)(((long long)(part + 1) * n) / parts);
}

__device__ __forceinline__ Geo stage_geo(const NbEnc1Args &a, int l, int s, int cta, int grid) {
    const NbEnc1Layer &w = a.L[l];
    const int D = a.D, FF = a.FF;
    Geo g;
    g.glu = false;
    switch (s) {
    case 0: g.W = w.ff1_w1; g.N = FF; g.K = D; break;
    case 1: g.W = w.ff1_w2; g.N = D; g.K = FF; break;
    case 2: g.W = w.wqkv; g.N = 3 * D; g.K = D; break;
    case 3: g.W = w.wo; g.N = D; g.K = D; break;
    case 4: g.W = w.pw1; g.N = 2 * D; g.K = D; g.glu = true; break;
    case 5: g.W = w.pw2; g.N = D; g.K = D; break;
    case 6: g.W = w.ff2_w1; g.N = FF; g.K = D; break;
    case 7: g.W = w.ff2_w2; g.N = D; g.K = FF; break;
    // the tail (one each per launch): prompt projections and joint encoder projection
    case 8: g.W = a.pw0; g.N = a.PRH; g.K = D; break;
    case 9: g.W = a.pw2; g.N = D; g.K = a.PRH; break;
    default: g.W = a.jw; g.N = a.JH; g.K = D; break;
    }
    g.ldw = s == 8 ? a.pw0_ld : g.K;
    const int nout = g.glu ? g.N / 2 : g.N;
    if (g.K <= KRW) {
        g.krw = g.K;
        g.kr = 0;
        slice(nout, grid, cta, g.lo, g.hi);
    } else {
        g.krw = KRW;
        const int ranges = g.K / KRW, groups = grid / ranges;
        if (cta >= ranges * groups) {
            g.kr = 0;
            g.lo = g.hi = 0;
        } else {
            g.kr = cta / groups;
            slice(nout, groups, cta % groups, g.lo, g.hi);
        }
    }
    return g;
}

__device__ __forceinline__ int geo_rows(const Geo &g) { return (g.glu ? 2 : 1) * (g.hi - g.lo); }
__device__ __forceinline__ int geo_pitch(const Geo &g) { return g.krw * 2 + 16; }

// ---- weight image ------------------------------------------------------------------------------
// The weights re-laid out once, at set-up, in the order and padded row pitch the CTAs read them:
// block (l, s, b) holds CTA b's rows of projection s of block l (value rows then, for GLU, gate
// rows; the k-range of its column group for a split projection), each row krw bf16 followed by 16
// zero bytes, so one bulk copy brings a projection into the ring. Blocks follow (l, s, b) order;
// within a projection CTA b's block starts after the rows of the CTAs before it.
__host__ __device__ inline void stage_shape(int s, int D, int FF, int &nout, int &K, int &mult) {
    const int outs[NSTAGE] = { FF, D, 3 * D, D, D, D, FF, D }, Ks[NSTAGE] = { D, FF, D, D, D, D, D, FF }, m[NSTAGE] = { 1, 1, 1, 1, 2, 1, 1, 1 };
    nout = outs[s];
    K = Ks[s];
    mult = m[s];
}
// Image bytes per weight row of projection s: the padded row, plus for a projection that follows a
// folded LayerNorm (FF1a, QKV, PW1, FF2a: s even, below NSTAGE) its float4 of fold constants, stored
// after all rows of the CTA's block (one bulk copy brings both).
__host__ __device__ inline int stage_row_bytes(int s, int krw) { return krw * 2 + 16 + ((s & 1) || s >= NSTAGE ? 0 : 16); }
__host__ __device__ inline long long stage_image_bytes(int s, int D, int FF) {
    int nout, K, mult;
    stage_shape(s, D, FF, nout, K, mult);
    const int krw = K <= KRW ? K : KRW;
    return (long long)stage_row_bytes(s, krw) * mult * nout * (K / krw);
}
__host__ __device__ inline long long layer_image_bytes(int D, int FF) {
    long long b = 0;
    for (int s = 0; s < NSTAGE; ++s) b += stage_image_bytes(s, D, FF);
    return b;
}
// The tail follows the blocks: projection NSTAGE + t, t < NTAIL, all CTAs' rows in turn.
__host__ __device__ inline void tail_shape(int t, int D, int PRH, int JH, int &nout, int &K) {
    nout = t == 0 ? PRH : t == 1 ? D : JH;
    K = t == 1 ? PRH : D;
}
__host__ __device__ inline long long tail_stage_bytes(int t, int D, int PRH, int JH) {
    int nout, K;
    tail_shape(t, D, PRH, JH, nout, K);
    const int krw = K <= KRW ? K : KRW;
    return (long long)stage_row_bytes(NSTAGE + t, krw) * nout * (K / krw);
}
__host__ __device__ inline long long tail_image_bytes(int D, int PRH, int JH) {
    long long b = 0;
    for (int t = 0; t < NTAIL; ++t) b += tail_stage_bytes(t, D, PRH, JH);
    return b;
}
__device__ __forceinline__ long long image_offset(const NbEnc1Args &a, int l, int s, const Geo &g, int cta, int grid) {
    long long off = 0;
    if (s >= NSTAGE) {
        off = (long long)a.layers * layer_image_bytes(a.D, a.FF);
        for (int t = 0; t < s - NSTAGE; ++t) off += tail_stage_bytes(t, a.D, a.PRH, a.JH);
    } else {
        off = (long long)l * layer_image_bytes(a.D, a.FF);
        for (int t = 0; t < s; ++t) off += stage_image_bytes(t, a.D, a.FF);
    }
    const int nout = g.glu ? g.N / 2 : g.N, mult = g.glu ? 2 : 1;
    long long rows_before = (long long)mult * g.lo;
    if (g.K > KRW) rows_before += (long long)g.kr * nout;
    (void)cta; (void)grid;
    return off + rows_before * stage_row_bytes(s, g.krw);
}

__host__ __device__ inline int fold_rows(int D, int FF);
__host__ __device__ inline int fold_off(int s, int D, int FF);

// Set-up: one CTA per (CTA of the persistent grid, projection, block) copies that CTA's rows (and
// for s even their fold constants, from a.fold, computed before).
__global__ void encoder1_repack_kernel(const __grid_constant__ NbEnc1Args a, uint8_t *image, int s_base) {
    const int cta = blockIdx.x, s = s_base + blockIdx.y, l = blockIdx.z;
    const Geo g = stage_geo(a, l, s, cta, gridDim.x);
    const int rows = geo_rows(g), pitch = geo_pitch(g), R = g.hi - g.lo, vec = g.krw / 8;  // 16-byte pieces per row
    uint8_t *dst = image + image_offset(a, l, s, g, cta, gridDim.x);
    for (int e = threadIdx.x; e < rows * (vec + 1); e += blockDim.x) {
        const int j = e / (vec + 1), v = e % (vec + 1);
        uint4 x = make_uint4(0u, 0u, 0u, 0u);
        if (v < vec) {
            const int wrow = j < R ? g.lo + j : g.N / 2 + g.lo + (j - R);
            x = *(const uint4 *)(g.W + (int64_t)wrow * g.ldw + (int64_t)g.kr * g.krw + v * 8);
        }
        *(uint4 *)(dst + (size_t)j * pitch + v * 16) = x;
    }
    if (!(s & 1) && s < NSTAGE)
        for (int j = threadIdx.x; j < rows; j += blockDim.x) {
            const int wrow = j < R ? g.lo + j : g.N / 2 + g.lo + (j - R);
            ((float4 *)(dst + (size_t)rows * pitch))[j] = ((const float4 *)a.fold)[(int64_t)l * fold_rows(a.D, a.FF) + fold_off(s, a.D, a.FF) + wrow];
        }
}

// ---- weight ring: the CTA's weight rows of every projection, in order ---------------------------
// Warp ISSUE_WARP requests projections `issued`, `issued` + 1, ... (below `limit`) while they fit: at
// most NB in flight, and their bytes not overlapping any entry the compute warps have not released
// yet (released = `consumed`; entries are released in order). The warp keeps the ring table in
// registers (lane j: the entry in slot j; lane s < NSTAGE: projection type s's bytes and image
// offset), so a request costs a vote and one bulk copy, and the compute warps find each entry's
// offset in S.ring_off. Called at the start, before a stage's weights are waited for (if they were
// not requested yet), and during every stage's math, which touches only shared memory: issued at a
// grid barrier instead, the requests (one ~57 KB copy per CTA at once) delay the barrier's own few
// latency-critical accesses.
struct Ring {
    int o, z, j;     // lane's slot: byte offset, bytes, projection (-1: none)
    int bytes;       // lane s < NALL: bytes of projection type s
    long long img;   // and its offset in block 0 of the image (the tail's: in the tail)
    int issued, head;
};
__device__ __forceinline__ void ring_init(const NbEnc1Args &a, const Smem &S, Ring &q) {
    const int lane = threadIdx.x & 31;
    q.o = q.z = 0;
    q.j = -1;
    q.bytes = lane < (a.tail ? NALL : NSTAGE) ? S.g_bytes[lane] : 0;
    q.img = lane < (a.tail ? NALL : NSTAGE) ? S.g_img[lane] : 0;
    q.issued = q.head = 0;
}
__device__ void issue_ahead(const NbEnc1Args &a, Smem &S, uint8_t *ring, Ring &q, int consumed, uint64_t pol, int limit) {
    if ((threadIdx.x >> 5) != ISSUE_WARP) return;
    const int lane = threadIdx.x & 31, RB = a.ring_bytes;
    const long long layer_bytes = S.g_layer;
    const int blocks = a.layers * NSTAGE;  // projections of the blocks; the tail's follow
    limit = min(limit, blocks + (a.tail ? NTAIL : 0));
    while (q.issued < limit && q.issued - consumed < NB) {
        const int i = q.issued, st = i < blocks ? i % NSTAGE : NSTAGE + (i - blocks), slot = i % NB;
        const int sz = __shfl_sync(0xffffffffu, q.bytes, st);
        const long long img = __shfl_sync(0xffffffffu, q.img, st);
        const int off = q.head + sz > RB ? 0 : q.head;
        const bool live = lane < NB && q.j >= consumed && q.j < i;
        if (__any_sync(0xffffffffu, live && q.z > 0 && sz > 0 && q.o < off + sz && off < q.o + q.z)) break;
        if (lane == slot) { q.o = off; q.z = sz; q.j = i; }
        if (lane == 0) {
            S.ring_off[slot] = off;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the bytes' earlier generic reads before the copies
            sm100::mbar_arrive_expect_tx(&S.full[slot], (uint32_t)sz);
            const long long src = (i < blocks ? (long long)(i / NSTAGE) : (long long)a.layers) * layer_bytes + img;
            if (sz > 0) bulk_g2s_stream(ring + off, a.image + src, (uint32_t)sz, &S.full[slot], pol);
        }
        q.head = off + sz;
        q.issued = i + 1;
    }
    if (lane == 0) S.issued = q.issued;
}

// ---- compute warps -----------------------------------------------------------------------------

// warp_fold (common.cuh): lane l ends with the warp totals of values l * V / 32 + j (V >= 32) or of
// value l >> 1 (V = 16); stored at position lane * max(V / 32, 1) + j, value v sits at fs_pos(v).
using nb::warp_fold;

// Sums over the compute threads of two values per row (every thread gets the totals), NR rows
// (8 or 16). One butterfly per warp reduces all 2 NR values at once: at the step with lane offset
// o each lane keeps the half of its values selected by (lane & o) and adds its partner's copy of
// that half; once one value is left the remaining steps add it plainly. Lane l then holds the
// warp's total of value l >> SH (SH = 1 for 16 values, 0 for 32); the eight warps' totals meet in
// shared memory (two buffers, alternating, so back-to-back calls need one barrier each).
template <int NR>
__device__ __forceinline__ void rows_sum2(float (&v)[NR], float (&w)[NR], Smem &S, int &buf) {
    static_assert(NR == 8 || NR == 16, "8 or 16 rows");
    constexpr int V = 2 * NR, SH = NR == 16 ? 0 : 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float x[V];
#pragma unroll
    for (int u = 0; u < NR; ++u) { x[2 * u] = v[u]; x[2 * u + 1] = w[u]; }
    warp_fold<V>(x);
    S.rs[buf][warp][lane] = x[0];
    cbar();
    float t = 0.0f;
#pragma unroll
    for (int ww = 0; ww < CWARPS; ++ww) t += S.rs[buf][ww][lane];
    buf ^= 1;
#pragma unroll
    for (int u = 0; u < NR; ++u) {
        v[u] = __shfl_sync(0xffffffffu, t, (2 * u) << SH);
        w[u] = __shfl_sync(0xffffffffu, t, (2 * u + 1) << SH);
    }
}

// e / R and e % R for 0 <= e < 2048 and 1 <= R <= 32 without a division: q = e m >> 16 with
// m = ceil(2^16 / R). e m / 2^16 exceeds e / R by less than e / 2^16 < 1 / R, which never carries
// it past the next integer.
struct Div { int R, m; };
__device__ __forceinline__ Div make_div(int R) { R = max(R, 1); return { R, (65536 + R - 1) / R }; }
__device__ __forceinline__ int div_q(const Div &d, int e) { return (e * d.m) >> 16; }

enum { P_PLAIN = 0, P_LN = 1, P_LN2 = 2, P_DWLN = 3, P_LNX = 4 };  // P_LNX: LayerNorm applied in the gather, no SiLU

// The stage's input rows in registers: thread t holds columns 4t .. 4t+3 of every row (t < K/4).
template <int NR> struct Act { float4 x[NR]; };

// Predicated 16-byte L2 load into a register that keeps its value when the predicate is false (so
// the loads of all rows are in flight together, with nothing waiting on any of them).
__device__ __forceinline__ void ld_cg_pred(float4 &v, const float *p, bool pred) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
        "@q ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];\n\t}"
        : "+f"(v.x), "+f"(v.y), "+f"(v.z), "+f"(v.w)
        : "l"(p), "r"((int)pred));
}

template <int NR>
__device__ __forceinline__ void gather(Act<NR> &A, const float *X, int ldx, int k0, int K, int c) {
    const int t = threadIdx.x;
    const bool own = 4 * t < K;
#pragma unroll
    for (int u = 0; u < NR; ++u) {
        A.x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        ld_cg_pred(A.x[u], X + (int64_t)u * ldx + k0 + 4 * t, own && u < c);
    }
}

// LayerNorm statistics of each row (mean, inv = 1/sqrt(var + eps)) over K columns, from the sums of
// x and x^2 in one reduction (the Metal kernel subtracts the mean first; the two agree to fp32
// rounding for these activations).
template <int NR>
__device__ __forceinline__ void row_stats(const Act<NR> &A, Smem &S, int &buf, int K, float eps, float (&mean)[NR], float (&inv)[NR]) {
    float s1[NR], s2[NR];
#pragma unroll
    for (int u = 0; u < NR; ++u) {
        const float4 x = A.x[u];
        s1[u] = x.x + x.y + x.z + x.w;
        s2[u] = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
    rows_sum2<NR>(s1, s2, S, buf);
    const float invK = 1.0f / (float)K;
#pragma unroll
    for (int u = 0; u < NR; ++u) {
        mean[u] = s1[u] * invK;
        inv[u] = rsqrtf(fmaxf(s2[u] * invK - mean[u] * mean[u], 0.0f) + eps);
    }
}

// Store the (normalised) rows as bf16 hi / lo planes of the activation tile.
template <int NR>
__device__ __forceinline__ void stage_store(const Act<NR> &A, uint8_t *act, int c, int K) {
    const int t = threadIdx.x;
    if (4 * t >= K) return;
#pragma unroll
    for (int u = 0; u < NR; ++u) {
        if (u < c) {
            // hi = bf16(x) (two per cvt, the first operand to the upper half), lo = bf16(x - hi)
            const float4 v = A.x[u];
            uint32_t h0, h1, l0, l1;
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h0) : "f"(v.y), "f"(v.x));
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h1) : "f"(v.w), "f"(v.z));
            const float r0 = v.x - __uint_as_float(h0 << 16), r1 = v.y - __uint_as_float(h0 & 0xffff0000u);
            const float r2 = v.z - __uint_as_float(h1 << 16), r3 = v.w - __uint_as_float(h1 & 0xffff0000u);
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(l0) : "f"(r1), "f"(r0));
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(l1) : "f"(r3), "f"(r2));
            uint8_t *hp = act + u * APITCH + t * 8;
            *(uint2 *)hp = make_uint2(h0, h1);
            *(uint2 *)(hp + NR * APITCH) = make_uint2(l0, l1);
        }
    }
}

__device__ __forceinline__ float4 ld4g(const float *p) { return __ldg((const float4 *)p); }

// The fragments of one k-step (16 columns at kk): activation tiles (hi and lo planes) and the weight
// rows of each granule.
struct Frag { uint32_t b[2][4], a[2][4]; };

// (activation planes of NR rows: the lo plane NR * APITCH bytes after the hi plane)
template <int NR>
__device__ __forceinline__ void frag_load(Frag &f, uint32_t act, uint32_t wb, int pitch, int nrows, int kk, int ng, int nnt) {
    const int lane = threadIdx.x & 31, mi = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int nt = 0; nt < NR / 8; ++nt)
        if (nt < nnt) ldsm_x4(act + (mi >> 1) * (NR * APITCH) + (nt * 8 + rr) * APITCH + (kk + (mi & 1) * 8) * 2, f.b[nt][0], f.b[nt][1], f.b[nt][2], f.b[nt][3]);
#pragma unroll
    for (int g = 0; g < 2; ++g)
        if (g < ng) {
            const int row = min(g * 16 + (mi & 1) * 8 + rr, nrows - 1);
            ldsm_x4(wb + row * pitch + (kk + (mi >> 1) * 8) * 2, f.a[g][0], f.a[g][1], f.a[g][2], f.a[g][3]);
        }
}

// acc_h / acc_l[g][nt] += weight rows of granule g times the hi / lo activation rows of tile nt.
template <int NT>
__device__ __forceinline__ void frag_mma(const Frag &f, int ng, int nnt, float (&ah)[2][NT][4], float (&al)[2][NT][4]) {
#pragma unroll
    for (int g = 0; g < 2; ++g)
        if (g < ng)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                if (nt < nnt) {
                    mma16816(ah[g][nt], f.a[g][0], f.a[g][1], f.a[g][2], f.a[g][3], f.b[nt][0], f.b[nt][1]);  // hi plane
                    mma16816(al[g][nt], f.a[g][0], f.a[g][1], f.a[g][2], f.a[g][3], f.b[nt][2], f.b[nt][3]);  // lo plane
                }
}

// Relative-position attention of one (head, query row) (src/kernels.metal:293-348). Right after
// the barrier the item requests everything it needs at once: the query, key and position rows to
// registers, the value rows through registers into shared memory (16-byte L2 loads spread over all
// threads; they are needed last).
// LM: the window's rows at most (64 for the 8-row form, 72 for the 16-row one), LM / 8 keys per warp.
template <int LM>
__device__ __forceinline__ void attention_item(const NbEnc1Args &a, Smem &S, uint8_t *act, const NbEnc1Layer &w, int hd, int r, int pos, int cache_len) {
    constexpr int KI = LM / CWARPS;
    const int D = a.D, c = a.c, L = cache_len + c, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ld = 3 * (int64_t)D;
    const int off = hd * 128;
    const float *Kb = w.kv + (int64_t)(pos - cache_len) * ld + D + off;
    const float *Vb = Kb + D;
    const float *Pb = w.ptab + (int64_t)(a.Lmax - L + c - 1 - r) * D + off;
    float *Vs = (float *)act;  // [L][128]: the activation tile is idle here
    // query (lane's 4 dims) and this warp's keys j = warp + 8 i (i < KI covers L <= LM)
    const float4 q4 = __ldcg((const float4 *)(w.kv + (int64_t)(pos + r) * ld + off + 4 * lane));
    const float4 u4 = ld4g(w.bias_u + off + 4 * lane), v4 = ld4g(w.bias_v + off + 4 * lane);
    float4 k4[KI], p4[KI];
#pragma unroll
    for (int i = 0; i < KI; ++i) {
        const int j = warp + CWARPS * i;
        if (j < L) {
            k4[i] = __ldcg((const float4 *)(Kb + (int64_t)j * ld + 4 * lane));
            p4[i] = ld4g(Pb + (int64_t)j * D + 4 * lane);
        }
    }
    // value rows: element e = row e / 32, columns 4 (e % 32) .. +3, 16-byte asynchronous copies
    // straight into shared memory (no registers held), every one in flight at once, waited for
    // before the weighted sum
    for (int e = tid; e < L * 32; e += CTHREADS)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm100::smem_u32(Vs + 4 * e)), "l"((const float4 *)(Vb + (int64_t)(e >> 5) * ld) + (e & 31))
                     : "memory");
    const float4 qu = make_float4(q4.x + u4.x, q4.y + u4.y, q4.z + u4.z, q4.w + u4.w);
    const float4 qv = make_float4(q4.x + v4.x, q4.y + v4.y, q4.z + v4.z, q4.w + v4.w);
    // this lane's part of the KI scores (q + u).k_j + (q + v).p_j, all reduced over the warp by one
    // butterfly (lane 2 i then holds score i)
    static_assert(KI <= 16, "scores of one butterfly");
    float sv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int j = warp + CWARPS * i;
        sv[i] = 0.0f;
        if (i < KI && j < L)
            sv[i] = (qu.x * k4[i].x + qu.y * k4[i].y + qu.z * k4[i].z + qu.w * k4[i].w) + (qv.x * p4[i].x + qv.y * p4[i].y + qv.z * p4[i].z + qv.w * p4[i].w);
    }
    warp_fold<16>(sv);
    {
        const int i = lane >> 1, j = warp + CWARPS * i;
        if ((lane & 1) == 0 && i < KI && j < L) S.sc[j] = sv[0] * a.scale;
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");  // this thread's value copies
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
    cbar();
    const int d = tid & 127, half = tid >> 7;
    float acc = 0.0f;
    for (int j = half; j < L; j += 2) acc += S.sc[j] * Vs[j * 128 + d];
    S.vpart[half][d] = acc;
    cbar();
    if (tid < 128) a.att[(int64_t)r * D + off + tid] = S.vpart[0][tid] + S.vpart[1][tid];
    cbar();  // the value rows are read before the area is reused
}

// Grid-wide barrier of the compute threads (gridsync.cuh). Returns false when the launch is being
// abandoned.
// The small tensors block l reads (LayerNorm vectors, depthwise taps, position biases, the rows
// of its position table this chunk's attention reads) and its cache rows from earlier chunks (the
// attention's key/value history, the depthwise conv's history) brought into L2 by the issue warp
// ahead of the block, so the stages that read them find them there instead of waiting on HBM.
// The items are spread over the grid (CTA b takes items b, b + grid, ...; lane j of its issue warp
// the j-th of those), each requested once: 14 vectors, the depthwise taps, the conv history rows
// [pos - (taps - 1), pos) of the GLU output (pos >= taps - 1: they precede every chunk), the
// position-table rows, the history rows [pos - cache_len, pos) of q|k|v (3 D wide).
__device__ void prefetch_layer(const NbEnc1Args &a, int l, int pos, int cache_len, int pos_rows0, int pos_rows) {
    if (l >= a.layers || (threadIdx.x >> 5) != ISSUE_WARP) return;
    const NbEnc1Layer &w = a.L[l];
    const uint32_t vb = (uint32_t)a.D * 4;
    const int lane = threadIdx.x & 31, G = gridDim.x, nitems = 16 + pos_rows + cache_len;
    for (int i = blockIdx.x + lane * G; i < nitems; i += 32 * G) {
        if (i < 14) {
            const float *vec[14] = { w.ln_ff1_g, w.ln_ff1_b, w.ln_att_g, w.ln_att_b, w.ln_conv_g, w.ln_conv_b, w.ln_ff2_g,
                                     w.ln_ff2_b, w.ln_out_g, w.ln_out_b, w.bn_g, w.bn_b, w.bias_u, w.bias_v };
            prefetch_l2(vec[i], vb);
        } else if (i == 14) {
            prefetch_l2(w.dw_w, vb * (uint32_t)a.taps);
        } else if (i == 15) {
            if (a.taps > 1) prefetch_l2(w.din + (int64_t)(pos - (a.taps - 1)) * a.D, vb * (uint32_t)(a.taps - 1));
        } else if (i < 16 + pos_rows) {
            prefetch_l2(w.ptab + (int64_t)(pos_rows0 + i - 16) * a.D, vb);
        } else {
            prefetch_l2(w.kv + (int64_t)(pos - cache_len + (i - 16 - pos_rows)) * 3 * a.D, 3 * vb);
        }
    }
}


__device__ bool grid_sync(const NbEnc1Args &a, Smem &S, unsigned &epoch) {
    cbar();
    if (threadIdx.x == 0) {
        ++epoch;
        if (!nb::grid_arrive_wait(a.bar, epoch * gridDim.x, a.err, 1, WAIT_LIMIT)) S.abort = 1;
    }
    cbar();
    return !S.abort;
}

// Input rows of projection s of block l (hA: the block's input, hB: its residual after FF1b) and
// how they are normalised; the normalisation vectors (up to two LayerNorms).
__device__ __forceinline__ void stage_input(const NbEnc1Args &a, int l, int s, const float *hA, const float *hB, const float *&X, int &ldx, int &mode) {
    ldx = a.D;
    switch (s) {
    case 0: X = hA; mode = l > 0 ? P_LN2 : P_LN; break;
    case 1: case 7: X = a.ff; ldx = a.FF; mode = P_PLAIN; break;
    case 2: case 4: case 6: X = hB; mode = P_LN; break;
    case 3: X = a.att; mode = P_PLAIN; break;
    case 5: X = a.att; mode = P_DWLN; break;  // att holds the depthwise-conv output
    case 8: X = hA; mode = P_LNX; break;      // LN_out of the last block, then the prompt projection
    case 9: X = a.ph; ldx = a.PRH; mode = P_PLAIN; break;
    default: X = a.prompted; mode = P_PLAIN; break;
    }
}
__device__ __forceinline__ void stage_norm(const NbEnc1Args &a, int l, int s, float4 &ga, float4 &ba, float4 &gb, float4 &bb) {
    const NbEnc1Layer &w = a.L[s >= NSTAGE ? a.layers - 1 : l];
    const float *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
    switch (s) {
    case 0:
        if (l > 0) { g1 = a.L[l - 1].ln_out_g; b1 = a.L[l - 1].ln_out_b; g2 = w.ln_ff1_g; b2 = w.ln_ff1_b; }
        else { g1 = w.ln_ff1_g; b1 = w.ln_ff1_b; }
        break;
    case 2: g1 = w.ln_att_g; b1 = w.ln_att_b; break;
    case 4: g1 = w.ln_conv_g; b1 = w.ln_conv_b; break;
    case 5: g1 = w.bn_g; b1 = w.bn_b; break;
    case 6: g1 = w.ln_ff2_g; b1 = w.ln_ff2_b; break;
    case 8: g1 = w.ln_out_g; b1 = w.ln_out_b; break;  // the last block's output norm, before the prompt
    default: break;
    }
    const int k = 4 * threadIdx.x;
    ga = make_float4(1.f, 1.f, 1.f, 1.f);
    ba = make_float4(0.f, 0.f, 0.f, 0.f);
    gb = ga;
    bb = ba;
    if (g1 && k < (s == 1 || s == 7 ? a.FF : a.D)) {
        ga = ld4g(g1 + k);
        ba = ld4g(b1 + k);
        if (g2) { gb = ld4g(g2 + k); bb = ld4g(b2 + k); }
    }
}

// ---- LayerNorm folded into the projection that follows it ---------------------------------------
// For a row x with mean mu and inv = 1/sqrt(var + eps),
//   LN(x) W^T = inv (x (.) g) W^T - inv mu (g W^T) + b W^T,
// so the MMA runs on x (.) g while the statistics are reduced beside it, and the epilogue applies
//   out = inv (acc - mu F.x) + F.y,   F.x = sum_k g_k W_nk, F.y = sum_k b_k W_nk
// (per weight row, computed at set-up). The input of block l > 0 passes through LN_out of block
// l - 1 (g1, b1) and then LN_ff1 (g2, b2): the MMA runs on x (.) g1 (.) g2 and
//   out = inv2 (inv1 (acc - mu1 F.x) + F.y - mu2 F.z) + F.w,
//   F = (sum g1 g2 W, sum b1 g2 W, sum g2 W, sum b2 W),
// where mu2, inv2 (the statistics of y = LN_out(x)) follow from six row sums of x (x, x^2, x g1,
// x^2 g1^2, x g1^2, x g1 b1) and five sums of g1, b1 over the row (lnsum). With mu2 = 0, inv2 = 1
// and F.z = F.w = 0 the second form is the first, which is how the epilogue applies both.

// Rows of fold constants per block: FF1a (FF), QKV (3 D), PW1 (2 D, value and gate rows), FF2a (FF).
__host__ __device__ inline int fold_rows(int D, int FF) { return 2 * FF + 5 * D; }
__host__ __device__ inline int fold_off(int s, int D, int FF) { return s == 0 ? 0 : s == 2 ? FF : s == 4 ? FF + 3 * D : FF + 5 * D; }

// Set-up: one warp per (weight row, folded projection, block).
__global__ void encoder1_fold_kernel(const __grid_constant__ NbEnc1Args a, float4 *fold) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, s = 2 * blockIdx.y, l = blockIdx.z, D = a.D, FF = a.FF;
    const int rows = (s == 0 || s == 6) ? FF : s == 2 ? 3 * D : 2 * D, row = blockIdx.x * 8 + warp;
    if (row >= rows) return;
    const NbEnc1Layer &w = a.L[l];
    const uint16_t *W = (s == 0 ? w.ff1_w1 : s == 2 ? w.wqkv : s == 4 ? w.pw1 : w.ff2_w1) + (int64_t)row * D;
    const float *g2 = s == 0 ? w.ln_ff1_g : s == 2 ? w.ln_att_g : s == 4 ? w.ln_conv_g : w.ln_ff2_g;
    const float *b2 = s == 0 ? w.ln_ff1_b : s == 2 ? w.ln_att_b : s == 4 ? w.ln_conv_b : w.ln_ff2_b;
    const bool two = s == 0 && l > 0;
    const float *g1 = two ? a.L[l - 1].ln_out_g : g2, *b1 = two ? a.L[l - 1].ln_out_b : b2;
    float f0 = 0.0f, f1 = 0.0f, f2 = 0.0f, f3 = 0.0f;
    for (int k = lane; k < D; k += 32) {
        const float wk = nb::bf2f(W[k]);
        if (two) {
            f0 += (g1[k] * g2[k]) * wk;
            f1 += (b1[k] * g2[k]) * wk;
            f2 += g2[k] * wk;
            f3 += b2[k] * wk;
        } else {
            f0 += g2[k] * wk;
            f1 += b2[k] * wk;
        }
    }
    f0 = nb::warp_sum(f0);
    f1 = nb::warp_sum(f1);
    f2 = nb::warp_sum(f2);
    f3 = nb::warp_sum(f3);
    if (lane == 0) fold[(int64_t)l * fold_rows(D, FF) + fold_off(s, D, FF) + row] = make_float4(f0, f1, f2, f3);
}

// Set-up: the sums of LN_out's vectors of block l - 1 over the row, for block l (one warp each):
// lnsum[2 l] = (sum g1, sum g1^2, sum g1 b1, sum b1), lnsum[2 l + 1].x = sum b1^2.
__global__ void encoder1_lnsum_kernel(const __grid_constant__ NbEnc1Args a, float4 *lnsum) {
    const int l = blockIdx.x, lane = threadIdx.x;
    if (l == 0 || lane >= 32) return;
    const float *g1 = a.L[l - 1].ln_out_g, *b1 = a.L[l - 1].ln_out_b;
    float t[5] = { 0.f, 0.f, 0.f, 0.f, 0.f };
    for (int k = lane; k < a.D; k += 32) {
        t[0] += g1[k];
        t[1] += g1[k] * g1[k];
        t[2] += g1[k] * b1[k];
        t[3] += b1[k];
        t[4] += b1[k] * b1[k];
    }
#pragma unroll
    for (int j = 0; j < 5; ++j) t[j] = nb::warp_sum(t[j]);
    if (lane == 0) {
        lnsum[2 * l] = make_float4(t[0], t[1], t[2], t[3]);
        lnsum[2 * l + 1] = make_float4(t[4], 0.f, 0.f, 0.f);
    }
}

template <int V>
__device__ __forceinline__ void warp_fold_store(float (&x)[V], float *dst) {
    constexpr int VPL = V >= 32 ? V / 32 : 1;
    warp_fold<V>(x);
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < VPL; ++j) dst[lane * VPL + j] = x[j];
}
template <int V>
__device__ __forceinline__ int fs_pos(int v) { return V >= 32 ? v : 2 * v; }

// The row sums of a folded LayerNorm's input rows (this thread's columns), reduced per warp into
// S.fs[warp]: (sum x, sum x^2) per row, or for the block input of block l > 0 (two LayerNorms,
// g1 b1 the first one's vectors) (x, x^2, x g1, x^2 g1^2) per row at 0 and (x g1^2, x g1 b1) per
// row at 64.
template <int NR>
__device__ __forceinline__ void fold_sums(const Act<NR> &A, Smem &S, bool two, float4 g1, float4 b1) {
    float *dst = S.fs[threadIdx.x >> 5];
    if (!two) {
        float v[2 * NR];
#pragma unroll
        for (int u = 0; u < NR; ++u) {
            const float4 x = A.x[u];
            v[2 * u] = (x.x + x.y) + (x.z + x.w);
            v[2 * u + 1] = (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
        }
        warp_fold_store<2 * NR>(v, dst);
    } else {
        const float4 g2 = make_float4(g1.x * g1.x, g1.y * g1.y, g1.z * g1.z, g1.w * g1.w);
        const float4 gb = make_float4(g1.x * b1.x, g1.y * b1.y, g1.z * b1.z, g1.w * b1.w);
        {
            float v[4 * NR];
#pragma unroll
            for (int u = 0; u < NR; ++u) {
                const float4 x = A.x[u];
                const float4 xx = make_float4(x.x * x.x, x.y * x.y, x.z * x.z, x.w * x.w);
                v[4 * u] = (x.x + x.y) + (x.z + x.w);
                v[4 * u + 1] = (xx.x + xx.y) + (xx.z + xx.w);
                v[4 * u + 2] = (x.x * g1.x + x.y * g1.y) + (x.z * g1.z + x.w * g1.w);
                v[4 * u + 3] = (xx.x * g2.x + xx.y * g2.y) + (xx.z * g2.z + xx.w * g2.w);
            }
            warp_fold_store<4 * NR>(v, dst);
        }
        float v[2 * NR];
#pragma unroll
        for (int u = 0; u < NR; ++u) {
            const float4 x = A.x[u];
            v[2 * u] = (x.x * g2.x + x.y * g2.y) + (x.z * g2.z + x.w * g2.w);
            v[2 * u + 1] = (x.x * gb.x + x.y * gb.y) + (x.z * gb.z + x.w * gb.w);
        }
        warp_fold_store<2 * NR>(v, dst + 64);
    }
}

// Statistics of a folded LayerNorm for row u < c from the per-warp sums (the issue warp, after the
// CTA barrier that follows fold_sums): S.st[u][2..5] = mu1, inv1, mu2, inv2 (mu2 = 0, inv2 = 1 for
// one LayerNorm) and, for two, S.st[u][0..1] = mu1, inv1 for the FF1b epilogue.
template <int NR>
__device__ __forceinline__ void fold_stats(Smem &S, int u, bool two, int K, float eps, float4 G0, float G4) {
    const float invK = 1.0f / (float)K;
    if (!two) {
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) {
            s1 += S.fs[w][fs_pos<2 * NR>(2 * u)];
            s2 += S.fs[w][fs_pos<2 * NR>(2 * u + 1)];
        }
        const float mu = s1 * invK, inv = rsqrtf(fmaxf(s2 * invK - mu * mu, 0.0f) + eps);
        S.st[u][2] = mu; S.st[u][3] = inv; S.st[u][4] = 0.0f; S.st[u][5] = 1.0f;
        return;
    }
    float t[6] = { 0.f, 0.f, 0.f, 0.f, 0.f, 0.f };
#pragma unroll
    for (int w = 0; w < CWARPS; ++w) {
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] += S.fs[w][fs_pos<4 * NR>(4 * u + j)];
        t[4] += S.fs[w][64 + fs_pos<2 * NR>(2 * u)];
        t[5] += S.fs[w][64 + fs_pos<2 * NR>(2 * u + 1)];
    }
    // G0 = (sum g1, sum g1^2, sum g1 b1, sum b1), G4 = sum b1^2
    const float mu1 = t[0] * invK, inv1 = rsqrtf(fmaxf(t[1] * invK - mu1 * mu1, 0.0f) + eps);
    const float sy = inv1 * (t[2] - mu1 * G0.x) + G0.w;
    const float sa = t[3] - 2.0f * mu1 * t[4] + mu1 * mu1 * G0.y;  // sum (x - mu1)^2 g1^2
    const float sb = t[5] - mu1 * G0.z;                             // sum (x - mu1) g1 b1
    const float syy = inv1 * inv1 * sa + 2.0f * inv1 * sb + G4;
    const float mu2 = sy * invK, inv2 = rsqrtf(fmaxf(syy * invK - mu2 * mu2, 0.0f) + eps);
    S.st[u][0] = mu1; S.st[u][1] = inv1;
    S.st[u][2] = mu1; S.st[u][3] = inv1; S.st[u][4] = mu2; S.st[u][5] = inv2;
}

// NR: activation rows handled per stage (8 when c <= 8, else 16), NR / 8 MMA column tiles.
template <int NR>
__device__ void compute(const NbEnc1Args &a, Smem &S, uint8_t *ring, uint8_t *act) {
    constexpr int NT = NR / 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int D = a.D, c = a.c, nnt = NT;
    const int pos = *a.pos, cache_len = *a.cache_len;
    unsigned epoch = 0;
    int rbuf = 0;  // row-sum buffer
    int dlo, dhi;
    slice(D, gridDim.x, blockIdx.x, dlo, dhi);  // this CTA's columns of the D-wide buffers it zeroes
    float *hA = a.h, *hB = a.h2;                // a block runs hA -> hB (FF1b) -> hA (FF2b)
    int gi = 0;                                 // projection index
    Ring rq;                                    // weight ring (warp ISSUE_WARP)
    ring_init(a, S, rq);
    const uint64_t pol = evict_first_policy();
    issue_ahead(a, S, ring, rq, 0, pol, 1 << 30);
    float4 nga, nba, ngb, nbb;  // the next stage's normalisation vectors (this thread's columns)
    stage_norm(a, 0, 0, nga, nba, ngb, nbb);
    // position-table rows this chunk's attention reads: (Lmax - L) + (c - 1 - r) + j, j < L, r < c
    const int L_att = cache_len + c, pos_rows0 = a.Lmax - L_att, pos_rows = L_att + c - 1;
    prefetch_layer(a, 0, pos, cache_len, pos_rows0, pos_rows);
    prefetch_layer(a, 1, pos, cache_len, pos_rows0, pos_rows);
    // the blocks, then (tail) one more pass for the prompt and joint encoder projections
    const int passes = a.layers + (a.tail ? 1 : 0);
    for (int l = 0; l < passes && !S.abort; ++l) {
        const bool tl = l == a.layers;
        const NbEnc1Layer &w = a.L[tl ? a.layers - 1 : l];
        const int s_end = tl ? NALL : NSTAGE;
#pragma unroll 1
        for (int s = tl ? NSTAGE : 0; s < s_end; ++s, ++gi) {
            if (s == 3) {
                // attention over the cache window (the QKV stage's barrier made the rows visible)
                const int items = a.H * c;
                for (int it = blockIdx.x; it < items; it += gridDim.x) attention_item<NR == 8 ? 64 : MAXL>(a, S, act, w, it % a.H, it / a.H, pos, cache_len);
                if (!grid_sync(a, S, epoch)) break;
            }
            struct { int lo, hi, kr, krw; } g = { S.g_lo[s], S.g_hi[s], S.g_kr[s], S.g_krw[s] };
            const int R = g.hi - g.lo, nrows = S.g_rows[s], pitch = S.g_pitch[s], ng = (nrows + 15) / 16, K = g.krw;
            // input rows and their normalisation (this thread's vectors were requested before the
            // barrier that opened the stage)
            int mode, ldx;
            const float *X;
            stage_input(a, l, s, hA, hB, X, ldx, mode);
            const float4 ga = nga, ba = nba, gb = ngb;
            const bool fold = mode == P_LN || mode == P_LN2;
            // the input rows, all loads in flight together
            Act<NR> A;
            gather<NR>(A, X, ldx, g.kr * g.krw, K, c);
            const bool own = 4 * tid < K;
            // what the epilogue needs, requested with the input rows: the residual values (and
            // LN_out vectors) of this thread's items e = tid + 256 q, output column g.lo + e % R, row
            // e / R; for PW1 the depthwise taps and history rows of its conv item; for a fold of two
            // LayerNorms (issue warp) the LN_out sums of the row
            const Div dR = make_div(R);
            const bool need_base = ((s == 1 || s == 7) && g.kr == 0) || s == 3 || s == 5, need_ln = s == 1 && g.kr == 0 && l > 0;
            const float *resid = (s == 1) ? hA : hB;
            float base[2] = { 0.f, 0.f }, og[2] = { 1.f, 1.f }, ob[2] = { 0.f, 0.f };
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int e = tid + CTHREADS * q;
                if (R > 0 && e < R * c) {
                    const int r = div_q(dR, e), col = g.lo + (e - r * R);
                    if (need_base) base[q] = __ldcg(resid + (int64_t)r * D + col);
                    if (need_ln) { og[q] = __ldg(a.L[l - 1].ln_out_g + col); ob[q] = __ldg(a.L[l - 1].ln_out_b + col); }
                }
            }
            const bool dact = s == 4 && R > 0 && tid < R * c;
            const int er = div_q(dR, tid), en = tid - er * R;
            if (s == 4 && R > 0) {
                // the depthwise taps [channel][tap] and history rows [h][channel] (h < taps - 1: row
                // pos - (taps - 1) + h, which precedes pos) of this CTA's channels: 4-byte asynchronous
                // copies into shared memory, waited for before the conv (both are read-only during the
                // launch: the taps are weights, the history rows were written by earlier chunks)
                for (int e = tid; e < R * a.taps; e += CTHREADS)
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sm100::smem_u32(&S.cdw[0][0] + e)), "l"(w.dw_w + (int64_t)g.lo * a.taps + e) : "memory");
                for (int e = tid; e < (a.taps - 1) * R; e += CTHREADS) {
                    const int h = div_q(dR, e), n = e - h * R;
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sm100::smem_u32(&S.chist[h][n])),
                                 "l"(w.din + (int64_t)(pos - (a.taps - 1) + h) * D + g.lo + n) : "memory");
                }
            }
            float4 G0 = make_float4(0.f, 0.f, 0.f, 0.f);
            float G4 = 0.0f;
            if (mode == P_LN2 && warp == ISSUE_WARP) {
                const float4 *ls = (const float4 *)a.fold + (int64_t)a.layers * fold_rows(D, a.FF) + 2 * l;
                G0 = __ldg(ls);
                G4 = __ldg(ls + 1).x;
            }
            // the residual buffer the next FF-out stage accumulates into starts at zero (and the
            // prompt output the tail's second projection accumulates into)
            if (s == 0 || s == 6 || s == 8) {
                float *z = s == 0 ? hB : s == 6 ? hA : a.prompted;
                for (int e = tid; e < (dhi - dlo) * c; e += CTHREADS) z[(int64_t)(e / (dhi - dlo)) * D + dlo + e % (dhi - dlo)] = 0.0f;
            }
            // A compute warp whose projection was requested in an earlier stage waits for its weight
            // rows here, while the input rows are in flight; otherwise it waits after the activation
            // barrier, once the issue warp has made this stage's requests.
            const int slot = gi % NB;
            int wait_ok = 1;
            bool waited = false;
            if (warp != ISSUE_WARP && lane == 0 && *(volatile int *)&S.issued > gi) {
                waited = true;
                if (!sm100::mbar_wait(&S.full[slot], (gi / NB) & 1, WAIT_LIMIT)) wait_ok = 0;
            }
            if (fold) {
                // the MMA runs on x (.) g (x (.) g1 (.) g2 for two LayerNorms); the statistics are
                // finished by the issue warp during the MMAs
                fold_sums<NR>(A, S, mode == P_LN2, ga, ba);
                const float4 gp = mode == P_LN2 ? make_float4(ga.x * gb.x, ga.y * gb.y, ga.z * gb.z, ga.w * gb.w) : ga;
#pragma unroll
                for (int u = 0; u < NR; ++u) {
                    float4 &x = A.x[u];
                    x = own ? make_float4(x.x * gp.x, x.y * gp.y, x.z * gp.z, x.w * gp.w) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            } else if (mode == P_DWLN || mode == P_LNX) {
                float mean[NR], inv[NR];
                row_stats<NR>(A, S, rbuf, K, a.eps, mean, inv);
                const bool silu = mode == P_DWLN;
#pragma unroll
                for (int u = 0; u < NR; ++u) {
                    float4 &x = A.x[u];
                    x.x = (x.x - mean[u]) * inv[u] * ga.x + ba.x;
                    x.y = (x.y - mean[u]) * inv[u] * ga.y + ba.y;
                    x.z = (x.z - mean[u]) * inv[u] * ga.z + ba.z;
                    x.w = (x.w - mean[u]) * inv[u] * ga.w + ba.w;
                    if (silu) { x.x *= sigm(x.x); x.y *= sigm(x.y); x.z *= sigm(x.z); x.w *= sigm(x.w); }
                    if (!own) x = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            stage_store<NR>(A, act, c, K);
            // The activation tile is complete once all eight warps have stored their columns. The
            // issue warp signals its part (bar.arrive) and makes the weight stream's next requests
            // (everything before gi is released here; the current projection's rows too if the ring
            // had no room for them while the previous entry was held) while the other seven warps
            // run the MMAs: the requests cost ~0.5-1.7 K cycles, which the CTA barrier before the
            // MMAs used to add to every stage. The compute warps wait for the tile (and, if they
            // have not yet, each for this projection's weight rows; a warp whose wait gave up skips
            // its MMAs, and the launch stops after the MMA barrier).
            if (warp == ISSUE_WARP) {
                sm100::named_arrive(2, CTHREADS);
                issue_ahead(a, S, ring, rq, gi, pol, 1 << 30);
            } else {
                sm100::named_barrier(2, CTHREADS);
            }
            if (s == 0) prefetch_layer(a, l + 2, pos, cache_len, pos_rows0, pos_rows);
            bool wok = warp != ISSUE_WARP;
            if (wok) {
                if (lane == 0 && !waited && !sm100::mbar_wait(&S.full[slot], (gi / NB) & 1, WAIT_LIMIT)) wait_ok = 0;
                if (lane == 0 && !wait_ok) {
                    S.abort = 1;
                    atomicExch(&a.bar[1], 1u);
                    atomicCAS(a.err, 0, 3);
                }
                __syncwarp();  // the rows lane 0 saw arrive, before the other lanes' fragment loads
                wok = __shfl_sync(0xffffffffu, wait_ok, 0) != 0;
            }
            {
                float acc[2][NT][4], acl[2][NT][4], acc2[2][NT][4], acl2[2][NT][4];
#pragma unroll
                for (int gg = 0; gg < 2; ++gg)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[gg][nt][q] = acl[gg][nt][q] = acc2[gg][nt][q] = acl2[gg][nt][q] = 0.0f;
                if (nrows > 0 && wok) {
                    const uint32_t actb = sm100::smem_u32(act), wb = sm100::smem_u32(ring + S.ring_off[slot]);
                    // k-steps of this warp (the seven compute warps share them). Software-pipelined: the
                    // next k-step's fragments are requested before this one's MMAs, which alternate
                    // between two accumulator sets.
                    const int T = K / 16, kb = T / MWARPS, extra = T % MWARPS;
                    const int per = kb + (warp < extra ? 1 : 0), k0 = 16 * (warp * kb + min(warp, extra));
                    Frag f[2];
                    if (per > 0) frag_load<NR>(f[0], actb, wb, pitch, nrows, k0, ng, nnt);
#pragma unroll
                    for (int q = 0; q < KRW / 16 / MWARPS + 1; ++q) {
                        if (q >= per) break;
                        if (q + 1 < per) frag_load<NR>(f[(q + 1) & 1], actb, wb, pitch, nrows, k0 + (q + 1) * 16, ng, nnt);
                        if (q & 1) frag_mma<NT>(f[q & 1], ng, nnt, acc2, acl2);
                        else frag_mma<NT>(f[q & 1], ng, nnt, acc, acl);
                    }
                }
                if (warp != ISSUE_WARP)
#pragma unroll
                    for (int gg = 0; gg < 2; ++gg)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int q = 0; q < 4; ++q) S.red[warp][gg][nt][lane * 4 + q] = acc[gg][nt][q] + acl[gg][nt][q] + (acc2[gg][nt][q] + acl2[gg][nt][q]);
            }
            cbar();
            if (S.abort) break;
            // the statistics of a folded LayerNorm (issue warp, from the per-warp sums of fold_sums),
            // beside the reduction of the per-warp accumulators
            if (fold && warp == ISSUE_WARP && lane < c) fold_stats<NR>(S, lane, mode == P_LN2, D, a.eps, G0, G4);
            for (int e = tid; e < 2 * NT * 128; e += CTHREADS) {
                const int gg = e / (NT * 128), nt = (e >> 7) % NT, v = e & 127, ln = v >> 2, q = v & 3;
                float sum = 0.0f;
#pragma unroll
                for (int ww = 0; ww < MWARPS; ++ww) sum += S.red[ww][gg][nt][v];
                const int n = gg * 16 + (ln >> 2) + (q >= 2 ? 8 : 0), r = nt * 8 + (ln & 3) * 2 + (q & 1);
                S.outv[n][r] = sum;
            }
            cbar();
            // epilogue: items e = tid + 256 q (q < 2), output column g.lo + e % R, row e / R
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int e = tid + CTHREADS * q;
                if (R == 0 || e >= R * c) continue;
                const int r = div_q(dR, e), n = e - r * R, col = g.lo + n;
                float v = S.outv[n][r];
                const float4 *Fr = (const float4 *)(ring + S.ring_off[slot] + nrows * pitch);  // fold constants of the rows
                if (fold) {
                    const float4 F = Fr[n];
                    v = S.st[r][5] * (S.st[r][3] * (v - S.st[r][2] * F.x) + F.y - S.st[r][4] * F.z) + F.w;
                }
                switch (s) {
                case 0: case 6: a.ff[(int64_t)r * a.FF + col] = v * sigm(v); break;
                case 1: case 7: {
                    float add = 0.5f * v;
                    if (g.kr == 0) {
                        float b = base[q];
                        if (s == 1 && l > 0) b = (b - S.st[r][0]) * S.st[r][1] * og[q] + ob[q];  // x = LN_out_{l-1}(h)
                        add += b;
                    }
                    red_add((s == 1 ? hB : hA) + (int64_t)r * D + col, add);
                    break;
                }
                case 2: w.kv[(int64_t)(pos + r) * 3 * D + col] = v; break;
                case 3: case 5: hB[(int64_t)r * D + col] = base[q] + v; break;
                case 8: a.ph[(int64_t)r * a.PRH + col] = fmaxf(v + __ldg(a.pb0 + col), 0.0f); break;  // relu(x pw0^T + b_eff)
                case 9: red_add(a.prompted + (int64_t)r * D + col, v + (g.kr == 0 ? __ldg(a.pb2 + col) : 0.0f)); break;
                case 10: a.joint[(int64_t)r * a.JH + col] = v + __ldg(a.jb + col); break;
                default: {  // s == 4: GLU (gate row R + n, folded likewise)
                    const float4 F = Fr[R + n];
                    const float gt = S.st[r][5] * (S.st[r][3] * (S.outv[R + n][r] - S.st[r][2] * F.x) + F.y - S.st[r][4] * F.z) + F.w;
                    const float gv = v * sigm(gt);
                    w.din[(int64_t)(pos + r) * D + col] = gv;
                    S.glu[n][r] = gv;
                    break;
                }
                }
            }
            if (s == 4) {
                // causal depthwise conv of this CTA's channels (src/kernels.metal:361-380) over rows
                // pos - (taps - 1) .. pos + c - 1: tap t of row er reads history row er + t while that
                // precedes pos, else the GLU output of row er + t - (taps - 1)
                asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");  // the taps and history
                cbar();
                if (dact) {
                    float x = 0.0f;
#pragma unroll
                    for (int t = 0; t < 9; ++t) {
                        if (t >= a.taps) break;
                        const int h = er + t;  // tap t of row er: history row er + t, else GLU row h - (taps - 1)
                        x += (&S.cdw[0][0])[en * a.taps + t] * (h < a.taps - 1 ? S.chist[h][en] : S.glu[en][h - (a.taps - 1)]);
                    }
                    a.att[(int64_t)er * D + g.lo + en] = x;
                }
            }
            if (s + 1 < s_end) stage_norm(a, l, s + 1, nga, nba, ngb, nbb);
            else if (l + 1 < passes) stage_norm(a, l + 1, l + 1 == a.layers ? NSTAGE : 0, nga, nba, ngb, nbb);
            if (s + 1 == NALL) break;  // the joint encoder projection ends the launch: nothing reads it here
            if (!grid_sync(a, S, epoch)) break;
        }
    }
    if (tid == 0) S.consumed = gi;
    // output LayerNorm of the last block, as bf16 hi/lo planes for the prompt projection (one CTA:
    // 16 KB of stores after the last barrier)
    if (!S.abort && !a.tail && blockIdx.x == 0) {
        const NbEnc1Layer &w = a.L[a.layers - 1];
        Act<NR> A;
        gather<NR>(A, hA, D, 0, D, c);
        float mean[NR], inv[NR];
        row_stats<NR>(A, S, rbuf, D, a.eps, mean, inv);
        if (4 * tid < D) {
            const float4 gg = ld4g(w.ln_out_g + 4 * tid), bb = ld4g(w.ln_out_b + 4 * tid);
#pragma unroll
            for (int u = 0; u < NR; ++u) {
                if (u >= c) break;
                const float y[4] = { (A.x[u].x - mean[u]) * inv[u] * gg.x + bb.x, (A.x[u].y - mean[u]) * inv[u] * gg.y + bb.y,
                                     (A.x[u].z - mean[u]) * inv[u] * gg.z + bb.z, (A.x[u].w - mean[u]) * inv[u] * gg.w + bb.w };
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t idx = (int64_t)u * D + 4 * tid + j;
                    const uint16_t hb = nb::f2bf(y[j]);
                    a.xout[idx] = hb;
                    a.xout[idx + a.xout_plane] = nb::f2bf(y[j] - nb::bf2f(hb));
                }
            }
        }
    }
}

template <int NR>
__global__ void __launch_bounds__(THREADS, 1) encoder1_kernel(const __grid_constant__ NbEnc1Args a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *ring = smem_raw;
    uint8_t *act = smem_raw + a.ring_bytes;
    const int abytes = act_bytes(a.c, a.left + a.c);
    Smem &S = *(Smem *)(act + abytes);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NB; ++s) sm100::mbar_init(&S.full[s], 1);
        S.abort = 0;
        S.consumed = S.issued = 0;
        S.g_layer = layer_image_bytes(a.D, a.FF);
        sm100::fence_mbar_init();
    }
    // this CTA's part of each projection type (the same in every block)
    if (threadIdx.x < (a.tail ? NALL : NSTAGE)) {
        const int st = threadIdx.x;
        const Geo g = stage_geo(a, 0, st, blockIdx.x, gridDim.x);
        S.g_lo[st] = g.lo; S.g_hi[st] = g.hi; S.g_kr[st] = g.kr; S.g_krw[st] = g.krw;
        S.g_rows[st] = geo_rows(g); S.g_pitch[st] = geo_pitch(g); S.g_bytes[st] = geo_rows(g) * stage_row_bytes(st, g.krw);
        S.g_img[st] = image_offset(a, 0, st, g, blockIdx.x, gridDim.x) - (st >= NSTAGE ? (long long)a.layers * layer_image_bytes(a.D, a.FF) : 0);
    }
    // activation rows past c stay zero for the whole launch (the MMAs read 8 or 16 rows)
    for (int i = threadIdx.x; i < abytes / 16; i += THREADS) ((uint4 *)act)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    compute<NR>(a, S, ring, act);
    __syncthreads();
    // copies requested but never taken (an abandoned launch): wait for them (bounded) before the
    // CTA's shared memory goes away. At most NB entries are in flight, each in its own slot.
    if (threadIdx.x == 0 && S.abort) {
        for (int j = S.consumed; j < S.issued; ++j) sm100::mbar_wait(&S.full[j % NB], (j / NB) & 1, WAIT_LIMIT / 8);
    }
}

}  // namespace

// Bytes of the weight ring for a model of width D / FF on `grid` CTAs with `smem_optin` bytes of
// shared memory per CTA, for a chunk of c rows and attention windows of up to Lw rows (the ring
// takes what the activation area leaves; its entries live within one launch); 0 when the ring
// could not hold two of the largest entries.
extern "C" int nb_encoder1_ring_bytes(int D, int FF, int grid, size_t smem_optin, int c, int Lw) {
    int biggest = 0;
    const int outs[NSTAGE] = { FF, D, 3 * D, D, D, D, FF, D }, Ks[NSTAGE] = { D, FF, D, D, D, D, D, FF }, mult[NSTAGE] = { 1, 1, 1, 1, 2, 1, 1, 1 };
    for (int s = 0; s < NSTAGE; ++s) {
        const int krw = Ks[s] <= KRW ? Ks[s] : KRW, ranges = Ks[s] / krw, groups = grid / ranges;
        if (groups < 1) return 0;
        const int R = (outs[s] + groups - 1) / groups;
        if (mult[s] * R > MAXR) return 0;
        const int b = mult[s] * R * stage_row_bytes(s, krw);
        if (b > biggest) biggest = b;
    }
    const long long avail = (long long)smem_optin - act_bytes(c, Lw) - (long long)sizeof(Smem) - 1024;
    const long long ring = avail / 128 * 128;
    return ring >= 2LL * biggest ? (int)ring : 0;
}

extern "C" size_t nb_encoder1_smem(int ring_bytes, int c, int Lw) { return (size_t)ring_bytes + act_bytes(c, Lw) + sizeof(Smem); }

extern "C" size_t nb_encoder1_image_bytes(int D, int FF, int layers) { return (size_t)layers * (size_t)layer_image_bytes(D, FF); }
extern "C" size_t nb_encoder1_tail_image_bytes(int D, int PRH, int JH) { return (size_t)tail_image_bytes(D, PRH, JH); }

// Bytes of the LayerNorm fold constants: per block one float4 per row of the folded projections,
// then two float4 of LN_out sums per block.
extern "C" size_t nb_encoder1_fold_bytes(int D, int FF, int layers) { return (size_t)layers * (size_t)(fold_rows(D, FF) + 2) * 16; }

// Builds the weight image for a persistent grid of `grid` CTAs and the LayerNorm fold constants
// (args: the layer table and widths).
extern "C" int nb_encoder1_repack(const NbEnc1Args *args, int grid, uint8_t *image, float *fold, void *stream) {
    if (!image || ((uintptr_t)image & 15)) return nb_set_error("persistent encoder: weight image missing or misaligned");
    if (!fold || ((uintptr_t)fold & 15)) return nb_set_error("persistent encoder: fold constants missing or misaligned");
    NbEnc1Args a = *args;
    a.fold = fold;  // the repack kernel copies the constants into the image
    cudaStream_t st = (cudaStream_t)stream;
    const int maxrows = a.FF > 3 * a.D ? a.FF : 3 * a.D;
    if (cudaMemsetAsync(fold, 0, nb_encoder1_fold_bytes(a.D, a.FF, a.layers), st) != cudaSuccess)
        return nb_set_error("persistent encoder: %s", cudaGetErrorString(cudaGetLastError()));
    encoder1_fold_kernel<<<dim3((maxrows + 7) / 8, 4, a.layers), 256, 0, st>>>(a, (float4 *)fold);
    if (nb_check_launch("encoder1_fold_kernel")) return -1;
    encoder1_lnsum_kernel<<<a.layers, 32, 0, st>>>(a, (float4 *)fold + (size_t)a.layers * fold_rows(a.D, a.FF));
    if (nb_check_launch("encoder1_lnsum_kernel")) return -1;
    encoder1_repack_kernel<<<dim3(grid, NSTAGE, a.layers), 256, 0, st>>>(a, image, 0);
    if (nb_check_launch("encoder1_repack_kernel")) return -1;
    if (!a.tail) return 0;
    if (!a.pw0 || !a.pw2 || !a.jw || a.PRH % 128 || (a.PRH > KRW && a.PRH % KRW) || a.JH % 16 || a.pw0_ld < a.D || a.pw0_ld % 8)
        return nb_set_error("persistent encoder: unsupported tail (prompt %d, joint %d)", a.PRH, a.JH);
    encoder1_repack_kernel<<<dim3(grid, NTAIL, 1), 256, 0, st>>>(a, image, NSTAGE);
    return nb_check_launch("encoder1_repack_kernel");
}

extern "C" int nb_encoder1(const NbEnc1Args *args, int grid, void *stream) {
    const NbEnc1Args &a = *args;
    if (a.c < 1 || a.c > MAXC) return nb_set_error("persistent encoder: %d rows per chunk (1..%d)", a.c, MAXC);
    if (a.D % 128 || a.D > KRW || a.FF % 128 || (a.FF > KRW && a.FF % KRW))
        return nb_set_error("persistent encoder: unsupported widths D=%d FF=%d", a.D, a.FF);
    if (a.H * 128 != a.D) return nb_set_error("persistent encoder: heads of 128 expected");
    if (a.Lmax > MAXL || a.left < 0 || a.left + a.c > MAXL) return nb_set_error("persistent encoder: attention window %d above %d rows", a.left + a.c, MAXL);
    if (a.taps < 1 || a.taps > 9) return nb_set_error("persistent encoder: depthwise kernel of %d taps (1..9)", a.taps);
    if (!a.h2 || a.h2 == a.h) return nb_set_error("persistent encoder: needs two residual buffers");
    if (!a.image || !a.fold) return nb_set_error("persistent encoder: no weight image or fold constants");
    if (a.ring_bytes <= 0 || a.ring_bytes % 128) return nb_set_error("persistent encoder: weight ring of %d bytes", a.ring_bytes);
    if (a.tail && (!a.pw0 || !a.pw2 || !a.jw || !a.pb0 || !a.pb2 || !a.jb || !a.ph || !a.prompted || !a.joint || a.PRH % 128 || (a.PRH > KRW && a.PRH % KRW) ||
                   a.JH % 16))
        return nb_set_error("persistent encoder: incomplete tail (prompt %d, joint %d)", a.PRH, a.JH);
    const size_t smem = nb_encoder1_smem(a.ring_bytes, a.c, a.left + a.c);
    // rows <= 8: one MMA column tile and half the registers of the 16-row form
    const bool eight = act_rows(a.c, a.left + a.c) == 8;
    const void *fn = eight ? (const void *)encoder1_kernel<8> : (const void *)encoder1_kernel<16>;
    if (nb_smem_attr(fn, smem)) return nb_set_error("persistent encoder: %s", nemo_gpu_last_error());
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
    const cudaError_t e = eight ? cudaLaunchKernelEx(&cfg, encoder1_kernel<8>, a) : cudaLaunchKernelEx(&cfg, encoder1_kernel<16>, a);
    if (e != cudaSuccess) return nb_set_error("persistent encoder: %s", cudaGetErrorString(cudaGetLastError()));
    return nb_check_launch("encoder1_kernel");
}
