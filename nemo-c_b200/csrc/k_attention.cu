// Relative-position self-attention of one chunk over the per-stream K/V cache window
// (src/kernels.metal:293-348, dispatched at src/encoder.c:161-165):
//   s[i][j] = ((q_i + u) . k_j + (q_i + v) . P[(Lmax - L) + (c - 1 - i + j)]) * scale
//   softmax over all L keys (no mask inside the window), o_i = sum_j p[i][j] v_j.
// The position term only depends on c - 1 - i + j, so G[i][r] = (q_i + v) . P[r0 + r] is
// computed once per position row r (L + c - 1 rows) and read back diagonally.
//
// Two kernels, one CTA (8 warps) per (head, stream) each: attention8_kernel for chunks of up to 8
// rows (keys and position rows on the MMA's 16-row side, queries on its 8 columns) and
// attention_kernel for up to 16 rows (queries on the 16-row side). The three products (content
// and position scores, probabilities times V) run on the tensor cores as mma.sync m16n8k16 tiles
// with both operands split into bf16 hi + lo parts and four products per k-step (hi.hi, lo.hi,
// hi.lo, lo.lo) into three fp32 accumulators. The softmax stays in fp32 with IEEE expf.
//
// attention_kernel: the stream's V rows of the head (half of the HBM traffic of the kernel) are
// requested as the CTA starts, 16-byte asynchronous copies into shared memory spread over all
// threads (no registers held, so three CTAs fit an SM); the K rows are read straight into the
// score tiles' fragments by warps 0-3 (each row read by one thread group as float4s, 64 bytes
// per k-step) while warps 4-7 form the position scores. Issuing one bulk copy per 512-byte row
// instead cost more than the transfer itself.
#include <cuda_bf16.h>
#include "common.cuh"
#include "sm100.cuh"

namespace {

constexpr int DH = 128;
constexpr int THREADS = 256;
constexpr int MAXC = 16;   // rows per chunk (the MMA's 16 rows)
constexpr int MAXL = 96;   // keys in the window
// Shared-memory row pitch of V (floats), read as scalars down 4 row pairs: 4 mod 32 banks keeps the
// fragment loads conflict-free.
constexpr int VP = DH + 4;

__device__ int g_att_error;  // nonzero once a CTA gave up waiting (no wait left in this kernel: stays 0)

// hi = bf16(x), lo = bf16(x - hi) of a pair, packed two per register (first element low)
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - __low2float(h), x1 - __high2float(h));
    hi = *(const uint32_t *)&h;
    lo = *(const uint32_t *)&l;
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The four products of split operands into three accumulators (hi.hi; lo.hi; hi.lo and lo.lo):
// independent chains, so consecutive MMAs of a warp overlap instead of waiting on one another.
__device__ __forceinline__ void mma3(float (&d)[3][4], const uint32_t (&ah)[4], const uint32_t (&al)[4], const uint32_t (&bh)[2], const uint32_t (&bl)[2]) {
    mma16816(d[0], ah, bh[0], bh[1]);
    mma16816(d[1], al, bh[0], bh[1]);
    mma16816(d[2], al, bl[0], bl[1]);
    mma16816(d[2], ah, bl[0], bl[1]);
}

// Sum of accumulator sets: small terms first
template <int N>
__device__ __forceinline__ void acc_sum(const float (&d)[N][4], float (&out)[4]) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float v = 0.0f;
#pragma unroll
        for (int j = N - 1; j >= 0; --j) v += d[j][e];
        out[e] = v;
    }
}

// Query operand of the score tiles as bf16 hi and lo planes [16][QP] (rows i >= c zero): built
// once per CTA, read by every warp as A fragments with 32-bit loads.
constexpr int QP = DH + 8;  // bf16 pitch: 68 words, so the 8 row groups of a fragment hit distinct banks

// Plane column of the head-dim pair (d, d + 1), d even: within each 16-dim block, dims 4u .. 4u + 3
// sit at columns 2u, 2u + 1, 2u + 8, 2u + 9, so that lane t's B operand of a k-step is the float4 at
// dims 4t .. 4t + 3 of a row (the dot products are unchanged by this common permutation).
__device__ __forceinline__ int qcol(int d) { return (d & ~15) + ((d & 2) ? 8 : 0) + ((d & 12) >> 1); }

// A fragment (16 x 16, row-major) of k-step k0: a0 (g, 2t..2t+1), a1 (g+8, 2t..), a2 (g, 2t+8..),
// a3 (g+8, 2t+8..), g = lane / 4, t = lane % 4.
__device__ __forceinline__ void a_frag(const uint16_t *hi, const uint16_t *lo, int k0, int lane, uint32_t (&ah)[4], uint32_t (&al)[4]) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int o = (g + 8 * (e & 1)) * QP + k0 + 2 * t + 8 * (e >> 1);
        ah[e] = *(const uint32_t *)(hi + o);
        al[e] = *(const uint32_t *)(lo + o);
    }
}

// The lane's operand values of one score tile (see score_tile), every load in flight at once.
__device__ __forceinline__ void tile_load(const float *src, int64_t pitch, int r0, int nrows, int lane, float2 (&b)[16]) {
    const int g = lane >> 2, t = lane & 3;
    const bool ok = r0 + g < nrows;
    const float *row = src + (int64_t)(ok ? r0 + g : 0) * pitch + 4 * t;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        const float4 v = ok ? *(const float4 *)(row + 16 * ks) : make_float4(0.f, 0.f, 0.f, 0.f);
        b[2 * ks] = make_float2(v.x, v.y);
        b[2 * ks + 1] = make_float2(v.z, v.w);
    }
}

// Scores of 8 rows (one n-tile) against the 16 query rows: rows r0 + g of `src` (pitch `pitch`,
// rows >= nrows read as zero), 128 dims; result d[] in C-fragment layout. b: the tile's values
// when already loaded (pre), else loaded here.
__device__ __forceinline__ void score_tile(const uint16_t *qhi, const uint16_t *qlo, const float *src, int64_t pitch, int r0, int nrows, int lane,
                                           float (&d)[4], const float2 *pre = nullptr) {
    float2 b[16];
    if (pre) {
#pragma unroll
        for (int j = 0; j < 16; ++j) b[j] = pre[j];
    } else {
        tile_load(src, pitch, r0, nrows, lane, b);
    }
    // two k-step parities x three products: six accumulation chains of four MMAs each
    float acc[2][3][4] = {};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        uint32_t ah[4], al[4], bh[2], bl[2];
        a_frag(qhi, qlo, 16 * ks, lane, ah, al);
        split2(b[2 * ks].x, b[2 * ks].y, bh[0], bl[0]);
        split2(b[2 * ks + 1].x, b[2 * ks + 1].y, bh[1], bl[1]);
        mma3(acc[ks & 1], ah, al, bh, bl);
    }
    float d0[4], d1[4];
    acc_sum(acc[0], d0);
    acc_sum(acc[1], d1);
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] = d0[e] + d1[e];
}

// Shared-memory floats of one CTA: V rows [Lmax][VP], content scores / probabilities [16][Lmax],
// position scores [16][Lmax + 16], then the query operands (q + v) and (q + u) as bf16 hi / lo
// planes [16][QP] each.
__host__ __device__ __forceinline__ int smem_floats(int Lmax) {
    return Lmax * VP + MAXC * Lmax + MAXC * (Lmax + MAXC) + 4 * MAXC * QP / 2;
}

// 16-byte global -> shared copy through L2 (the rows were written by the projection just before),
// completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm100::smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(THREADS, 3) attention_kernel(const float *__restrict__ Q, int64_t ldq, int64_t q_sstride, const float *__restrict__ K,
                                                            const float *__restrict__ V, int64_t ldk, int64_t kv_sstride, const int *pos_p,
                                                            const int *cache_len_p, const float *__restrict__ P, const float *__restrict__ bias_u,
                                                            const float *__restrict__ bias_v, void *O, int o_fmt, int64_t o_plane, int64_t o_sstride,
                                                            int c, int Lmax, int D, float scale) {
    extern __shared__ __align__(16) float sm[];
    float *Vs = sm, *sk = Vs + Lmax * VP, *gp = sk + MAXC * Lmax;
    uint16_t *qvh = (uint16_t *)(gp + MAXC * (Lmax + MAXC)), *qvl = qvh + MAXC * QP, *quh = qvl + MAXC * QP, *qul = quh + MAXC * QP;
    const int gpl = Lmax + MAXC;  // pitch of gp
    nb::pdl_wait();
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int pos = *pos_p, cache_len = *cache_len_p, L = cache_len + c;
    if (L > MAXL || L > Lmax || c > MAXC || pos - cache_len < 0) return; // the host keeps these in range
    const int NP = L + c - 1, prow0 = Lmax - L, off = h * DH;
    const float *Kb = K + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    const float *Vb = V + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    // content tile `warp` (K rows 8 warp .. +7, from HBM), requested before anything else: its
    // latency passes while the query operand is built
    const int ntP = (NP + 7) >> 3, ntK = (L + 7) >> 3;
    float2 b0[16];
    if (warp < ntK) tile_load(Kb, ldk, warp * 8, L, lane, b0);
    // the query pairs straight from global memory (just written by the projection) and the biases,
    // requested first: the position scores wait on them, not on the window
    const float *Qb = Q + (int64_t)s * q_sstride + (int64_t)pos * ldq + off;
    float2 qq[4], bu2[4], bv2[4];  // this thread's pairs (i, 2p .. 2p + 1), i = e / 64, p = e % 64
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int e = tid + r * THREADS, i = e >> 6, k = 2 * (e & 63);
        qq[r] = i < c ? *(const float2 *)(Qb + (int64_t)i * ldq + k) : make_float2(0.f, 0.f);
        bu2[r] = *(const float2 *)(bias_u + off + k);
        bv2[r] = *(const float2 *)(bias_v + off + k);
    }
    // the window's V rows: asynchronous 16-byte copies into shared memory, every one in flight now
    // (element e: row e / 32, columns 4 (e % 32) .. +3), no registers held
    for (int e = tid; e < L * 32; e += THREADS) {
        const int r = e >> 5, c4 = 4 * (e & 31);
        cp_async16(Vs + r * VP + c4, Vb + (int64_t)r * ldk + c4);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int e = tid + r * THREADS, i = e >> 6, k = qcol(2 * (e & 63));
        const float2 q = qq[r];
        uint32_t h, l;
        split2(i < c ? q.x + bv2[r].x : 0.0f, i < c ? q.y + bv2[r].y : 0.0f, h, l);
        *(uint32_t *)(qvh + i * QP + k) = h;
        *(uint32_t *)(qvl + i * QP + k) = l;
        split2(i < c ? q.x + bu2[r].x : 0.0f, i < c ? q.y + bu2[r].y : 0.0f, h, l);
        *(uint32_t *)(quh + i * QP + k) = h;
        *(uint32_t *)(qul + i * QP + k) = l;
    }
    __syncthreads();
    // the score tiles: content (q + u) . k from the K rows, read straight from global memory, and
    // position (q + v) . P from the L2-resident table. Each warp first finishes the content tile it
    // requested above; the rest (the position tiles, then content tiles 8 ..) go round-robin.
    const float *Pb = P + (int64_t)prow0 * D + off;
    auto put_k = [&](int nt, const float (&d)[4]) {
        const int col = nt * 8 + 2 * t;
        if (g < c) { if (col < L) sk[g * Lmax + col] = d[0]; if (col + 1 < L) sk[g * Lmax + col + 1] = d[1]; }
        if (g + 8 < c) { if (col < L) sk[(g + 8) * Lmax + col] = d[2]; if (col + 1 < L) sk[(g + 8) * Lmax + col + 1] = d[3]; }
    };
    if (warp < ntK) {
        float d[4];
        score_tile(quh, qul, Kb, ldk, warp * 8, L, lane, d, b0);
        put_k(warp, d);
    }
    const int nrest = ntP + (ntK > THREADS / 32 ? ntK - THREADS / 32 : 0);
    for (int j = warp; j < nrest; j += THREADS / 32) {
        float d[4];
        if (j < ntP) {
            score_tile(qvh, qvl, Pb, D, j * 8, NP, lane, d);
            const int col = j * 8 + 2 * t;
            if (g < c) { if (col < NP) gp[g * gpl + col] = d[0]; if (col + 1 < NP) gp[g * gpl + col + 1] = d[1]; }
            if (g + 8 < c) { if (col < NP) gp[(g + 8) * gpl + col] = d[2]; if (col + 1 < NP) gp[(g + 8) * gpl + col + 1] = d[3]; }
        } else {
            const int nt = THREADS / 32 + j - ntP;
            score_tile(quh, qul, Kb, ldk, nt * 8, L, lane, d);
            put_k(nt, d);
        }
    }
    cp_async_wait_all();
    __syncthreads();
    // softmax of each query row (one warp per row); rows c..15 become zero probabilities
    for (int i = warp; i < MAXC; i += THREADS / 32) {
        if (i >= c) {
            for (int j = lane; j < Lmax; j += 32) sk[i * Lmax + j] = 0.0f;
            continue;
        }
        float sv[3], mx = -INFINITY;
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int j = lane + 32 * q;
            sv[q] = j < L ? (sk[i * Lmax + j] + gp[i * gpl + c - 1 - i + j]) * scale : -INFINITY;
            mx = fmaxf(mx, sv[q]);
        }
        mx = nb::warp_max(mx);
        float sum = 0.0f;
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int j = lane + 32 * q;
            sv[q] = j < L ? expf(sv[q] - mx) : 0.0f;
            sum += sv[q];
        }
        sum = nb::warp_sum(sum);
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int j = lane + 32 * q;
            if (j < Lmax) sk[i * Lmax + j] = j < L ? sv[q] / sum : 0.0f;
        }
    }
    __syncthreads();
    // o = p . V: warp w owns head dims [16w, 16w + 16) (two n-tiles); k runs over the L keys
    // (probabilities beyond L are zero and V rows beyond L are not read)
    float acc[2][2][3][4] = {};  // [n-tile][k-step parity][product]
    const int ksteps = (L + 15) >> 4;
    for (int ks0 = 0; ks0 < ksteps; ks0 += 2)
#pragma unroll
        for (int par = 0; par < 2; ++par) {  // k-step parity picks the accumulator set (static index)
            const int k0 = 16 * (ks0 + par);
            if (ks0 + par >= ksteps) break;
            uint32_t ah[4], al[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = g + 8 * (q & 1), k = k0 + 2 * t + 8 * (q >> 1);
                const float x0 = k < Lmax ? sk[i * Lmax + k] : 0.0f, x1 = k + 1 < Lmax ? sk[i * Lmax + k + 1] : 0.0f;
                split2(x0, x1, ah[q], al[q]);
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const int n = 16 * warp + 8 * nt + g;
                float v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int k = k0 + 2 * t + (q & 1) + 8 * (q >> 1);
                    v[q] = k < L ? Vs[k * VP + n] : 0.0f;
                }
                uint32_t bh[2], bl[2];
                split2(v[0], v[1], bh[0], bl[0]);
                split2(v[2], v[3], bh[1], bl[1]);
                mma3(acc[nt][par], ah, al, bh, bl);
            }
        }
    float o[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
        float a0[4], a1[4];
        acc_sum(acc[nt][0], a0);
        acc_sum(acc[nt][1], a1);
#pragma unroll
        for (int e = 0; e < 4; ++e) o[nt][e] = a0[e] + a1[e];
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
        const int col = off + 16 * warp + 8 * nt + 2 * t;
        if (g < c) {
            nb::store_act(O, o_fmt, o_plane, (int64_t)s * o_sstride + (int64_t)g * D + col, o[nt][0]);
            nb::store_act(O, o_fmt, o_plane, (int64_t)s * o_sstride + (int64_t)g * D + col + 1, o[nt][1]);
        }
        if (g + 8 < c) {
            nb::store_act(O, o_fmt, o_plane, (int64_t)s * o_sstride + (int64_t)(g + 8) * D + col, o[nt][2]);
            nb::store_act(O, o_fmt, o_plane, (int64_t)s * o_sstride + (int64_t)(g + 8) * D + col + 1, o[nt][3]);
        }
    }
}

// ---- chunks of up to 8 rows ---------------------------------------------------------------
// The same products with the window's keys / position rows as the MMA's 16-row side and the
// chunk's <= 8 query rows as its 8 columns, so no MMA row is padding when c <= 8 (the kernel
// above spends 16 query rows on every tile). K and V rows of the head come into shared memory as
// 16-byte asynchronous copies: K by warps 0-3 right after the query rows are requested (so that
// those do not queue behind them), V by warps 4-7 only once their first position tile's loads are
// out (the V rows are needed last; requested with K they delayed it: 49 -> 45 us per launch). Warps 4-7 form
// position row tiles 0-3 from P rows read straight from L2 (a whole tile in flight at once);
// warps 0-3 form position tiles 4, 5, ... while their K rows are in flight, then the content
// scores from shared K. The query operands are bf16 hi / lo planes read with ldmatrix, the
// probabilities are split into hi / lo planes once by the softmax, and the P . V product runs as
// V^T (16 head dims per warp) times P^T (8 query columns). Two CTAs fit an SM. (A persistent
// variant with one head per CTA, its position fragments kept in registers and a 3-slot ring of
// K / V rows, took 47 us against 49 us alone but cost more inside the encoder step, where the
// window grows from chunk to chunk and every stream paid its four barriers.)
constexpr int KP = DH + 16;  // K row pitch (floats): 16 mod 32 banks, conflict-free float4 fragment reads
constexpr int QP8 = DH + 8;  // query plane pitch (bf16): 272 bytes, odd multiple of 16 (ldmatrix rows on distinct banks)

// Query planes' column of the head-dim pair (d, d + 1) is qcol(d) (as above): lane t's A operand of
// a k-step is then the float4 at dims 16 ks + 4 t of a K / P row.

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}

// A fragment (rows g and g + 8 of a 16-row tile) of one k-step from the float4s x0 (row g) and
// x1 (row g + 8) at dims 16 ks + 4 t .. + 3, split into hi / lo.
__device__ __forceinline__ void a_split(const float4 &x0, const float4 &x1, uint32_t (&ah)[4], uint32_t (&al)[4]) {
    split2(x0.x, x0.y, ah[0], al[0]);
    split2(x1.x, x1.y, ah[1], al[1]);
    split2(x0.z, x0.w, ah[2], al[2]);
    split2(x1.z, x1.w, ah[3], al[3]);
}

// Shared-memory floats of attention8_kernel: K rows [L16][KP], V rows [L16][VP], content scores
// [8][Lmax], position scores [8][Lmax + 16], query planes (q + u, q + v; hi / lo) [8][QP8] bf16,
// probability planes hi / lo [8][L16 + 8] bf16. L16 = Lmax rounded up to 16.
__host__ __device__ __forceinline__ int smem8_floats(int Lmax) {
    const int L16 = (Lmax + 15) & ~15;
    return L16 * KP + L16 * VP + 8 * Lmax + 8 * (Lmax + 16) + (4 * 8 * QP8 + 2 * 8 * (L16 + 8)) / 2;
}

__global__ void __launch_bounds__(THREADS, 2) attention8_kernel(const float *__restrict__ Q, int64_t ldq, int64_t q_sstride, const float *__restrict__ K,
                                                             const float *__restrict__ V, int64_t ldk, int64_t kv_sstride, const int *pos_p,
                                                             const int *cache_len_p, const float *__restrict__ P, const float *__restrict__ bias_u,
                                                             const float *__restrict__ bias_v, void *O, int o_fmt, int64_t o_plane, int64_t o_sstride,
                                                             int c, int Lmax, int D, float scale) {
    extern __shared__ __align__(16) float sm[];
    const int L16 = (Lmax + 15) & ~15, gpl = Lmax + 16, PP = L16 + 8;
    float *Ks = sm, *Vs = Ks + L16 * KP, *sk = Vs + L16 * VP, *gp = sk + 8 * Lmax;
    uint16_t *quh = (uint16_t *)(gp + 8 * gpl), *qul = quh + 8 * QP8, *qvh = qul + 8 * QP8, *qvl = qvh + 8 * QP8;
    uint16_t *pph = qvl + 8 * QP8, *ppl = pph + 8 * PP;
    nb::pdl_wait();
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int pos = *pos_p, cache_len = *cache_len_p, L = cache_len + c;
    if (L > MAXL || L > Lmax || c > 8 || pos - cache_len < 0) return;  // the host keeps these in range
    const int NP = L + c - 1, prow0 = Lmax - L, off = h * DH, Lr = (L + 15) & ~15;
    const float *Kb = K + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    const float *Vb = V + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    // this thread's query pairs (rows i = tid / 64 and + 4, dims d, d + 1) and biases, requested
    // before the window's copies so that they do not queue behind them
    const float *Qb = Q + (int64_t)s * q_sstride + (int64_t)pos * ldq + off;
    const int qd = 2 * (tid & 63);
    const float2 bu = *(const float2 *)(bias_u + off + qd), bv = *(const float2 *)(bias_v + off + qd);
    float2 qq[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int i = (tid >> 6) + 4 * r;
        qq[r] = i < c ? *(const float2 *)(Qb + (int64_t)i * ldq + qd) : make_float2(0.f, 0.f);
    }
    // the window's K rows (warps 0-3): 16-byte asynchronous copies, all in flight now (element e:
    // row e / 32, columns 4 (e % 32) .. + 3); V rows L .. Lr - 1 zero (their probabilities are
    // zero, and the rows must be finite)
    if (warp < 4) {
        for (int e = tid; e < L * 32; e += 128) {
            const int r = e >> 5, c4 = 4 * (e & 31);
            cp_async16(Ks + r * KP + c4, Kb + (int64_t)r * ldk + c4);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
        for (int e = tid - 128; e < (Lr - L) * DH; e += 128) Vs[(L + e / DH) * VP + e % DH] = 0.0f;
    }
    // query operands: (q + u) and (q + v) as bf16 hi / lo planes, rows >= c zero
    {
        const int k = qcol(qd);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int i = (tid >> 6) + 4 * r;
            const bool ok = i < c;
            uint32_t hh, ll;
            split2(ok ? qq[r].x + bu.x : 0.0f, ok ? qq[r].y + bu.y : 0.0f, hh, ll);
            *(uint32_t *)(quh + i * QP8 + k) = hh;
            *(uint32_t *)(qul + i * QP8 + k) = ll;
            split2(ok ? qq[r].x + bv.x : 0.0f, ok ? qq[r].y + bv.y : 0.0f, hh, ll);
            *(uint32_t *)(qvh + i * QP8 + k) = hh;
            *(uint32_t *)(qvl + i * QP8 + k) = ll;
        }
    }
    __syncthreads();
    // ldmatrix row addresses of a query (or probability) plane pair: matrix lane / 8 = (hi, cols
    // 0-7), (hi, 8-15), (lo, 0-7), (lo, 8-15) of the k-step, row lane % 8
    const int mi = lane >> 3, mr = lane & 7;
    auto issue_v = [&]() {  // warps 4-7: the window's V rows, after their first position tile's loads
        for (int e = tid - 128; e < L * 32; e += 128) {
            const int r = e >> 5, c4 = 4 * (e & 31);
            cp_async16(Vs + r * VP + c4, Vb + (int64_t)r * ldk + c4);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // position scores (q + v) . P[prow0 + r], r < NP, of row tile m (rows 16 m .. + 15), the
    // tile's P rows read from L2 all at once
    const uint32_t qva = sm100::smem_u32((mi < 2 ? qvh : qvl) + mr * QP8 + 8 * (mi & 1));
    auto pos_tile = [&](int m) {
        const int r0 = 16 * m + g, r1 = r0 + 8;
        const float *p0 = P + (int64_t)(prow0 + (r0 < NP ? r0 : 0)) * D + off + 4 * t;
        const float *p1 = P + (int64_t)(prow0 + (r1 < NP ? r1 : 0)) * D + off + 4 * t;
        float4 x0[8], x1[8];
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // the tile's rows in flight at once
            x0[ks] = r0 < NP ? *(const float4 *)(p0 + 16 * ks) : make_float4(0.f, 0.f, 0.f, 0.f);
            x1[ks] = r1 < NP ? *(const float4 *)(p1 + 16 * ks) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (warp >= 4 && m == warp - 4) issue_v();
        float acc[2][3][4] = {};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t ah[4], al[4], b[4];
            a_split(x0[ks], x1[ks], ah, al);
            ldsm4(qva + 32 * ks, b);
            const uint32_t bh[2] = {b[0], b[1]}, bl[2] = {b[2], b[3]};
            mma3(acc[ks & 1], ah, al, bh, bl);
        }
        float d0[4], d1[4];
        acc_sum(acc[0], d0);
        acc_sum(acc[1], d1);
        const int i0 = 2 * t;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = r0 + 8 * (e >> 1), i = i0 + (e & 1);
            if (i < c && r < NP) gp[i * gpl + r] = d0[e] + d1[e];
        }
    };
    if (warp < 4) {
        // position row tiles 4 + warp, 8 + warp, ... while this warp's K rows are in flight, then the
        // content scores (q + u) . k from the shared K rows: key tiles warp, warp + 4, ...
        for (int m = 4 + warp; 16 * m < NP; m += 4) pos_tile(m);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        sm100::named_barrier(1, 128);
        const uint32_t qa = sm100::smem_u32((mi < 2 ? quh : qul) + mr * QP8 + 8 * (mi & 1));
        for (int m = warp; 16 * m < L; m += 4) {
            float acc[2][3][4] = {};
            const float *k0 = Ks + (16 * m + g) * KP + 4 * t, *k1 = k0 + 8 * KP;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                uint32_t ah[4], al[4], b[4];
                a_split(*(const float4 *)(k0 + 16 * ks), *(const float4 *)(k1 + 16 * ks), ah, al);
                ldsm4(qa + 32 * ks, b);
                const uint32_t bh[2] = {b[0], b[1]}, bl[2] = {b[2], b[3]};
                mma3(acc[ks & 1], ah, al, bh, bl);
            }
            float d0[4], d1[4];
            acc_sum(acc[0], d0);
            acc_sum(acc[1], d1);
            const int j0 = 16 * m + g, i0 = 2 * t;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = j0 + 8 * (e >> 1), i = i0 + (e & 1);
                if (i < c && j < L) sk[i * Lmax + j] = d0[e] + d1[e];
            }
        }
    } else {
        if (16 * (warp - 4) < NP) pos_tile(warp - 4);  // position row tiles 0-3
        else issue_v();
        asm volatile("cp.async.wait_group 0;" ::: "memory");  // this warp's V copies
    }
    __syncthreads();
    // softmax of query row `warp` (rows >= c: zero probabilities), written as bf16 hi / lo planes
    // over keys 0 .. Lr - 1 (zero from L on)
    {
        const int i = warp;
        float sv[3], mx = -INFINITY, sum = 0.0f;
        if (i < c) {
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const int j = lane + 32 * q;
                sv[q] = j < L ? (sk[i * Lmax + j] + gp[i * gpl + c - 1 - i + j]) * scale : -INFINITY;
                mx = fmaxf(mx, sv[q]);
            }
            mx = nb::warp_max(mx);
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const int j = lane + 32 * q;
                sv[q] = j < L ? expf(sv[q] - mx) : 0.0f;
                sum += sv[q];
            }
            sum = 1.0f / nb::warp_sum(sum);
        }
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int j = lane + 32 * q;
            if (j < Lr) {
                const float pv = (i < c && j < L) ? sv[q] * sum : 0.0f;
                const __nv_bfloat16 hb = __float2bfloat16_rn(pv);
                const __nv_bfloat16 lb = __float2bfloat16_rn(pv - __bfloat162float(hb));
                pph[i * PP + j] = *(const uint16_t *)&hb;
                ppl[i * PP + j] = *(const uint16_t *)&lb;
            }
        }
    }
    __syncthreads();
    // o^T = V^T . P^T: warp w owns head dims [16 w, 16 w + 16) (the 16-row side); k runs over the
    // keys 0 .. Lr - 1
    {
        float acc[2][3][4] = {};
        const uint32_t pa = sm100::smem_u32((mi < 2 ? pph : ppl) + mr * PP + 8 * (mi & 1));
        const float *vc = Vs + 2 * t * VP + 16 * warp + g;
        for (int ks0 = 0; 16 * ks0 < Lr; ks0 += 2)
#pragma unroll
            for (int par = 0; par < 2; ++par) {
                const int k0 = 16 * (ks0 + par);
                if (k0 >= Lr) break;
                const float *v = vc + k0 * VP;
                uint32_t ah[4], al[4], b[4];
                split2(v[0], v[VP], ah[0], al[0]);                 // dim g, keys 2t, 2t + 1
                split2(v[8], v[VP + 8], ah[1], al[1]);             // dim g + 8
                split2(v[8 * VP], v[9 * VP], ah[2], al[2]);        // dim g, keys 2t + 8, 2t + 9
                split2(v[8 * VP + 8], v[9 * VP + 8], ah[3], al[3]);
                ldsm4(pa + 2 * k0, b);
                const uint32_t bh[2] = {b[0], b[1]}, bl[2] = {b[2], b[3]};
                mma3(acc[par], ah, al, bh, bl);
            }
        float o0[4], o1[4];
        acc_sum(acc[0], o0);
        acc_sum(acc[1], o1);
        // lane element e: head dim 16 w + g + 8 (e >> 1), query row 2 t + (e & 1)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i = 2 * t + (e & 1), col = off + 16 * warp + g + 8 * (e >> 1);
            if (i < c) nb::store_act(O, o_fmt, o_plane, (int64_t)s * o_sstride + (int64_t)i * D + col, o0[e] + o1[e]);
        }
    }
}

}  // namespace

extern "C" int nemo_attention_rel(const float *Q, int64_t ldq, int64_t q_sstride, const float *K, const float *V, int64_t ldk, int64_t kv_sstride,
                                  const int *pos, const int *cache_len, const float *P, const float *bias_u, const float *bias_v, void *O,
                                  int o_fmt, int64_t o_plane, int64_t o_sstride, int streams, int c, int Lmax, int H, int dh, int D, float scale,
                                  void *stream) {
    if (dh != DH) return nb_set_error("nemo_attention_rel: head dim must be 128");
    if (c <= 0 || streams <= 0) return 0;
    if (c > MAXC || Lmax > MAXL) return nb_set_error("nemo_attention_rel: chunk of %d rows / window %d too large", c, Lmax);
    if (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)P | (uintptr_t)bias_u | (uintptr_t)bias_v) & 15 || (ldq | ldk | D | kv_sstride | q_sstride) & 3)
        return nb_set_error("nemo_attention_rel: rows must be 16-byte aligned");
    if (c <= 8) {
        const size_t smem = (size_t)smem8_floats(Lmax) * sizeof(float);
        if (nb_smem_attr((const void *)attention8_kernel, smem)) return nb_set_error("nemo_attention_rel: %s", nemo_gpu_last_error());
        nb::launch(attention8_kernel, dim3(H, streams), THREADS, smem, (cudaStream_t)stream, Q, ldq, q_sstride, K, V, ldk, kv_sstride, pos, cache_len, P, bias_u,
                   bias_v, O, o_fmt, o_plane, o_sstride, c, Lmax, D, scale);
        return nb_check_launch("attention8_kernel");
    }
    const size_t smem = (size_t)smem_floats(Lmax) * sizeof(float);
    if (nb_smem_attr((const void *)attention_kernel, smem)) return nb_set_error("nemo_attention_rel: %s", nemo_gpu_last_error());
    nb::launch(attention_kernel, dim3(H, streams), THREADS, smem, (cudaStream_t)stream, Q, ldq, q_sstride, K, V, ldk, kv_sstride, pos, cache_len, P, bias_u, bias_v,
                                                                           O, o_fmt, o_plane, o_sstride, c, Lmax, D, scale);
    return nb_check_launch("attention_kernel");
}

// Nonzero (and cleared) once an attention CTA gave up waiting for its rows.
extern "C" int nb_attention_device_error(void) {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_att_error, sizeof v) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_att_error, &z, sizeof z);
    return v;
}
