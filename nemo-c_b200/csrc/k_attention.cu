// Relative-position self-attention of one chunk over the per-stream K/V cache window
// (src/kernels.metal:293-348, dispatched at src/encoder.c:161-165):
//   s[i][j] = ((q_i + u) . k_j + (q_i + v) . P[(Lmax - L) + (c - 1 - i + j)]) * scale
//   softmax over all L keys (no mask inside the window), o_i = sum_j p[i][j] v_j.
// The position term only depends on c - 1 - i + j, so G[i][r] = (q_i + v) . P[r0 + r] is
// computed once per position row r (L + c - 1 rows) and read back diagonally.
//
// One CTA (8 warps) per (head, stream). The stream's V rows of the head (half of the HBM traffic
// of the kernel) are requested as the CTA starts, 16-byte asynchronous copies into shared memory
// spread over all threads (no registers held, so three CTAs fit an SM); the K rows are read
// straight into the score tiles' fragments by warps 0-3 (each 32-byte sector read whole, by one
// thread group) while warps 4-7 form the position scores. Issuing one bulk copy per 512-byte row
// instead cost more than the transfer itself. The three products (content
// and position scores, probabilities times V) run on the
// tensor cores as mma.sync m16n8k16 tiles (the chunk's <= 16 query rows are the M side) with
// both operands split into bf16 hi + lo parts and three products per tile (hi.hi, hi.lo, lo.hi;
// the dropped lo.lo term is below 2^-16 of each product), accumulating in fp32. The softmax stays
// in fp32 with IEEE expf.
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

// Scores of 8 rows (one n-tile) against the 16 query rows: rows r0 + g of `src` (pitch `pitch`,
// rows >= nrows read as zero), 128 dims; result d[] in C-fragment layout.
__device__ __forceinline__ void score_tile(const uint16_t *qhi, const uint16_t *qlo, const float *src, int64_t pitch, int r0, int nrows, int lane,
                                           float (&d)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const bool ok = r0 + g < nrows;
    const float *row = src + (int64_t)(ok ? r0 + g : 0) * pitch + 2 * t;
    float2 b[16];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {  // every load of the tile before the first product
        b[2 * ks] = ok ? *(const float2 *)(row + 16 * ks) : make_float2(0.f, 0.f);
        b[2 * ks + 1] = ok ? *(const float2 *)(row + 16 * ks + 8) : make_float2(0.f, 0.f);
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
        const int e = tid + r * THREADS, i = e >> 6, k = 2 * (e & 63);
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
    // the two score products side by side: warps 0-3 the content scores (q + u) . k from the K
    // rows, read straight from global memory (their HBM latency passes while warps 4-7 form the
    // position scores (q + v) . P from the L2-resident table)
    const float *Pb = P + (int64_t)prow0 * D + off;
    const int ntP = (NP + 7) >> 3, ntK = (L + 7) >> 3;
    if (warp < 4) {
        for (int nt = warp; nt < ntK; nt += 4) {
            float d[4];
            score_tile(quh, qul, Kb, ldk, nt * 8, L, lane, d);
            const int col = nt * 8 + 2 * t;
            if (g < c) { if (col < L) sk[g * Lmax + col] = d[0]; if (col + 1 < L) sk[g * Lmax + col + 1] = d[1]; }
            if (g + 8 < c) { if (col < L) sk[(g + 8) * Lmax + col] = d[2]; if (col + 1 < L) sk[(g + 8) * Lmax + col + 1] = d[3]; }
        }
    } else {
        for (int nt = warp - 4; nt < ntP; nt += 4) {
            float d[4];
            score_tile(qvh, qvl, Pb, D, nt * 8, NP, lane, d);
            const int col = nt * 8 + 2 * t;
            if (g < c) { if (col < NP) gp[g * gpl + col] = d[0]; if (col + 1 < NP) gp[g * gpl + col + 1] = d[1]; }
            if (g + 8 < c) { if (col < NP) gp[(g + 8) * gpl + col] = d[2]; if (col + 1 < NP) gp[(g + 8) * gpl + col + 1] = d[3]; }
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

}  // namespace

extern "C" int nemo_attention_rel(const float *Q, int64_t ldq, int64_t q_sstride, const float *K, const float *V, int64_t ldk, int64_t kv_sstride,
                                  const int *pos, const int *cache_len, const float *P, const float *bias_u, const float *bias_v, void *O,
                                  int o_fmt, int64_t o_plane, int64_t o_sstride, int streams, int c, int Lmax, int H, int dh, int D, float scale,
                                  void *stream) {
    if (dh != DH) return nb_set_error("nemo_attention_rel: head dim must be 128");
    if (c <= 0 || streams <= 0) return 0;
    if (c > MAXC || Lmax > MAXL) return nb_set_error("nemo_attention_rel: chunk of %d rows / window %d too large", c, Lmax);
    if (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)P) & 15 || (ldq | ldk | D | kv_sstride | q_sstride) & 3)
        return nb_set_error("nemo_attention_rel: rows must be 16-byte aligned");
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
