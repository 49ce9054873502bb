// Relative-position self-attention of one chunk over the per-stream K/V cache window
// (src/kernels.metal:293-348, dispatched at src/encoder.c:161-165):
//   s[i][j] = ((q_i + u) . k_j + (q_i + v) . P[(Lmax - L) + (c - 1 - i + j)]) * scale
//   softmax over all L keys (no mask inside the window), o_i = sum_j p[i][j] v_j.
// The position term only depends on c - 1 - i + j, so G[i][r] = (q_i + v) . P[r0 + r] is
// computed once per position row r (L + c - 1 rows) and read back diagonally.
//
// One CTA (8 warps) per (head, stream). The stream's K and V rows of the head (the HBM traffic
// of the kernel) are copied into shared memory with cp.async as the CTA starts, K and V in two
// groups, while the position scores are formed from P (shared by all streams, L2-resident); the
// content scores then read K and the value pass V from shared memory. Warps take rows
// round-robin; a lane holds 4 of the 128 head dims, so a row is one 512-byte access.
#include "common.cuh"

namespace {

constexpr int DH = 128;
constexpr int THREADS = 256;
constexpr int MAXC = 16;   // rows per chunk
constexpr int MAXL = 96;   // keys in the window

__device__ __forceinline__ float dot4(const float4 a, const float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Shared-memory floats of one CTA: K and V rows [Lmax][DH] each, (q + u) and (q + v) [c][DH],
// content scores / probabilities [c][Lmax], position scores [c][Lmax + c].
__host__ __device__ __forceinline__ int smem_floats(int c, int Lmax) { return 2 * Lmax * DH + 2 * c * DH + c * Lmax + c * (Lmax + c); }

// out[i * out_ld + r] = qx[i] . row r for rows r < rows (row r at base + r * ld). A warp takes
// R = 32 / Q rows at a time and forms the R x Q partial dot products of its lanes' 4 dims; one
// halving butterfly (31 shuffles for 32 values instead of 5 per value) leaves lane l with the
// total of value l = (row l / Q, query l % Q).
template <int Q>
__device__ __forceinline__ void score_rows(const float *base, int64_t ld, int rows, int c, const float *qx, float *out, int out_ld, int warp,
                                           int lane) {
    constexpr int R = 32 / Q;
    for (int r0 = warp * R; r0 < rows; r0 += (THREADS / 32) * R) {
        float4 x[R];
#pragma unroll
        for (int k = 0; k < R; ++k)
            x[k] = r0 + k < rows ? *(const float4 *)(base + (int64_t)(r0 + k) * ld + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
        float a[32];
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int i = 0; i < Q; ++i) a[k * Q + i] = i < c ? dot4(x[k], *(const float4 *)(qx + i * DH + 4 * lane)) : 0.0f;
#pragma unroll
        for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
            const bool up = lane & o;
#pragma unroll
            for (int k = 0; k < n / 2; ++k) {
                const float send = up ? a[k] : a[k + n / 2];
                const float keep = up ? a[k + n / 2] : a[k];
                a[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const int i = lane % Q, r = r0 + lane / Q;
        if (i < c && r < rows) out[i * out_ld + r] = a[0];
    }
}

__global__ void __launch_bounds__(THREADS) attention_kernel(const float *__restrict__ Q, int64_t ldq, int64_t q_sstride, const float *__restrict__ K,
                                                            const float *__restrict__ V, int64_t ldk, int64_t kv_sstride, const int *pos_p,
                                                            const int *cache_len_p, const float *__restrict__ P, const float *__restrict__ bias_u,
                                                            const float *__restrict__ bias_v, void *O, int o_fmt, int64_t o_plane, int64_t o_sstride,
                                                            int c, int Lmax, int D, float scale) {
    extern __shared__ __align__(16) float sm[];
    float *Ks = sm, *Vs = sm + Lmax * DH, *qu = sm + 2 * Lmax * DH, *qv = qu + c * DH, *sk = qv + c * DH, *gp = sk + c * Lmax;
    nb::pdl_wait();
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pos = *pos_p, cache_len = *cache_len_p, L = cache_len + c;
    if (L > MAXL || L > Lmax || c > MAXC || pos - cache_len < 0) return; // the host keeps these in range
    const int NP = L + c - 1, prow0 = Lmax - L, off = h * DH;
    const float *Kb = K + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    const float *Vb = V + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    // the window's K rows, then its V rows, into shared memory (16 bytes per copy)
    for (int e = tid; e < L * (DH / 4); e += THREADS) {
        const int r = e >> 5, q4 = (e & 31) * 4;
        cp_async16(Ks + r * DH + q4, Kb + (int64_t)r * ldk + q4);
    }
    cp_async_commit();
    for (int e = tid; e < L * (DH / 4); e += THREADS) {
        const int r = e >> 5, q4 = (e & 31) * 4;
        cp_async16(Vs + r * DH + q4, Vb + (int64_t)r * ldk + q4);
    }
    cp_async_commit();
    const float *Qb = Q + (int64_t)s * q_sstride + (int64_t)pos * ldq + off;
    for (int e = tid; e < c * DH; e += THREADS) {
        const int i = e / DH, d = e - i * DH;
        const float q = Qb[(int64_t)i * ldq + d];
        qu[i * DH + d] = q + bias_u[off + d];
        qv[i * DH + d] = q + bias_v[off + d];
    }
    __syncthreads();
    // position scores from P while K and V arrive, then the content scores from shared K
    const float *Pb = P + (int64_t)prow0 * D + off;
    if (c <= 8) score_rows<8>(Pb, D, NP, c, qv, gp, Lmax + c, warp, lane);
    else score_rows<16>(Pb, D, NP, c, qv, gp, Lmax + c, warp, lane);
    cp_async_wait<1>();
    __syncthreads();
    if (c <= 8) score_rows<8>(Ks, DH, L, c, qu, sk, Lmax, warp, lane);
    else score_rows<16>(Ks, DH, L, c, qu, sk, Lmax, warp, lane);
    __syncthreads();
    // softmax of each query row (one warp per row)
    for (int i = warp; i < c; i += THREADS / 32) {
        float sv[3], mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const int j = lane + 32 * t;
            sv[t] = j < L ? (sk[i * Lmax + j] + gp[i * (Lmax + c) + c - 1 - i + j]) * scale : -INFINITY;
            mx = fmaxf(mx, sv[t]);
        }
        mx = nb::warp_max(mx);
        float sum = 0.0f;
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const int j = lane + 32 * t;
            sv[t] = j < L ? expf(sv[t] - mx) : 0.0f;
            sum += sv[t];
        }
        sum = nb::warp_sum(sum);
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const int j = lane + 32 * t;
            if (j < L) sk[i * Lmax + j] = sv[t] / sum;
        }
    }
    cp_async_wait<0>();
    __syncthreads();
    // o[i][d] = sum_j p[i][j] v[j][d]: thread (d, half) accumulates every other query row
    const int d = tid & (DH - 1), hrow = tid >> 7;
    float acc[MAXC / 2];
#pragma unroll
    for (int k = 0; k < MAXC / 2; ++k) acc[k] = 0.0f;
    for (int j = 0; j < L; ++j) {
        const float vj = Vs[j * DH + d];
#pragma unroll
        for (int k = 0; k < MAXC / 2; ++k) {
            const int i = hrow + 2 * k;
            if (i < c) acc[k] += sk[i * Lmax + j] * vj;
        }
    }
#pragma unroll
    for (int k = 0; k < MAXC / 2; ++k) {
        const int i = hrow + 2 * k;
        if (i < c) nb::store_act(O, o_fmt, o_plane, (int64_t)s * o_sstride + (int64_t)i * D + off + d, acc[k]);
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
    if (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)P) & 15 || (ldq | ldk | D | kv_sstride) & 3)
        return nb_set_error("nemo_attention_rel: rows must be 16-byte aligned");
    const size_t smem = (size_t)smem_floats(c, Lmax) * sizeof(float);
    static size_t attr_set = 0;  // largest dynamic shared-memory size enabled so far
    if (smem > attr_set) {
        if (cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return nb_set_error("nemo_attention_rel: %zu bytes of shared memory unavailable", smem);
        attr_set = smem;
    }
    nb::launch(attention_kernel, dim3(H, streams), THREADS, smem, (cudaStream_t)stream, Q, ldq, q_sstride, K, V, ldk, kv_sstride, pos, cache_len, P, bias_u, bias_v,
                                                                           O, o_fmt, o_plane, o_sstride, c, Lmax, D, scale);
    return nb_check_launch("attention_kernel");
}
