// Relative-position self-attention of one chunk over the per-stream K/V cache window
// (src/kernels.metal:293-348, dispatched at src/encoder.c:161-165):
//   s[i][j] = ((q_i + u) . k_j + (q_i + v) . P[(Lmax - L) + (c - 1 - i + j)]) * scale
//   softmax over all L keys (no mask inside the window), o_i = sum_j p[i][j] v_j.
// The position term only depends on c - 1 - i + j, so G[i][r] = (q_i + v) . P[r0 + r] is
// computed once per position row r (L + c - 1 rows) and read back diagonally.
//
// One CTA (8 warps) per (head, stream). Warps take keys (and position rows) round-robin; a lane
// holds 4 of the 128 head dims, so each key row is one coalesced 512-byte read; the c dot
// products per row are reduced across lanes. Scores and probabilities stay in shared memory;
// the value pass reads each v_j once and accumulates all queries of the chunk.
#include "common.cuh"

namespace {

constexpr int DH = 128;
constexpr int THREADS = 256;
constexpr int MAXC = 16;   // rows per chunk
constexpr int MAXL = 96;   // keys in the window

__device__ __forceinline__ float dot4(const float4 a, const float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

__global__ void __launch_bounds__(THREADS) attention_kernel(const float *__restrict__ Q, int64_t ldq, int64_t q_sstride, const float *__restrict__ K,
                                                            const float *__restrict__ V, int64_t ldk, int64_t kv_sstride, const int *pos_p,
                                                            const int *cache_len_p, const float *__restrict__ P, const float *__restrict__ bias_u,
                                                            const float *__restrict__ bias_v, void *O, int o_fmt, int64_t o_plane, int64_t o_sstride,
                                                            int c, int Lmax, int D, float scale) {
    __shared__ __align__(16) float qu[MAXC][DH], qv[MAXC][DH];
    __shared__ float sk[MAXC][MAXL];          // content scores, then probabilities
    __shared__ float gp[MAXC][MAXL + MAXC];   // position scores per position row
    nb::pdl_wait();
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pos = *pos_p, cache_len = *cache_len_p, L = cache_len + c;
    if (L > MAXL || L > Lmax || c > MAXC || pos - cache_len < 0) return; // the host keeps these in range
    const int NP = L + c - 1, prow0 = Lmax - L, off = h * DH;
    const float *Qb = Q + (int64_t)s * q_sstride + (int64_t)pos * ldq + off;
    for (int e = tid; e < c * DH; e += THREADS) {
        const int i = e / DH, d = e - i * DH;
        const float q = Qb[(int64_t)i * ldq + d];
        qu[i][d] = q + bias_u[off + d];
        qv[i][d] = q + bias_v[off + d];
    }
    __syncthreads();
    const float *Kb = K + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    const float *Vb = V + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    const float *Pb = P + (int64_t)prow0 * D + off;
    // content scores (rows 0..L-1) and position scores (rows L..L+NP-1), one row per warp step
    for (int r = warp; r < L + NP; r += THREADS / 32) {
        const bool is_k = r < L;
        const float4 x = is_k ? *(const float4 *)(Kb + (int64_t)r * ldk + 4 * lane) : *(const float4 *)(Pb + (int64_t)(r - L) * D + 4 * lane);
        float part[MAXC];
#pragma unroll
        for (int i = 0; i < MAXC; ++i)
            if (i < c) part[i] = dot4(x, *(const float4 *)((is_k ? qu[i] : qv[i]) + 4 * lane));
#pragma unroll
        for (int i = 0; i < MAXC; ++i)
            if (i < c) {
                const float v = nb::warp_sum(part[i]);
                if (lane == 0) {
                    if (is_k) sk[i][r] = v;
                    else gp[i][r - L] = v;
                }
            }
    }
    __syncthreads();
    // softmax of each query row (one warp per row)
    for (int i = warp; i < c; i += THREADS / 32) {
        float sv[3], mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const int j = lane + 32 * t;
            sv[t] = j < L ? (sk[i][j] + gp[i][c - 1 - i + j]) * scale : -INFINITY;
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
            if (j < L) sk[i][j] = sv[t] / sum;
        }
    }
    __syncthreads();
    // o[i][d] = sum_j p[i][j] v[j][d]: thread (d, half) accumulates every other query row
    const int d = tid & (DH - 1), hrow = tid >> 7;
    float acc[MAXC / 2];
#pragma unroll
    for (int k = 0; k < MAXC / 2; ++k) acc[k] = 0.0f;
    for (int j = 0; j < L; ++j) {
        const float vj = Vb[(int64_t)j * ldk + d];
#pragma unroll
        for (int k = 0; k < MAXC / 2; ++k) {
            const int i = hrow + 2 * k;
            if (i < c) acc[k] += sk[i][j] * vj;
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
    if (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)P) & 15 || (ldq | ldk | D) & 3)
        return nb_set_error("nemo_attention_rel: rows must be 16-byte aligned");
    attention_kernel<<<dim3(H, streams), THREADS, 0, (cudaStream_t)stream>>>(Q, ldq, q_sstride, K, V, ldk, kv_sstride, pos, cache_len, P, bias_u, bias_v,
                                                                           O, o_fmt, o_plane, o_sstride, c, Lmax, D, scale);
    return nb_check_launch("attention_kernel");
}
