// Relative-position attention over the K/V cache, and the RNNT decoder kernels (LSTM cell,
// joint + argmax, greedy-loop bookkeeping).
#include "common.cuh"

namespace {

constexpr int ATT_MAX_L = 96;   // cache (<= att_left) + chunk rows; checked on the host
constexpr int ATT_DH = 128;

// src/kernels.metal:293-348. One block per (head, stream), 128 threads (= dh); the K/V window and
// the position rows the chunk touches are staged in shared memory once, then each query of the
// chunk is processed: s_j = ((q+u).k_j + (q+v).P[prow]) * scale, prow = (Lmax-L) + (c-1-i+j),
// softmax over all L keys, O = sum_j p_j V_j.
__global__ void __launch_bounds__(ATT_DH) attention_rel_kernel(const float *__restrict__ Q, int64_t ldq, int64_t q_sstride,
                                                               const float *__restrict__ K, const float *__restrict__ V, int64_t ldk,
                                                               int64_t kv_sstride, const int *pos_p, const int *cache_len_p,
                                                               const float *__restrict__ P, const float *__restrict__ bias_u,
                                                               const float *__restrict__ bias_v, void *O, int o_fmt, int64_t o_plane,
                                                               int64_t o_sstride, int c, int Lmax, int D, float scale) {
    extern __shared__ float sm[];
    nb::pdl_wait();
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pos = *pos_p, cache_len = *cache_len_p, L = cache_len + c;
    if (L > ATT_MAX_L || L > Lmax || pos - cache_len < 0) return; /* the host bookkeeping keeps L in range */
    const int NP = L + c - 1, prow0 = Lmax - L;
    float *Ks = sm;                       // [L][129]
    float *Vs = Ks + ATT_MAX_L * 129;     // [L][128]
    float *Ps = Vs + ATT_MAX_L * 128;     // [NP][129]
    float *qu = Ps + (ATT_MAX_L + 16) * 129;
    float *qv = qu + ATT_DH;
    float *sc = qv + ATT_DH;              // [L]
    float *red = sc + ATT_MAX_L;          // [8]
    const int off = h * ATT_DH;
    const float *Kb = K + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    const float *Vb = V + (int64_t)s * kv_sstride + (int64_t)(pos - cache_len) * ldk + off;
    for (int j = 0; j < L; ++j) {
        Ks[j * 129 + tid] = Kb[(int64_t)j * ldk + tid];
        Vs[j * 128 + tid] = Vb[(int64_t)j * ldk + tid];
    }
    for (int r = 0; r < NP; ++r) Ps[r * 129 + tid] = P[(int64_t)(prow0 + r) * D + off + tid];
    const float bu = bias_u[off + tid], bv = bias_v[off + tid];
    const float *Qb = Q + (int64_t)s * q_sstride + (int64_t)pos * ldq + off;
    for (int i = 0; i < c; ++i) {
        __syncthreads();
        const float q = Qb[(int64_t)i * ldq + tid];
        qu[tid] = q + bu;
        qv[tid] = q + bv;
        __syncthreads();
        // scores: thread j (< L) owns key j; padded rows make the strided reads conflict-free
        for (int j = tid; j < L; j += ATT_DH) {
            const float *kr = Ks + j * 129;
            const float *pr = Ps + (c - 1 - i + j) * 129;
            float a = 0.0f, b = 0.0f;
#pragma unroll 8
            for (int d = 0; d < ATT_DH; ++d) { a += qu[d] * kr[d]; b += qv[d] * pr[d]; }
            sc[j] = (a + b) * scale;
        }
        __syncthreads();
        // softmax over L <= 96 scores
        float mx = -INFINITY;
        for (int j = tid; j < L; j += ATT_DH) mx = fmaxf(mx, sc[j]);
        mx = nb::warp_max(mx);
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        __syncthreads();
        float sum = 0.0f;
        for (int j = tid; j < L; j += ATT_DH) { const float e = expf(sc[j] - mx); sc[j] = e; sum += e; }
        sum = nb::warp_sum(sum);
        if (lane == 0) red[4 + warp] = sum;
        __syncthreads();
        sum = (red[4] + red[5]) + (red[6] + red[7]);
        float acc = 0.0f;
        for (int j = 0; j < L; ++j) acc += (sc[j] / sum) * Vs[j * 128 + tid];
        nb::store_act(O, o_fmt, o_plane, (int64_t)s * o_sstride + (int64_t)i * D + off + tid, acc);
    }
}

// src/kernels.metal:475-486 on `rows` gate vectors.
__global__ void lstm_cell_kernel(const float *__restrict__ gates, const float *__restrict__ c_in, float *c_out, float *h_out, int rows, int H) {
    nb::pdl_wait();
    const int64_t total = (int64_t)rows * H;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / H;
        const int j = (int)(i - r * H);
        const float *g = gates + r * 4 * H;
        const float ig = nb::sigmoid_f(g[j]), fg = nb::sigmoid_f(g[H + j]), gg = tanhf(g[2 * H + j]), og = nb::sigmoid_f(g[3 * H + j]);
        const float cc = fg * c_in[i] + ig * gg;
        c_out[i] = cc;
        h_out[i] = og * tanhf(cc);
    }
}

// src/kernels.metal:490-550: logits = W . relu(enc + pred) + b, argmax with ties -> lowest index.
// One block (256 threads) per row; warps take vocabulary rows round-robin, lanes split H.
// Rows may be listed (rowlist: the row to evaluate for each block, -1 = skip).
__global__ void __launch_bounds__(256) joint_argmax_kernel(const float *__restrict__ enc, int64_t enc_ld, const float *__restrict__ pred,
                                                           int64_t pred_ld, int pred_rpg, const uint16_t *__restrict__ W,
                                                           const float *__restrict__ bias, int V, int H, const int *enc_row_of,
                                                           int *out_idx, float *out_val) {
    __shared__ __align__(16) float x[1024];
    __shared__ float bvs[8];
    __shared__ int bis[8];
    nb::pdl_wait();
    const int r = blockIdx.x;
    const int er = enc_row_of ? enc_row_of[r] : r;
    if (er < 0) return;
    const float *e = enc + (int64_t)er * enc_ld;
    const float *p = pred + (int64_t)(r / pred_rpg) * pred_ld;
    for (int i = threadIdx.x; i < H; i += 256) x[i] = fmaxf(e[i] + p[i], 0.0f);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const int H4 = H >> 2;
    for (int n = warp; n < V; n += 8) {
        const uint2 *w = (const uint2 *)(W + (int64_t)n * H);
        float acc = 0.0f;
        for (int k = lane; k < H4; k += 32) {
            const uint2 q = __ldg(w + k);
            const float4 xx = *(const float4 *)(x + 4 * k);
            acc += xx.x * nb::bf16lo(q.x) + xx.y * nb::bf16hi(q.x) + xx.z * nb::bf16lo(q.y) + xx.w * nb::bf16hi(q.y);
        }
        acc = nb::warp_sum(acc) + bias[n];
        if (acc > bv) { bv = acc; bi = n; }  // n increases per warp: strict > keeps the lowest index
    }
    if (lane == 0) { bvs[warp] = bv; bis[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = bvs[0];
        int ix = bis[0];
        for (int w = 1; w < 8; ++w)
            if (bvs[w] > v || (bvs[w] == v && bis[w] < ix)) { v = bvs[w]; ix = bis[w]; }
        out_idx[r] = ix;
        if (out_val) out_val[r] = v;
    }
}

}  // namespace

extern "C" int nemo_attention_rel(const float *Q, int64_t ldq, int64_t q_sstride, const float *K, const float *V, int64_t ldk, int64_t kv_sstride,
                                  const int *pos, const int *cache_len, const float *P, const float *bias_u, const float *bias_v, void *O,
                                  int o_fmt, int64_t o_plane, int64_t o_sstride, int streams, int c, int Lmax, int H, int dh, int D, float scale,
                                  void *stream) {
    if (dh != ATT_DH) return nb_set_error("nemo_attention_rel: head dim must be 128");
    if (c <= 0 || streams <= 0) return 0;
    if (c > 16 || Lmax + c > ATT_MAX_L + 16) return nb_set_error("nemo_attention_rel: chunk of %d rows / Lmax %d too large", c, Lmax);
    const size_t smem = (size_t)(ATT_MAX_L * 129 + ATT_MAX_L * 128 + (ATT_MAX_L + 16) * 129 + 2 * ATT_DH + ATT_MAX_L + 8) * sizeof(float);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attention_rel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = true;
    }
    attention_rel_kernel<<<dim3(H, streams), ATT_DH, smem, (cudaStream_t)stream>>>(Q, ldq, q_sstride, K, V, ldk, kv_sstride, pos, cache_len, P, bias_u,
                                                                                   bias_v, O, o_fmt, o_plane, o_sstride, c, Lmax, D, scale);
    return nb_check_launch("attention_rel_kernel");
}

extern "C" int nemo_lstm_cell(const float *gates, const float *c_in, float *c_out, float *h_out, int rows, int H, void *stream) {
    const int64_t total = (int64_t)rows * H;
    if (total <= 0) return 0;
    const int grid = (int)((total + 255) / 256 < 1184 ? (total + 255) / 256 : 1184);
    lstm_cell_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(gates, c_in, c_out, h_out, rows, H);
    return nb_check_launch("lstm_cell_kernel");
}

extern "C" int nb_joint_argmax_rows(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, int pred_rpg, const uint16_t *W,
                                    const float *bias, int V, int H, int rows, const int *enc_row_of, int *out_idx, float *out_val, void *stream) {
    if (H > 1024 || (H & 3)) return nb_set_error("nemo_joint_argmax: H must be a multiple of 4 and <= 1024");
    if (rows <= 0) return 0;
    joint_argmax_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(enc, enc_ld, pred, pred_ld, pred_rpg > 0 ? pred_rpg : 1, W, bias, V, H, enc_row_of,
                                                               out_idx, out_val);
    return nb_check_launch("joint_argmax_kernel");
}

extern "C" int nemo_joint_argmax(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, const uint16_t *W, const float *bias, int V,
                                 int H, int rows, int *out_idx, float *out_val, void *stream) {
    return nb_joint_argmax_rows(enc, enc_ld, pred, pred_ld, 1, W, bias, V, H, rows, nullptr, out_idx, out_val, stream);
}
