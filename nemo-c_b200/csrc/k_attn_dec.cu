// RNNT decoder kernels: LSTM cell, joint + argmax.
//
// The joint (src/kernels.metal:490-550: logits = W . relu(enc + pred) + b, argmax with ties to
// the lowest index) runs as: relu(enc + pred) written as bf16 hi/lo planes, the tensor-core GEMM
// for W . x + b into fp32 logits, then one warp per row for the argmax. A direct CUDA-core
// version (one block per row) serves single rows through the C-ABI.
#include "common.cuh"

namespace {

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

// Direct joint + argmax, one block (256 threads) per row: warps take vocabulary rows round-robin,
// lanes split H. enc_row_of (optional) maps block -> encoder row (-1 = skip).
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

// GEMM input of the joint: x[r] = relu(enc[enc_row_of[r]] + pred[r]) as bf16 hi/lo planes
// (rows with enc_row_of < 0 are written as zeros). One block per row.
__global__ void joint_input_kernel(const float *__restrict__ enc, int64_t enc_ld, const float *__restrict__ pred, int64_t pred_ld,
                                   const int *enc_row_of, uint16_t *X, int64_t plane, int H) {
    nb::pdl_wait();
    const int r = blockIdx.x;
    const int er = enc_row_of ? enc_row_of[r] : r;
    const float *e = enc + (int64_t)(er < 0 ? 0 : er) * enc_ld;
    const float *p = pred + (int64_t)r * pred_ld;
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        nb::store_act(X, NEMO_FMT_BF16X2, plane, (int64_t)r * H + i, er < 0 ? 0.0f : fmaxf(e[i] + p[i], 0.0f));
}

// Row argmax of fp32 logits [rows][ld] over V columns, ties -> lowest index; one warp per row.
__global__ void row_argmax_kernel(const float *__restrict__ logits, int64_t ld, int V, const int *enc_row_of, int rows, int *out_idx, float *out_val) {
    nb::pdl_wait();
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows || (enc_row_of && enc_row_of[r] < 0)) return;
    const float *l = logits + (int64_t)r * ld;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int n = lane; n < V; n += 32) {
        const float v = l[n];
        if (v > bv) { bv = v; bi = n; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
        out_idx[r] = bi;
        if (out_val) out_val[r] = bv;
    }
}

}  // namespace

extern "C" int nemo_lstm_cell(const float *gates, const float *c_in, float *c_out, float *h_out, int rows, int H, void *stream) {
    const int64_t total = (int64_t)rows * H;
    if (total <= 0) return 0;
    const int grid = (int)((total + 255) / 256 < 1184 ? (total + 255) / 256 : 1184);
    nb::launch(lstm_cell_kernel, grid, 256, 0, (cudaStream_t)stream, gates, c_in, c_out, h_out, rows, H);
    return nb_check_launch("lstm_cell_kernel");
}

extern "C" int nb_joint_argmax_rows(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, int pred_rpg, const uint16_t *W,
                                    const float *bias, int V, int H, int rows, const int *enc_row_of, int *out_idx, float *out_val, void *stream) {
    if (H > 1024 || (H & 3)) return nb_set_error("nemo_joint_argmax: H must be a multiple of 4 and <= 1024");
    if (rows <= 0) return 0;
    nb::launch(joint_argmax_kernel, rows, 256, 0, (cudaStream_t)stream, enc, enc_ld, pred, pred_ld, pred_rpg > 0 ? pred_rpg : 1, W, bias, V, H, enc_row_of,
                                                               out_idx, out_val);
    return nb_check_launch("joint_argmax_kernel");
}

extern "C" int nemo_joint_argmax(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, const uint16_t *W, const float *bias, int V,
                                 int H, int rows, int *out_idx, float *out_val, void *stream) {
    return nb_joint_argmax_rows(enc, enc_ld, pred, pred_ld, 1, W, bias, V, H, rows, nullptr, out_idx, out_val, stream);
}

/* Joint through the tensor-core GEMM: X [rows][H] planes (workspace, 4*rows*H bytes), logits
   [rows][ldl] fp32 (workspace). enc row of stream r = enc_row_of[r] (-1 = inactive). */
extern "C" int nb_joint_argmax_gemm(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, const uint16_t *W, const float *bias,
                                    int V, int H, int rows, const int *enc_row_of, uint16_t *X, float *logits, int64_t ldl, int *out_idx,
                                    float *out_val, void *stream) {
    if (rows <= 0) return 0;
    cudaStream_t st = (cudaStream_t)stream;
    nb::launch(joint_input_kernel, rows, 128, 0, st, enc, enc_ld, pred, pred_ld, enc_row_of, X, (int64_t)rows * H, H);
    if (nb_check_launch("joint_input_kernel")) return -1;
    nemo_gemm_args_t a = {};
    a.A = X; a.lda = H; a.a_fmt = NEMO_FMT_BF16X2; a.a_plane = (int64_t)rows * H;
    a.W = W; a.ldw = H; a.bias = bias;
    a.C = logits; a.ldc = ldl; a.c_fmt = NEMO_FMT_F32;
    a.M = rows; a.N = V; a.K = H; a.alpha = 1.0f;
    if (nemo_gemm(&a, stream)) return -1;
    nb::launch(row_argmax_kernel, (rows + 7) / 8, 256, 0, st, logits, ldl, V, enc_row_of, rows, out_idx, out_val);
    return nb_check_launch("row_argmax_kernel");
}
