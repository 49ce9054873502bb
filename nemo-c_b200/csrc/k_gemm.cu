// bf16-weight GEMM with fused epilogues: C (=/+=) alpha * act(A . W^T + bias).
// Replaces k_gemm (src/model.c:70-99) and gemm_bf16 / gemm_spec / gemm_mma
// (src/kernels.metal:12-208). The kernel is picked by row count like k_gemm does:
//   M <= 16 : weight streaming on CUDA cores (one warp per output column, 128-bit bf16 loads,
//             warp-shuffle reduction), as the Metal gemm_spec;
//   M  > 16 : tensor-core tiles (k_gemm_tc.cu) when A is in bf16 hi/lo planes, else a shared-
//             memory tiled CUDA-core kernel.
#include <cstdio>
#include "gemm_epi.cuh"

int nb_gemm_tc(const nemo_gemm_args_t *a, void *stream);  // k_gemm_tc.cu
int nb_gemm_tc_layout(const nemo_gemm_args_t *a, int layout, void *stream);

namespace {

using nb::Epi;
using nb::epilogue;
using nb::make_epi;

// ---- M <= 16: weight streaming, one warp per output column (pair for GLU) ----------------
template <int MB>
__global__ void __launch_bounds__(256) gemm_ws_kernel(const float *__restrict__ A, int64_t lda, const uint16_t *__restrict__ W,
                                                      int64_t ldw, int M, const int *dynM, int N, int K, const int *rowoff_p, Epi e) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nout = e.act == NEMO_ACT_GLU ? N / 2 : N;
    const int u = blockIdx.x * 8 + warp;
    nb::pdl_wait();
    if (dynM) M = min(M, *dynM);
    if (u >= nout || M <= 0) return;
    const bool glu = e.act == NEMO_ACT_GLU;
    const uint4 *wa = (const uint4 *)(W + (int64_t)u * ldw);
    const uint4 *wb = (const uint4 *)(W + (int64_t)(glu ? u + N / 2 : u) * ldw);
    float acc[2][MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) acc[0][m] = acc[1][m] = 0.0f;
    const int K8 = K >> 3;
    for (int k8 = lane; k8 < K8; k8 += 32) {
        const uint4 x = __ldg(wa + k8);
        float w0[8] = { nb::bf16lo(x.x), nb::bf16hi(x.x), nb::bf16lo(x.y), nb::bf16hi(x.y),
                        nb::bf16lo(x.z), nb::bf16hi(x.z), nb::bf16lo(x.w), nb::bf16hi(x.w) };
        float w1[8];
        if (glu) {
            const uint4 y = __ldg(wb + k8);
            w1[0] = nb::bf16lo(y.x); w1[1] = nb::bf16hi(y.x); w1[2] = nb::bf16lo(y.y); w1[3] = nb::bf16hi(y.y);
            w1[4] = nb::bf16lo(y.z); w1[5] = nb::bf16hi(y.z); w1[6] = nb::bf16lo(y.w); w1[7] = nb::bf16hi(y.w);
        }
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            if (m < M) {
                const float4 *ap = (const float4 *)(A + (int64_t)m * lda) + 2 * k8;
                const float4 a0 = __ldg(ap), a1 = __ldg(ap + 1);
                acc[0][m] += a0.x * w0[0] + a0.y * w0[1] + a0.z * w0[2] + a0.w * w0[3] + a1.x * w0[4] + a1.y * w0[5] + a1.z * w0[6] + a1.w * w0[7];
                if (glu) acc[1][m] += a0.x * w1[0] + a0.y * w1[1] + a0.z * w1[2] + a0.w * w1[3] + a1.x * w1[4] + a1.y * w1[5] + a1.z * w1[6] + a1.w * w1[7];
            }
        }
    }
    const int rowoff = rowoff_p ? *rowoff_p : 0;
#pragma unroll
    for (int m = 0; m < MB; ++m) {
        if (m < M) {
            const float va = nb::warp_sum(acc[0][m]);
            const float vb = glu ? nb::warp_sum(acc[1][m]) : 0.0f;
            if (lane == 0) epilogue(e, rowoff, m, u, u + N / 2, va, vb);
        }
    }
}

// ---- M > 16, fp32 A: shared-memory tiled CUDA-core GEMM (64 x 64 x 32, 4x4 per thread) -----
__global__ void __launch_bounds__(256) gemm_tiled_kernel(const float *__restrict__ A, int64_t lda, const uint16_t *__restrict__ W,
                                                         int64_t ldw, int M, const int *dynM, int N, int K, const int *rowoff_p, Epi e) {
    __shared__ float As[32][64 + 4];
    __shared__ float Ws[32][64 + 4];
    __shared__ float Wb[32][64 + 4];
    const bool glu = e.act == NEMO_ACT_GLU;
    const int nout = glu ? N / 2 : N;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {}, accb[4][4] = {};
    nb::pdl_wait();
    if (dynM) M = min(M, *dynM);
    if (m0 >= M) return;
    for (int k0 = 0; k0 < K; k0 += 32) {
        for (int i = threadIdx.x; i < 64 * 32; i += 256) {
            const int r = i >> 5, kk = i & 31;
            const int m = m0 + r, n = n0 + r, k = k0 + kk;
            As[kk][r] = (m < M && k < K) ? A[(int64_t)m * lda + k] : 0.0f;
            Ws[kk][r] = (n < nout && k < K) ? nb::bf2f(W[(int64_t)n * ldw + k]) : 0.0f;
            if (glu) Wb[kk][r] = (n < nout && k < K) ? nb::bf2f(W[(int64_t)(n + N / 2) * ldw + k]) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < 32; ++kk) {
            float a[4], w[4], wb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; w[i] = Ws[kk][tx * 4 + i]; }
            if (glu) {
#pragma unroll
                for (int i = 0; i < 4; ++i) wb[i] = Wb[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] += a[i] * w[j];
                    if (glu) accb[i][j] += a[i] * wb[j];
                }
        }
        __syncthreads();
    }
    const int rowoff = rowoff_p ? *rowoff_p : 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
            if (m < M && n < nout) epilogue(e, rowoff, m, n, n + N / 2, acc[i][j], accb[i][j]);
        }
}

}  // namespace

// Argument checks shared by every GEMM entry point (`who` names the entry in the message).
extern "C" int nb_gemm_validate(const nemo_gemm_args_t *a, const char *who) {
    if (!a) return nb_set_error("%s: null arguments", who);
    if (!a->A || !a->W || !a->C) return nb_set_error("%s: null pointer", who);
    if (a->M < 0 || a->N <= 0 || a->K <= 0) return nb_set_error("%s: bad shape M=%d N=%d K=%d", who, a->M, a->N, a->K);
    if (a->act == NEMO_ACT_GLU && (a->N & 1)) return nb_set_error("%s: GLU needs an even N", who);
    if (a->accumulate && a->c_fmt != NEMO_FMT_F32) return nb_set_error("%s: accumulate needs an fp32 output", who);
    return 0;
}

static int launch_ws(const nemo_gemm_args_t *a, cudaStream_t st) {
    if ((a->K & 7) || (a->ldw & 7) || (a->lda & 3) || ((uintptr_t)a->W & 15) || ((uintptr_t)a->A & 15))
        return nb_set_error("nemo_gemm (streaming): K, ldw must be multiples of 8, lda of 4, A/W 16-byte aligned");
    const int nout = a->act == NEMO_ACT_GLU ? a->N / 2 : a->N;
    const dim3 grid((nout + 7) / 8);
    const Epi e = make_epi(a);
    const float *A = (const float *)a->A;
    if (a->M <= 1) nb::launch(gemm_ws_kernel<1>, grid, 256, 0, st, A, a->lda, a->W, a->ldw, a->M, a->dynM, a->N, a->K, a->rowoff, e);
    else if (a->M <= 2) nb::launch(gemm_ws_kernel<2>, grid, 256, 0, st, A, a->lda, a->W, a->ldw, a->M, a->dynM, a->N, a->K, a->rowoff, e);
    else if (a->M <= 4) nb::launch(gemm_ws_kernel<4>, grid, 256, 0, st, A, a->lda, a->W, a->ldw, a->M, a->dynM, a->N, a->K, a->rowoff, e);
    else if (a->M <= 8) nb::launch(gemm_ws_kernel<8>, grid, 256, 0, st, A, a->lda, a->W, a->ldw, a->M, a->dynM, a->N, a->K, a->rowoff, e);
    else nb::launch(gemm_ws_kernel<16>, grid, 256, 0, st, A, a->lda, a->W, a->ldw, a->M, a->dynM, a->N, a->K, a->rowoff, e);
    return nb_check_launch("gemm_ws_kernel");
}

static int launch_tiled(const nemo_gemm_args_t *a, cudaStream_t st) {
    const int nout = a->act == NEMO_ACT_GLU ? a->N / 2 : a->N;
    const dim3 grid((nout + 63) / 64, (a->M + 63) / 64);
    nb::launch(gemm_tiled_kernel, grid, 256, 0, st, (const float *)a->A, a->lda, a->W, a->ldw, a->M, a->dynM, a->N, a->K, a->rowoff, make_epi(a));
    return nb_check_launch("gemm_tiled_kernel");
}

extern "C" int nemo_gemm_forced(const nemo_gemm_args_t *a, int kind, void *stream) {
    if (nb_gemm_validate(a, "nemo_gemm")) return -1;
    if (a->M == 0) return 0;
    cudaStream_t st = (cudaStream_t)stream;
    if (kind == 0) {
        if (a->a_fmt == NEMO_FMT_BF16X2) kind = 2;
        else kind = a->M <= 16 ? 1 : 3;
    }
    if (kind == 2 || kind == 4 || kind == 5 || kind == 6) {
        if (a->a_fmt != NEMO_FMT_BF16X2) return nb_set_error("nemo_gemm: tensor-core path needs A as bf16 hi/lo planes");
        return nb_gemm_tc_layout(a, kind == 2 ? 0 : kind - 3, stream);
    }
    if (a->a_fmt != NEMO_FMT_F32) return nb_set_error("nemo_gemm: CUDA-core paths need fp32 A");
    if (kind == 1) {
        if (a->M > 16) return nb_set_error("nemo_gemm: streaming path handles M <= 16");
        return launch_ws(a, st);
    }
    return launch_tiled(a, st);
}

extern "C" int nemo_gemm(const nemo_gemm_args_t *a, void *stream) { return nemo_gemm_forced(a, 0, stream); }
