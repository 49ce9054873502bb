// Tensor-core GEMM for the bf16-weight projections: tcgen05.mma (kind::f16, fp32 accumulate in
// TMEM) fed by TMA tile loads into a shared-memory ring, fused epilogue from TMEM.
//
// Orientation: the weight rows are the MMA's 128-row M side and the activation rows its N side
// (16..256), so one kernel serves a single stream (a handful of rows: the weights stream through
// every SM with split-K) and batches of many streams (thousands of rows). D[n][m] accumulates
// W[n][:] . A[m][:]; TMEM lane = weight row n, TMEM column = activation row m.
//
// Activations arrive as two bf16 planes (hi = bf16(x), lo = bf16(x - hi)); each k-step issues
// two MMAs (W.hi and W.lo) into the same accumulator, so the products carry ~16 mantissa bits of
// the fp32 activations (bf16 weights are exact). Split-K partial tiles are reduced by the last
// CTA of each tile in a fixed order, so results do not depend on scheduling.
//
// Warp roles (192 threads): warp 0 issues TMA loads, warp 1 owns TMEM and issues the MMAs,
// warps 2-5 run the epilogue (warp w reads TMEM lanes 32*(w%4) .. +31). Every wait is bounded.
#include <cuda.h>
#include <cstdio>
#include <cstring>
#include <mutex>
#include "gemm_epi.cuh"
#include "sm100.cuh"

namespace {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // k per stage: 128 bytes of bf16 = one swizzle span
constexpr int W_STAGE = BM * BK * 2;
constexpr int THREADS = 192;

__device__ int g_tc_error;  // set when a bounded wait gave up (host reads it back)

struct TcArgs {
    int M, N, K, kblocks, splits, kb_per_split, n_wtiles, n_mtiles, glu;
    const int *dynM, *rowoff;
    nb::Epi e;
    float *ws;     // split-K partial tiles
    int *counters; // one arrival counter per output tile (zero between launches)
};

template <int BN>
struct Cfg {
    static constexpr int A_STAGE = BN * BK * 2;                 // one activation plane
    static constexpr int STAGE = W_STAGE + 2 * A_STAGE;
    static constexpr int STAGES = BN <= 32 ? 8 : BN <= 64 ? 6 : BN <= 128 ? 4 : 2;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr int SMEM = 1024 + STAGES * STAGE + 1024 + 64 * 16 * 4;
};

template <int BN>
__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmAh,
                                                           const __grid_constant__ CUtensorMap tmAl, const TcArgs p) {
    using C = Cfg<BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *stages = smem;
    uint64_t *full = (uint64_t *)(smem + C::STAGES * C::STAGE);
    uint64_t *empty = full + C::STAGES;
    uint64_t *done = empty + C::STAGES;
    uint32_t *tmem_holder = (uint32_t *)(done + 1);
    volatile int *flags = (volatile int *)(tmem_holder + 1); // [0] abort, [1] last-split
    float *xch = (float *)(smem + C::STAGES * C::STAGE + 1024); // GLU exchange [16][64]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x % p.splits, tile = blockIdx.x / p.splits;
    const int wt = tile % p.n_wtiles, mt = tile / p.n_wtiles;
    const int kb0 = split * p.kb_per_split;
    const int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
    const int nk = kb1 - kb0;

    nb::pdl_wait();
    const int M = p.dynM ? min(p.M, *p.dynM) : p.M;
    if (mt * BN >= M || nk <= 0) return; // whole CTA leaves before touching TMEM or barriers

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { sm100::mbar_init(&full[s], 1); sm100::mbar_init(&empty[s], 1); }
        sm100::mbar_init(done, 1);
        flags[0] = 0;
        flags[1] = 0;
        sm100::fence_mbar_init();
        sm100::tma_prefetch_desc(&tmW);
        sm100::tma_prefetch_desc(&tmAh);
        sm100::tma_prefetch_desc(&tmAl);
    }
    if (warp == 1) {
        sm100::tmem_alloc(tmem_holder, C::TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0 && lane == 0) {
        // ---- producer: weight tile (two 64-row halves for GLU) + activation hi/lo tiles ----
        for (int i = 0; i < nk; ++i) {
            const int s = i % C::STAGES;
            if (i >= C::STAGES && !sm100::mbar_wait(&empty[s], ((i / C::STAGES) - 1) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 1); break; }
            if (flags[0]) break;
            uint8_t *st = stages + s * C::STAGE;
            const int k0 = (kb0 + i) * BK;
            sm100::mbar_arrive_expect_tx(&full[s], C::STAGE);
            if (p.glu) {
                sm100::tma_load_2d(st, &tmW, &full[s], k0, wt * 64);
                sm100::tma_load_2d(st + W_STAGE / 2, &tmW, &full[s], k0, p.N / 2 + wt * 64);
            } else {
                sm100::tma_load_2d(st, &tmW, &full[s], k0, wt * BM);
            }
            sm100::tma_load_2d(st + W_STAGE, &tmAh, &full[s], k0, mt * BN);
            sm100::tma_load_2d(st + W_STAGE + C::A_STAGE, &tmAl, &full[s], k0, mt * BN);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        constexpr uint32_t idesc = sm100::idesc_bf16_f32(BM, BN);
        for (int i = 0; i < nk; ++i) {
            const int s = i % C::STAGES;
            if (!sm100::mbar_wait(&full[s], (i / C::STAGES) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 2); break; }
            sm100::tc_fence_after();
            const uint32_t w_addr = sm100::smem_u32(stages + s * C::STAGE);
            const uint32_t h_addr = w_addr + W_STAGE, l_addr = h_addr + C::A_STAGE;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
                const uint64_t ad = sm100::desc_k_sw128(w_addr + kk * 32);
                sm100::mma_bf16(tmem, ad, sm100::desc_k_sw128(h_addr + kk * 32), idesc, (i | kk) != 0);
                sm100::mma_bf16(tmem, ad, sm100::desc_k_sw128(l_addr + kk * 32), idesc, 1);
            }
            sm100::mma_commit(&empty[s]);
        }
        sm100::mma_commit(done);
    } else if (warp >= 2) {
        // ---- epilogue: TMEM -> registers -> (split-K reduce) -> fused epilogue -> global ----
        const int q = warp & 3;               // TMEM lane quarter this warp may access
        const int row = q * 32 + lane;        // weight row inside the tile
        const int etid = threadIdx.x - 64;    // 0..127
        const bool ok = sm100::mbar_wait(done, 0);
        if (!ok) { flags[0] = 1; atomicExch(&g_tc_error, 3); }
        sm100::tc_fence_after();
        const int rowoff = p.rowoff ? *p.rowoff : 0;
        const int nout = p.glu ? p.N / 2 : p.N;
        float *wsb = p.ws + (int64_t)tile * p.splits * BN * BM;
        if (ok && p.splits > 1) {
            for (int j0 = 0; j0 < BN; j0 += 16) {
                float v[16];
                sm100::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + j0, v);
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) wsb[((int64_t)split * BN + j0 + jj) * BM + row] = v[jj];
            }
            __threadfence();
            sm100::named_barrier(1, 128);
            if (etid == 0) flags[1] = atomicAdd(&p.counters[tile], 1) == p.splits - 1;
            sm100::named_barrier(1, 128);
        }
        const bool finish = ok && (p.splits == 1 || flags[1]);
        if (finish) {
            if (p.splits > 1) __threadfence();
            for (int j0 = 0; j0 < BN; j0 += 16) {
                float v[16];
                if (p.splits == 1) {
                    sm100::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + j0, v);
                } else {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) v[jj] = 0.0f;
                    for (int s = 0; s < p.splits; ++s)
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) v[jj] += __ldcg(&wsb[((int64_t)s * BN + j0 + jj) * BM + row]);
                }
                if (p.glu) {
                    // rows 64..127 hold the gate halves (columns n + N/2): hand them over
                    if (row >= 64)
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) xch[jj * 64 + row - 64] = v[jj];
                    sm100::named_barrier(1, 128);
                    if (row < 64) {
                        const int n = wt * 64 + row;
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int m = mt * BN + j0 + jj;
                            if (m < M && n < nout) nb::epilogue(p.e, rowoff, m, n, n + p.N / 2, v[jj], xch[jj * 64 + row]);
                        }
                    }
                    sm100::named_barrier(1, 128);
                } else {
                    const int n = wt * BM + row;
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int m = mt * BN + j0 + jj;
                        if (m < M && n < nout) nb::epilogue(p.e, rowoff, m, n, 0, v[jj], 0.0f);
                    }
                }
            }
            if (p.splits > 1 && etid == 0) p.counters[tile] = 0; // ready for the next launch
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---- host side -------------------------------------------------------------------------------
typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_mu;
EncodeTiled g_encode = nullptr;
float *g_ws = nullptr;
int *g_counters = nullptr;
size_t g_ws_floats = 0;
int g_ncounters = 0;
int g_sms = 148;

constexpr size_t WS_FLOATS = (size_t)16 << 20;   // 64 MB of split-K partials
constexpr int NCOUNTERS = 1 << 16;

int init_once() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode) return 0;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
        return nb_set_error("tensor-core GEMM: cuTensorMapEncodeTiled unavailable");
    if (cudaMalloc(&g_ws, WS_FLOATS * sizeof(float)) != cudaSuccess || cudaMalloc(&g_counters, NCOUNTERS * sizeof(int)) != cudaSuccess ||
        cudaMemset(g_counters, 0, NCOUNTERS * sizeof(int)) != cudaSuccess)
        return nb_set_error("tensor-core GEMM: cannot allocate the split-K workspace");
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    g_ws_floats = WS_FLOATS;
    g_ncounters = NCOUNTERS;
    cudaFuncSetAttribute(gemm_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<16>::SMEM);
    cudaFuncSetAttribute(gemm_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<32>::SMEM);
    cudaFuncSetAttribute(gemm_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<64>::SMEM);
    cudaFuncSetAttribute(gemm_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<128>::SMEM);
    cudaFuncSetAttribute(gemm_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256>::SMEM);
    g_encode = (EncodeTiled)fn;
    return 0;
}

int make_map(CUtensorMap *m, const void *base, int64_t cols, int64_t rows, int64_t ld_elems, int box_rows) {
    if (((uintptr_t)base & 15) || ((ld_elems * 2) & 15)) return nb_set_error("tensor-core GEMM: base and row pitch must be 16-byte aligned");
    cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    cuuint64_t strides[1] = { (cuuint64_t)(ld_elems * 2) };
    cuuint32_t box[2] = { (cuuint32_t)BK, (cuuint32_t)box_rows };
    cuuint32_t es[2] = { 1, 1 };
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return nb_set_error("tensor-core GEMM: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

template <int BN>
int launch(const nemo_gemm_args_t *a, cudaStream_t st) {
    CUtensorMap mw, mh, ml;
    const bool glu = a->act == NEMO_ACT_GLU;
    if (make_map(&mw, a->W, a->K, a->N, a->ldw, glu ? 64 : BM)) return -1;
    const uint16_t *A = (const uint16_t *)a->A;
    if (make_map(&mh, A, a->K, a->M, a->lda, BN) || make_map(&ml, A + a->a_plane, a->K, a->M, a->lda, BN)) return -1;
    TcArgs p;
    memset(&p, 0, sizeof p);
    p.M = a->M; p.N = a->N; p.K = a->K;
    p.kblocks = (a->K + BK - 1) / BK;
    p.glu = glu;
    p.n_wtiles = glu ? (a->N / 2 + 63) / 64 : (a->N + BM - 1) / BM;
    p.n_mtiles = (a->M + BN - 1) / BN;
    const int tiles = p.n_wtiles * p.n_mtiles;
    int splits = 1;
    if (tiles < g_sms) {
        splits = (g_sms + tiles - 1) / tiles;
        if (splits > p.kblocks) splits = p.kblocks;
        if ((size_t)tiles * splits * BN * BM > g_ws_floats || tiles > g_ncounters) splits = 1;
    }
    p.kb_per_split = (p.kblocks + splits - 1) / splits;
    p.splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split; // every split non-empty
    p.dynM = a->dynM;
    p.rowoff = a->rowoff;
    p.e = nb::make_epi(a);
    p.ws = g_ws;
    p.counters = g_counters;
    gemm_tc_kernel<BN><<<tiles * p.splits, THREADS, Cfg<BN>::SMEM, st>>>(mw, mh, ml, p);
    return nb_check_launch("gemm_tc_kernel");
}

}  // namespace

int nb_gemm_tc(const nemo_gemm_args_t *a, void *stream) {
    if (init_once()) return -1;
    if (a->act == NEMO_ACT_GLU && ((a->N / 2) % 64)) return nb_set_error("tensor-core GEMM: GLU needs N/2 to be a multiple of 64");
    if (a->K % 8) return nb_set_error("tensor-core GEMM: K must be a multiple of 8");
    cudaStream_t st = (cudaStream_t)stream;
    if (a->M <= 16) return launch<16>(a, st);
    if (a->M <= 32) return launch<32>(a, st);
    if (a->M <= 64) return launch<64>(a, st);
    if (a->M <= 128) return launch<128>(a, st);
    return launch<256>(a, st);
}

extern "C" int nemo_gpu_check_device_errors(void) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof v) != cudaSuccess) return nb_set_error("cannot read the device error flag");
    if (v) return nb_set_error("tensor-core GEMM: a bounded wait gave up (code %d)", v);
    return 0;
}
