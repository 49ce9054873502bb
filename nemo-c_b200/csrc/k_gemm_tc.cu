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
// Persistent: one CTA per SM walks a strided list of work units (tile, k-split). The TMEM
// accumulator is double-buffered, so the epilogue of one unit runs while the MMAs of the next
// proceed. Warp roles (320 threads): warp 0 issues TMA loads, warp 1 owns TMEM and issues the
// MMAs, warps 2-9 run the epilogue (warp w reads TMEM lanes 32*(w%4) .. +31; warps w and w+4
// split the columns). Every wait is bounded: on a timeout the CTA records an error and unwinds.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include "gemm_epi.cuh"
#include "sm100.cuh"
#include "gridsync.cuh"
#include "engine_dev.h"

namespace {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // k per stage: 128 bytes of bf16 = one swizzle span
constexpr int W_STAGE = BM * BK * 2;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;

__device__ int g_tc_error;  // set when a bounded wait gave up (host reads it back)

struct TcArgs {
    int M, N, K, kblocks, splits, kb_per_split, n_wtiles, n_mtiles, units, glu;
    int vec;       // activation-major epilogue may use 16-byte accesses (alignment checked on the host)
    const int *dynM, *rowoff;
    nb::Epi e;
    float *ws;     // split-K partial tiles
    int *counters; // one arrival counter per output tile (zero between launches)
    NbDecEpi de;   // de.mode != 0: a batched greedy decoder epilogue replaces the plain one (activation-major tiles)
    int sk_q;      // activation-major stream-K: k-blocks per CTA (0: units of whole k-splits instead)
    int slots;     // partial-tile slots per output tile in ws (splits, or the most stream-K pieces of a tile)
};

// The work of one activation-major CTA, walked identically by its producer, MMA and epilogue
// roles: pieces (tile, k-blocks [kb0, kb1), slot of the piece among the tile's `parts`).
// k-split units: unit u = blockIdx.x, blockIdx.x + gridDim.x, ... is (tile u / splits, split u % splits).
// Stream-K: the CTA owns the k-blocks [blockIdx.x * q, (blockIdx.x + 1) * q) of the flattened
// (tile, k-block) space, cut at tile boundaries; a tile's pieces are numbered by CTA.
struct Piece {
    int tile, kb0, kb1, slot, parts;
};
struct PieceIter {
    int cur, end;
    __device__ __forceinline__ PieceIter(const TcArgs &p, int tiles) {
        if (p.sk_q) {
            cur = blockIdx.x * p.sk_q;
            end = min(tiles * p.kblocks, cur + p.sk_q);
        } else {
            cur = blockIdx.x;
            end = tiles * p.splits;
        }
    }
    __device__ __forceinline__ bool next(const TcArgs &p, Piece &w) {
        if (cur >= end) return false;
        if (!p.sk_q) {
            const int split = cur % p.splits;
            w.tile = cur / p.splits;
            w.kb0 = split * p.kb_per_split;
            w.kb1 = min(p.kblocks, w.kb0 + p.kb_per_split);
            w.slot = split;
            w.parts = p.splits;
            cur += gridDim.x;
            return true;
        }
        const int kb = p.kblocks, q = p.sk_q;
        w.tile = cur / kb;
        w.kb0 = cur - w.tile * kb;
        const int tile_end = (w.tile + 1) * kb, e = min(end, tile_end);
        w.kb1 = w.kb0 + (e - cur);
        const int first = (w.tile * kb) / q;
        w.parts = (tile_end - 1) / q - first + 1;
        w.slot = (int)blockIdx.x - first;
        cur = e;
        return true;
    }
};

template <int BN>
struct Cfg {
    static constexpr int A_STAGE = BN * BK * 2;                 // one activation plane
    static constexpr int STAGE = W_STAGE + 2 * A_STAGE;
    static constexpr int STAGES = BN <= 32 ? 8 : BN <= 64 ? 6 : BN <= 128 ? 4 : 2;
    static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN; // two accumulator buffers
    static constexpr int HALF = BN >= 32 ? BN / 2 : BN;        // columns per epilogue warp
    static constexpr int XCH = 2 * 16 * 64;                     // GLU exchange, two halves [16][64]
    // stages | barriers (1 KB) | GLU exchange | per-row output offsets | per-row bias offsets
    static constexpr int SMEM = 1024 + STAGES * STAGE + 1024 + XCH * 4 + BN * 12;
};

// 1 / (1 + e^-x) with the hardware exp2 and reciprocal approximations (relative error ~1e-6)
__device__ __forceinline__ float fast_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// Epilogue for one 16-row chunk of one weight row: va[jj] belongs to activation row m0+j0+jj and
// output column n. Row offsets (group stride, in-group row offset, ldc) were precomputed once
// per unit; branches are uniform across the warp.
__device__ __forceinline__ void epi_chunk(const nb::Epi &e, const int64_t *__restrict__ rowbase, const int *__restrict__ brow, int m0, int j0,
                                          int mcount, int n, int nb_, const float (&va)[16], const float *vb, float bias_a, float bias_b,
                                          bool row_bias) {
    float *__restrict__ C32 = (float *)e.C;
    uint16_t *__restrict__ C16 = (uint16_t *)e.C;
    // every global load of the chunk (accumulated output, per-row bias) is issued before the
    // first store, so their latencies overlap instead of queueing behind the stores
    float cin[16], rba[16], rbb[16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
        const int ml = j0 + jj;
        cin[jj] = rba[jj] = rbb[jj] = 0.0f;
        if (ml < mcount) {
            if (e.accumulate) cin[jj] = C32[rowbase[ml] + n];
            if (row_bias) {
                rba[jj] = e.bias[brow[ml] + n];
                if (vb) rbb[jj] = e.bias[brow[ml] + nb_];
            }
        }
    }
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
        const int ml = j0 + jj;
        if (ml >= mcount) break;
        const float ba = row_bias ? rba[jj] : bias_a, bb = row_bias ? rbb[jj] : bias_b;
        float v;
        if (vb) {
            v = (va[jj] + ba) * fast_sigmoid(vb[jj] + bb) * e.alpha;
        } else {
            v = va[jj] + ba;
            if (e.act == NEMO_ACT_SILU) v = v * fast_sigmoid(v);
            else if (e.act == NEMO_ACT_RELU) v = fmaxf(v, 0.0f);
            v *= e.alpha;
        }
        const int64_t idx = rowbase[ml] + n;
        v += cin[jj];
        if (e.c_fmt == NEMO_FMT_F32) {
            C32[idx] = v;
        } else {
            const uint16_t hi = nb::f2bf(v);
            C16[idx] = hi;
            C16[idx + e.c_plane] = nb::f2bf(v - nb::bf2f(hi));
        }
        if (e.c32) e.c32[(int64_t)(m0 + ml) * e.ldc32 + n] = v;
    }
}

template <int BN>
__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmAh,
                                                           const __grid_constant__ CUtensorMap tmAl, const __grid_constant__ TcArgs p) {
    using C = Cfg<BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *stages = smem;
    uint64_t *full = (uint64_t *)(smem + C::STAGES * C::STAGE);
    uint64_t *empty = full + C::STAGES;
    uint64_t *acc_full = empty + C::STAGES;  // [2] MMA -> epilogue: accumulator buffer ready
    uint64_t *acc_empty = acc_full + 2;      // [2] epilogue -> MMA: accumulator buffer drained
    uint32_t *tmem_holder = (uint32_t *)(acc_empty + 2);
    volatile int *flags = (volatile int *)(tmem_holder + 1); // [0] abort, [1] last split of the unit, [2] epilogue abort
    float *xch = (float *)(smem + C::STAGES * C::STAGE + 1024);
    int64_t *rowbase = (int64_t *)(xch + C::XCH);
    int *brow = (int *)(rowbase + BN);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // set-up first: with programmatic dependent launch it overlaps the previous kernel's tail
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { sm100::mbar_init(&full[s], 1); sm100::mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { sm100::mbar_init(&acc_full[b], 1); sm100::mbar_init(&acc_empty[b], 1); }
        flags[0] = 0;
        flags[2] = 0;
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
    nb::pdl_wait();  // inputs of the previous kernel are visible from here on
    const int M = p.dynM ? min(p.M, *p.dynM) : p.M;
    const int live_mtiles = (M + BN - 1) / BN;            // row tiles that hold real rows
    const int units = live_mtiles * p.n_wtiles * p.splits; // CTAs at or beyond it have nothing to do

    if (warp == 0 && lane == 0) {
        // ---- producer: weight tile (two 64-row halves for GLU) + activation hi/lo tiles ----
        int i = 0; // k-blocks issued by this CTA (ring position)
        for (int u = blockIdx.x; u < units && !flags[0]; u += gridDim.x) {
            const int split = u % p.splits, tile = u / p.splits, wt = tile % p.n_wtiles, mt = tile / p.n_wtiles;
            const int kb0 = split * p.kb_per_split, kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            for (int kb = kb0; kb < kb1; ++kb, ++i) {
                const int s = i % C::STAGES;
                if (i >= C::STAGES && !sm100::mbar_wait(&empty[s], ((i / C::STAGES) - 1) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 1); break; }
                if (flags[0]) break;
                uint8_t *st = stages + s * C::STAGE;
                const int k0 = kb * BK;
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
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer: one accumulator buffer per unit, alternating ----
        constexpr uint32_t idesc = sm100::idesc_bf16_f32(BM, BN);
        int i = 0, t = 0;
        for (int u = blockIdx.x; u < units && !flags[0]; u += gridDim.x, ++t) {
            const int split = u % p.splits;
            const int kb0 = split * p.kb_per_split, kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            const int b = t & 1;
            if (t >= 2 && !sm100::mbar_wait(&acc_empty[b], ((t >> 1) - 1) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 4); break; }
            sm100::tc_fence_after();
            const uint32_t dacc = tmem + (uint32_t)(b * BN);
            for (int kb = kb0; kb < kb1; ++kb, ++i) {
                const int s = i % C::STAGES;
                if (!sm100::mbar_wait(&full[s], (i / C::STAGES) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 2); break; }
                sm100::tc_fence_after();
                const uint32_t w_addr = sm100::smem_u32(stages + s * C::STAGE);
                const uint32_t h_addr = w_addr + W_STAGE, l_addr = h_addr + C::A_STAGE;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t ad = sm100::desc_k_sw128(w_addr + kk * 32);
                    sm100::mma_bf16(dacc, ad, sm100::desc_k_sw128(h_addr + kk * 32), idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                    sm100::mma_bf16(dacc, ad, sm100::desc_k_sw128(l_addr + kk * 32), idesc, 1u);
                }
                sm100::mma_commit(&empty[s]);
            }
            sm100::mma_commit(&acc_full[b]);
        }
    } else if (warp >= 2) {
        // ---- epilogue: TMEM -> registers -> (split-K reduce) -> fused epilogue -> global ----
        const int ew = warp - 2;                 // 0..7
        const int q = warp & 3;                  // TMEM lane quarter this warp may access
        const int half = ew >> 2;                // which half of the columns
        const int row = q * 32 + lane;           // weight row inside the tile
        const int etid = threadIdx.x - 64;       // 0..255
        const int nout = p.glu ? p.N / 2 : p.N;
        const bool has_half = half * C::HALF < BN;
        const int jbeg = half * C::HALF, jend = has_half ? jbeg + C::HALF : jbeg;
        float *xh = xch + half * 16 * 64;
        const bool row_bias = p.e.bias && p.e.bias_gstride != 0;
        const int rowoff = p.rowoff ? *p.rowoff : 0;
        int t = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++t) {
            const int split = u % p.splits, tile = u / p.splits, wt = tile % p.n_wtiles, mt = tile / p.n_wtiles;
            const int b = t & 1;
            const int m0 = mt * BN, mcount = min(BN, M - m0);
            // output row offsets of this unit (computed while its MMAs run)
            sm100::named_barrier(1, 256);        // the previous unit is done with rowbase/brow
            for (int ml = etid; ml < BN; ml += 256) {
                const int m = m0 + ml, g = m / p.e.rpg, r = m - g * p.e.rpg;
                rowbase[ml] = (int64_t)g * p.e.gstride + (int64_t)(rowoff + r) * p.e.ldc;
                brow[ml] = (int)((int64_t)g * p.e.bias_gstride);
            }
            const int ncol = p.glu ? wt * 64 + row : wt * BM + row;
            const bool col_ok = ncol < nout && (!p.glu || row < 64);
            float bias_a = 0.0f, bias_b = 0.0f;
            if (p.e.bias && !row_bias && col_ok) {
                bias_a = p.e.bias[ncol];
                if (p.glu) bias_b = p.e.bias[ncol + p.N / 2];
            }
            if (!sm100::mbar_wait(&acc_full[b], (t >> 1) & 1)) { flags[2] = 1; flags[0] = 1; atomicExch(&g_tc_error, 3); }
            // flags[2] is written only by epilogue threads before this barrier: every epilogue
            // thread takes the same decision (a divergent exit would strand the others)
            sm100::named_barrier(1, 256);
            const bool ok = !flags[2];
            sm100::tc_fence_after();
            const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN);
            float *wsb = p.ws + (int64_t)tile * p.splits * BN * BM;
            bool finish = ok;
            if (ok && p.splits > 1) {
                for (int j0 = jbeg; j0 < jend && j0 < mcount; j0 += 16) {
                    float v[16];
                    sm100::tmem_ld16(tacc + j0, v);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) wsb[((int64_t)split * BN + j0 + jj) * BM + row] = v[jj];
                }
                __threadfence();
                sm100::named_barrier(1, 256);
                if (etid == 0) flags[1] = atomicAdd(&p.counters[tile], 1) == p.splits - 1;
                sm100::named_barrier(1, 256);
                finish = flags[1];
                if (finish) __threadfence();
            }
            if (finish) {
                for (int j0 = jbeg; j0 < jend; j0 += 16) {
                    if (j0 >= mcount) break;
                    float v[16];
                    if (p.splits == 1) {
                        sm100::tmem_ld16(tacc + j0, v);
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
                            for (int jj = 0; jj < 16; ++jj) xh[jj * 64 + row - 64] = v[jj];
                        sm100::named_barrier(2 + half, 128);
                        if (col_ok) {
                            float vb[16];
#pragma unroll
                            for (int jj = 0; jj < 16; ++jj) vb[jj] = xh[jj * 64 + row];
                            epi_chunk(p.e, rowbase, brow, m0, j0, mcount, ncol, ncol + p.N / 2, v, vb, bias_a, bias_b, row_bias);
                        }
                        sm100::named_barrier(2 + half, 128);
                    } else if (col_ok) {
                        epi_chunk(p.e, rowbase, brow, m0, j0, mcount, ncol, 0, v, nullptr, bias_a, 0.0f, row_bias);
                    }
                }
                if (p.splits > 1 && etid == 0) p.counters[tile] = 0; // ready for the next launch
            }
            // this accumulator buffer may be overwritten by the unit after next
            sm100::tc_fence_before();
            sm100::named_barrier(1, 256);
            if (etid == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm100::smem_u32(&acc_empty[b])) : "memory");
            if (!ok) break;
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---- activation-major tiles for batches -------------------------------------------------------
// For many rows the roles swap: 128 activation rows are the MMA's M side (TMEM lanes) and BW
// weight rows (80, 112, 128, 160, 208, 224 or 256) its N side (TMEM columns); 80 only for the
// greedy decoder's GEMMs. The widths other than 128 and 256 (plain tiles only, no k-splits) exist
// for wave quantisation on 148 SMs: at 1792
// rows, N = 4096 makes 280 tiles of 208 (1.9 rounds: 416 weight rows on the busiest SM, against
// 448 with 266 tiles of 224 and 512 with 224 tiles of 256, 1.5 rounds: half the SMs idle through
// the second), N = 3072 makes 280 tiles of 160 (1.9 rounds) and N = 1024 makes 140
// tiles of 112 (one round; 128-row tiles leave 36 SMs idle). Accumulator buffer 1 starts at TMEM
// column 128 or 256 whatever the width; the epilogue splits a 112-column tile 64 + 48 between its
// two thread halves, so every 16-column TMEM load starts on a 16-column boundary. One k-step stages 2 x 16 KB of activation
// planes and BW x 128 B of weights for 128 x BW x 64 x 2 multiply-adds, 1.5x fewer bytes per
// MMA than the weight-major tile at BW = 256. Each epilogue thread owns one activation row and
// reads 16 consecutive output columns per TMEM load; a GLU tile holds the value half in TMEM
// columns [0, BW/2) and the gate half in [BW/2, BW), so both halves sit in the same thread.
template <int BW>
struct CfgR {
    static constexpr int A_PLANE = 128 * BK * 2;                 // 16 KB
    static constexpr int W_BYTES = BW * BK * 2;                  // 16 / 28 / 32 KB
    static constexpr int STAGE = 2 * A_PLANE + W_BYTES;          // a multiple of 1 KB (128-byte swizzle)
    static constexpr int STAGES = BW > 128 ? 3 : 4;
    static constexpr int ACC_STRIDE = BW > 128 ? 256 : 128;     // TMEM column of accumulator buffer 1
    static constexpr int TMEM_COLS = 2 * ACC_STRIDE;              // two accumulator buffers (a power of 2)
    static constexpr int SMEM = 1024 + STAGES * STAGE + 1024;    // stages | barriers
};

// Global operands of one 16-column chunk of the activation-major epilogue, requested a chunk ahead
// (the first chunk's before the accumulator is complete), so that their latency overlaps the MMAs
// and the previous chunk's math instead of adding an L2 round trip to every chunk:
//   plain / GLU tiles: a = bias, b = GLU gate bias, or the fp32 output being accumulated into;
//   argmax (decoder mode 3): a = bias (the columns that exist);
//   LSTM (mode 1): a = the stream's gate-table row, c = the cell state of the chunk's 4 units;
//   joint input (mode 2): a = bias, b = the encoder row; aux columns: a = aux bias.
struct EpiIn { float4 a[4], b[4], c; };

__device__ __forceinline__ void set4(float4 &v, int j, float f) {
    if (j == 0) v.x = f; else if (j == 1) v.y = f; else if (j == 2) v.z = f; else v.w = f;
}

// 16 consecutive output columns of one activation row (activation-major epilogue):
// bias -> activation (ACT: NEMO_ACT_*, GLU pairs value and gate) -> x alpha -> (+= C) -> store as
// fp32 or bf16 hi/lo planes (BF16 = true), plus the optional fp32 copy. 16-byte accesses.
template <int ACT, bool BF16>
__device__ __forceinline__ void epi16(const TcArgs &p, int64_t rowbase, int m, int n0, const float (&va)[16], const float (&vg)[16], const EpiIn &in) {
    float *__restrict__ C32 = (float *)p.e.C;
    float o[16], bv[16], bg[16];
#pragma unroll
    for (int x = 0; x < 16; x += 4) {
        const float4 b4 = in.a[x >> 2], g4 = ACT == NEMO_ACT_GLU ? in.b[x >> 2] : make_float4(0.f, 0.f, 0.f, 0.f);
        bv[x] = b4.x; bv[x + 1] = b4.y; bv[x + 2] = b4.z; bv[x + 3] = b4.w;
        bg[x] = g4.x; bg[x + 1] = g4.y; bg[x + 2] = g4.z; bg[x + 3] = g4.w;
    }
    const float alpha = p.e.alpha;
#pragma unroll
    for (int x = 0; x < 16; ++x) {
        float v = va[x] + bv[x];
        if (ACT == NEMO_ACT_GLU) v = v * fast_sigmoid(vg[x] + bg[x]);
        else if (ACT == NEMO_ACT_SILU) v = v * fast_sigmoid(v);
        else if (ACT == NEMO_ACT_RELU) v = fmaxf(v, 0.0f);
        o[x] = v * alpha;
    }
    const int64_t idx = rowbase + n0;
    if (!BF16) {
        if (p.e.accumulate) {
            // the accumulated output came with the operands, except for GLU tiles (whose b holds
            // the gate bias)
#pragma unroll
            for (int x = 0; x < 16; x += 4) {
                const float4 c4 = ACT == NEMO_ACT_GLU ? *(const float4 *)(C32 + idx + x) : in.b[x >> 2];
                o[x] += c4.x; o[x + 1] += c4.y; o[x + 2] += c4.z; o[x + 3] += c4.w;
            }
        }
#pragma unroll
        for (int x = 0; x < 16; x += 4) *(float4 *)(C32 + idx + x) = make_float4(o[x], o[x + 1], o[x + 2], o[x + 3]);
    } else {
        uint16_t *__restrict__ C16 = (uint16_t *)p.e.C;
        uint32_t h[8], l[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
            const __nv_bfloat162 hv = __floats2bfloat162_rn(o[2 * x], o[2 * x + 1]);
            const __nv_bfloat162 lv = __floats2bfloat162_rn(o[2 * x] - __low2float(hv), o[2 * x + 1] - __high2float(hv));
            h[x] = *(const uint32_t *)&hv;
            l[x] = *(const uint32_t *)&lv;
        }
        uint4 *dh = (uint4 *)(C16 + idx), *dl = (uint4 *)(C16 + idx + p.e.c_plane);
        dh[0] = make_uint4(h[0], h[1], h[2], h[3]);
        dh[1] = make_uint4(h[4], h[5], h[6], h[7]);
        dl[0] = make_uint4(l[0], l[1], l[2], l[3]);
        dl[1] = make_uint4(l[4], l[5], l[6], l[7]);
    }
    if (p.e.c32)
#pragma unroll
        for (int x = 0; x < 16; x += 4) *(float4 *)(p.e.c32 + (int64_t)m * p.e.ldc32 + n0 + x) = make_float4(o[x], o[x + 1], o[x + 2], o[x + 3]);
}

// Batched greedy decoder epilogues: 16 output columns of GEMM row m, whose stream is b.
// LSTM cell (src/kernels.metal:475-486) on gate-interleaved columns: columns n0 .. n0 + 15 are
// gates i, f, g, o of units n0 / 4 .. n0 / 4 + 3; `row` is the stream's gate row (bias included).
__device__ __forceinline__ void dec_lstm16(const NbDecEpi &de, int m, int b, int n0, const float (&va)[16], const EpiIn &in) {
    const int u0 = n0 >> 2, ph = de.n_split >> 2;
    float g[16];
#pragma unroll
    for (int x = 0; x < 16; x += 4) {
        const float4 b4 = in.a[x >> 2];
        g[x] = va[x] + b4.x; g[x + 1] = va[x + 1] + b4.y; g[x + 2] = va[x + 2] + b4.z; g[x + 3] = va[x + 3] + b4.w;
    }
    float *cp = de.c + (int64_t)b * ph + u0;
    const float4 c4 = in.c;
    const float cold[4] = { c4.x, c4.y, c4.z, c4.w };
    float cc[4], hh[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float ig = nb::sigmoid_f(g[4 * q]), fg = nb::sigmoid_f(g[4 * q + 1]), gg = tanhf(g[4 * q + 2]), og = nb::sigmoid_f(g[4 * q + 3]);
        cc[q] = fg * cold[q] + ig * gg;
        hh[q] = og * tanhf(cc[q]);
    }
    *(float4 *)cp = make_float4(cc[0], cc[1], cc[2], cc[3]);
    uint32_t hi[2], lo[2];
#pragma unroll
    for (int x = 0; x < 2; ++x) {
        const __nv_bfloat162 hv = __floats2bfloat162_rn(hh[2 * x], hh[2 * x + 1]);
        const __nv_bfloat162 lv = __floats2bfloat162_rn(hh[2 * x] - __low2float(hv), hh[2 * x + 1] - __high2float(hv));
        hi[x] = *(const uint32_t *)&hv;
        lo[x] = *(const uint32_t *)&lv;
    }
    const int64_t idx = (int64_t)m * de.next_ld + u0;
    *(uint2 *)(de.next + idx) = make_uint2(hi[0], hi[1]);
    *(uint2 *)(de.next + idx + de.next_plane) = make_uint2(lo[0], lo[1]);
}

// Prediction projection row of stream b (pred = bias + acc, n_split columns) and its joint input
// X[b] = relu(enc[er] + pred) as bf16 hi/lo planes.
__device__ __forceinline__ void dec_joint16(const NbDecEpi &de, int b, int n0, const float (&va)[16], const EpiIn &in) {
    const int N = de.n_split;
    float v[16], x[16];
#pragma unroll
    for (int q = 0; q < 16; q += 4) {
        const float4 b4 = in.a[q >> 2];
        const float4 e4 = in.b[q >> 2];
        v[q] = va[q] + b4.x; v[q + 1] = va[q + 1] + b4.y; v[q + 2] = va[q + 2] + b4.z; v[q + 3] = va[q + 3] + b4.w;
        x[q] = fmaxf(e4.x + v[q], 0.0f); x[q + 1] = fmaxf(e4.y + v[q + 1], 0.0f);
        x[q + 2] = fmaxf(e4.z + v[q + 2], 0.0f); x[q + 3] = fmaxf(e4.w + v[q + 3], 0.0f);
    }
    const int64_t idx = (int64_t)b * N + n0;
#pragma unroll
    for (int q = 0; q < 16; q += 4) *(float4 *)(de.pred + idx + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const __nv_bfloat162 hv = __floats2bfloat162_rn(x[2 * q], x[2 * q + 1]);
        const __nv_bfloat162 lv = __floats2bfloat162_rn(x[2 * q] - __low2float(hv), x[2 * q + 1] - __high2float(hv));
        hi[q] = *(const uint32_t *)&hv;
        lo[q] = *(const uint32_t *)&lv;
    }
    *(uint4 *)(de.X + idx) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *(uint4 *)(de.X + idx + 8) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    *(uint4 *)(de.X + idx + de.x_plane) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *(uint4 *)(de.X + idx + de.x_plane + 8) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
}

// Columns at or past n_split: the stream's aux row (product plus aux_bias).
__device__ __forceinline__ void dec_aux16(const NbDecEpi &de, int N, int b, int n0, const float (&va)[16], const EpiIn &in) {
    const int w = N - de.n_split, col = n0 - de.n_split;
    float *dst = de.aux + (int64_t)b * w + col;
#pragma unroll
    for (int q = 0; q < 16; q += 4) {
        const float4 b4 = in.a[q >> 2];
        *(float4 *)(dst + q) = make_float4(va[q] + b4.x, va[q + 1] + b4.y, va[q + 2] + b4.z, va[q + 3] + b4.w);
    }
}

// Requests the operands of the chunk at output column n0 (see EpiIn), with the same conditions
// under which the chunk's epilogue reads them; everything else is zero.
__device__ __forceinline__ void epi_in(const TcArgs &p, bool row_ok, int n0, int nout, int64_t rowbase, int64_t brow, int ds, int der,
                                       const float *dbias, EpiIn &in) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int x = 0; x < 4; ++x) in.a[x] = in.b[x] = z;
    in.c = z;
    if (!row_ok || n0 >= nout) return;
    const int cnt = min(16, nout - n0);
    if (p.de.mode == 3) {
#pragma unroll
        for (int x = 0; x < 16; ++x)
            if (x < cnt) set4(in.a[x >> 2], x & 3, __ldg(p.e.bias + n0 + x));
        return;
    }
    if (p.de.mode) {
        const NbDecEpi &de = p.de;
        if (n0 >= de.n_split) {
            if (de.aux_bias)
#pragma unroll
                for (int q = 0; q < 4; ++q) in.a[q] = __ldg((const float4 *)(de.aux_bias + (n0 - de.n_split) + 4 * q));
        } else if (de.mode == 1) {
#pragma unroll
            for (int q = 0; q < 4; ++q) in.a[q] = *(const float4 *)(dbias + n0 + 4 * q);
            in.c = *(const float4 *)(de.c + (int64_t)ds * (de.n_split >> 2) + (n0 >> 2));
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                in.a[q] = __ldg((const float4 *)(dbias + n0 + 4 * q));
                in.b[q] = *(const float4 *)(de.enc + (int64_t)der * de.n_split + n0 + 4 * q);
            }
        }
        return;
    }
    if (!p.vec || cnt != 16) return;  // the scalar path loads its own operands
    if (p.e.bias)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            in.a[q] = __ldg((const float4 *)(p.e.bias + brow + n0 + 4 * q));
            if (p.glu) in.b[q] = __ldg((const float4 *)(p.e.bias + brow + n0 + 4 * q + p.N / 2));
        }
    if (!p.glu && p.e.accumulate && p.e.c_fmt == NEMO_FMT_F32)
#pragma unroll
        for (int q = 0; q < 4; ++q) in.b[q] = *(const float4 *)((const float *)p.e.C + rowbase + n0 + 4 * q);
}

// DEC: the batched greedy decoder's epilogues (one tile per CTA, exposed): operands requested a
// full chunk ahead, in a second register set; otherwise each chunk's operands are requested at the
// end of the previous chunk (one register set, the register budget of the pipelined tile loop).
template <int BW, bool DEC>
__global__ void __launch_bounds__(THREADS, 1) gemm_tcr_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmAh,
                                                            const __grid_constant__ CUtensorMap tmAl, const __grid_constant__ TcArgs p) {
    using C = CfgR<BW>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *stages = smem;
    uint64_t *full = (uint64_t *)(smem + C::STAGES * C::STAGE);
    uint64_t *empty = full + C::STAGES;
    uint64_t *acc_full = empty + C::STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tmem_holder = (uint32_t *)(acc_empty + 2);
    volatile int *flags = (volatile int *)(tmem_holder + 1); // [0] abort, [1] last split of the unit, [2] epilogue abort

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // set-up first: with programmatic dependent launch it overlaps the previous kernel's tail
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { sm100::mbar_init(&full[s], 1); sm100::mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { sm100::mbar_init(&acc_full[b], 1); sm100::mbar_init(&acc_empty[b], 1); }
        flags[0] = 0;
        flags[2] = 0;
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
    nb::pdl_wait();  // inputs of the previous kernel are visible from here on
    const int M = p.dynM ? min(p.M, *p.dynM) : p.M;
    const int live_mtiles = (M + 127) / 128;
    const int tiles = live_mtiles * p.n_wtiles;            // output tiles that hold real rows

    if (warp == 0 && lane == 0) {
        // ---- producer: activation hi/lo tiles + weight tile (value and gate halves for GLU) ----
        int i = 0;
        PieceIter it(p, tiles);
        Piece w;
        while (!flags[0] && it.next(p, w)) {
            const int wt = w.tile % p.n_wtiles, mt = w.tile / p.n_wtiles;
            for (int kb = w.kb0; kb < w.kb1; ++kb, ++i) {
                const int s = i % C::STAGES;
                if (i >= C::STAGES && !sm100::mbar_wait(&empty[s], ((i / C::STAGES) - 1) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 5); break; }
                if (flags[0]) break;
                uint8_t *st = stages + s * C::STAGE;
                const int k0 = kb * BK;
                sm100::mbar_arrive_expect_tx(&full[s], C::STAGE);
                sm100::tma_load_2d(st, &tmAh, &full[s], k0, mt * 128);
                sm100::tma_load_2d(st + C::A_PLANE, &tmAl, &full[s], k0, mt * 128);
                if (p.glu) {
                    sm100::tma_load_2d(st + 2 * C::A_PLANE, &tmW, &full[s], k0, wt * (BW / 2));
                    sm100::tma_load_2d(st + 2 * C::A_PLANE + C::W_BYTES / 2, &tmW, &full[s], k0, p.N / 2 + wt * (BW / 2));
                } else {
                    sm100::tma_load_2d(st + 2 * C::A_PLANE, &tmW, &full[s], k0, wt * BW);
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        constexpr uint32_t idesc = sm100::idesc_bf16_f32(128, BW);
        int i = 0, t = 0;
        PieceIter it(p, tiles);
        Piece w;
        for (; !flags[0] && it.next(p, w); ++t) {
            const int kb0 = w.kb0, kb1 = w.kb1;
            const int b = t & 1;
            if (t >= 2 && !sm100::mbar_wait(&acc_empty[b], ((t >> 1) - 1) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 6); break; }
            sm100::tc_fence_after();
            const uint32_t dacc = tmem + (uint32_t)(b * C::ACC_STRIDE);
            for (int kb = kb0; kb < kb1; ++kb, ++i) {
                const int s = i % C::STAGES;
                if (!sm100::mbar_wait(&full[s], (i / C::STAGES) & 1)) { flags[0] = 1; atomicExch(&g_tc_error, 7); break; }
                sm100::tc_fence_after();
                const uint32_t h_addr = sm100::smem_u32(stages + s * C::STAGE);
                const uint32_t l_addr = h_addr + C::A_PLANE, w_addr = h_addr + 2 * C::A_PLANE;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t bd = sm100::desc_k_sw128(w_addr + kk * 32);
                    sm100::mma_bf16(dacc, sm100::desc_k_sw128(h_addr + kk * 32), bd, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                    sm100::mma_bf16(dacc, sm100::desc_k_sw128(l_addr + kk * 32), bd, idesc, 1u);
                }
                sm100::mma_commit(&empty[s]);
            }
            sm100::mma_commit(&acc_full[b]);
        }
    } else if (warp >= 2) {
        // ---- epilogue: thread = activation row, 16 output columns per TMEM load ----
        const int ew = warp - 2, q = warp & 3, half = ew >> 2;
        const int row = q * 32 + lane;
        const int etid = threadIdx.x - 64;
        const int nout = p.glu ? p.N / 2 : p.N;
        constexpr int OUT_COLS = BW;                 // output columns of a non-GLU tile
        const bool row_bias = p.e.bias && p.e.bias_gstride != 0;
        const int rowoff = p.rowoff ? *p.rowoff : 0;
        float *__restrict__ C32 = (float *)p.e.C;
        uint16_t *__restrict__ C16 = (uint16_t *)p.e.C;
        int t = 0;
        PieceIter it(p, tiles);
        Piece w;
        for (; it.next(p, w); ++t) {
            const int tile = w.tile, wt = tile % p.n_wtiles, mt = tile / p.n_wtiles;
            const int b = t & 1;
            const int m = mt * 128 + row;
            const bool row_ok = m < M;
            int64_t rowbase = 0, brow = 0;
            int ds = 0, der = 0;               // decoder epilogues: the row's stream and its encoder row
            const float *dbias = p.e.bias;     // decoder epilogues: bias row (or the stream's table row)
            if (row_ok) {
                const int g = m / p.e.rpg, r = m - g * p.e.rpg;
                rowbase = (int64_t)g * p.e.gstride + (int64_t)(rowoff + r) * p.e.ldc;
                brow = (int64_t)g * p.e.bias_gstride;
                if (p.de.mode == 1 || p.de.mode == 2) {
                    ds = p.de.need_idx[m];
                    if (p.de.mode == 1) dbias = p.de.row + (int64_t)(p.de.last_token ? p.de.last_token[ds] : ds) * p.de.n_split;
                    if (p.de.mode == 2) der = p.de.erow[ds];
                }
            }
            // columns of this thread: GLU -> value cols [half*BW/4, +BW/4) and their gates at +BW/2;
            // plain -> [half*BW/2, +BW/2)
            // (a 112-column tile splits 64 + 48, so every chunk starts on a 16-column boundary)
            const int hs = p.glu ? BW / 4 : (BW / 2 + 15) / 16 * 16;
            const int span = p.glu ? BW / 4 : half ? BW - hs : hs;
            const int j0 = half * hs;
            const int n_base = p.glu ? wt * (BW / 2) : wt * OUT_COLS;
            // the first chunk's operands, in flight while the MMAs finish
            EpiIn cur;
            epi_in(p, row_ok, n_base + j0, nout, rowbase, brow, ds, der, dbias, cur);
            if (!sm100::mbar_wait(&acc_full[b], (t >> 1) & 1)) { flags[2] = 1; flags[0] = 1; atomicExch(&g_tc_error, 8); }
            sm100::named_barrier(1, 256);
            const bool ok = !flags[2];
            sm100::tc_fence_after();
            const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * C::ACC_STRIDE);
            float *wsb = p.ws + (int64_t)tile * p.slots * 128 * BW;
            bool finish = ok;
            if (ok && w.parts > 1) {
                // partial tile [slot][row][BW] (all TMEM columns, value and gate alike)
                for (int j = half * (BW / 2); j < (half + 1) * (BW / 2); j += 16) {
                    float v[16];
                    sm100::tmem_ld16(tacc + j, v);
                    float4 *dst = (float4 *)(wsb + ((int64_t)w.slot * 128 + row) * BW + j);
#pragma unroll
                    for (int x = 0; x < 4; ++x) dst[x] = make_float4(v[4 * x], v[4 * x + 1], v[4 * x + 2], v[4 * x + 3]);
                }
                __threadfence();
                sm100::named_barrier(1, 256);
                if (etid == 0) flags[1] = atomicAdd(&p.counters[tile], 1) == w.parts - 1;
                sm100::named_barrier(1, 256);
                finish = flags[1];
                if (finish) __threadfence();
            }
            if (finish) {
                float amax = -INFINITY;  // mode 3: this thread's best column (ascending, strict >: lowest index on ties)
                int aidx = 0x7fffffff;
                for (int jj0 = j0; jj0 < j0 + span; jj0 += 16) {
                    float va[16], vg[16];
                    if (w.parts == 1) {
                        sm100::tmem_ld16(tacc + jj0, va);
                        if (p.glu) sm100::tmem_ld16(tacc + BW / 2 + jj0, vg);
                    } else {
#pragma unroll
                        for (int x = 0; x < 16; ++x) va[x] = vg[x] = 0.0f;
                        if (row_ok)
                            for (int s = 0; s < w.parts; ++s) {
                                const float *src = wsb + ((int64_t)s * 128 + row) * BW;
#pragma unroll
                                for (int x = 0; x < 16; x += 4) {
                                    const float4 a4 = __ldcg((const float4 *)(src + jj0 + x));
                                    va[x] += a4.x; va[x + 1] += a4.y; va[x + 2] += a4.z; va[x + 3] += a4.w;
                                    if (p.glu) {
                                        const float4 g4 = __ldcg((const float4 *)(src + BW / 2 + jj0 + x));
                                        vg[x] += g4.x; vg[x + 1] += g4.y; vg[x + 2] += g4.z; vg[x + 3] += g4.w;
                                    }
                                }
                            }
                    }
                    // decoder epilogues: the next chunk's operands, in flight during this chunk's math
                    EpiIn nxt;
                    if (DEC) epi_in(p, row_ok && jj0 + 16 < j0 + span, n_base + jj0 + 16, nout, rowbase, brow, ds, der, dbias, nxt);
                    const int n0 = n_base + jj0;
                    if (row_ok && n0 < nout) {
                        const int cnt = min(16, nout - n0);
                        if (p.de.mode == 3) {
#pragma unroll
                            for (int x = 0; x < 16; ++x) {
                                if (x >= cnt) break;
                                const float4 b4 = cur.a[x >> 2];
                                const float v = va[x] + ((x & 3) == 0 ? b4.x : (x & 3) == 1 ? b4.y : (x & 3) == 2 ? b4.z : b4.w);
                                if (v > amax) { amax = v; aidx = n0 + x; }
                            }
                        } else if (p.de.mode) {
                            if (n0 >= p.de.n_split) dec_aux16(p.de, p.N, ds, n0, va, cur);
                            else if (p.de.mode == 1) dec_lstm16(p.de, m, ds, n0, va, cur);
                            else dec_joint16(p.de, ds, n0, va, cur);
                        } else if (p.vec && cnt == 16) {
                            // 16-byte accesses (alignment of every pointer and stride checked on the
                            // host), the activation / output format resolved at compile time
                            const int mode = (p.glu ? 3 : p.e.act) | (p.e.c_fmt == NEMO_FMT_F32 ? 0 : 4);
                            switch (mode) {
                            case 0: epi16<0, false>(p, rowbase, m, n0, va, vg, cur); break;
                            case 1: epi16<1, false>(p, rowbase, m, n0, va, vg, cur); break;
                            case 2: epi16<2, false>(p, rowbase, m, n0, va, vg, cur); break;
                            case 3: epi16<3, false>(p, rowbase, m, n0, va, vg, cur); break;
                            case 4: epi16<0, true>(p, rowbase, m, n0, va, vg, cur); break;
                            case 5: epi16<1, true>(p, rowbase, m, n0, va, vg, cur); break;
                            case 6: epi16<2, true>(p, rowbase, m, n0, va, vg, cur); break;
                            default: epi16<3, true>(p, rowbase, m, n0, va, vg, cur); break;
                            }
                        } else {
                            float cin[16], bv[16], bg[16];
#pragma unroll
                            for (int x = 0; x < 16; ++x) {
                                cin[x] = bv[x] = bg[x] = 0.0f;
                                if (x < cnt) {
                                    if (p.e.accumulate) cin[x] = C32[rowbase + n0 + x];
                                    if (p.e.bias) {
                                        bv[x] = p.e.bias[brow + n0 + x];
                                        if (p.glu) bg[x] = p.e.bias[brow + n0 + x + p.N / 2];
                                    }
                                }
                            }
#pragma unroll
                            for (int x = 0; x < 16; ++x) {
                                if (x >= cnt) break;
                                float v;
                                if (p.glu) {
                                    v = (va[x] + bv[x]) * fast_sigmoid(vg[x] + bg[x]) * p.e.alpha;
                                } else {
                                    v = va[x] + bv[x];
                                    if (p.e.act == NEMO_ACT_SILU) v = v * fast_sigmoid(v);
                                    else if (p.e.act == NEMO_ACT_RELU) v = fmaxf(v, 0.0f);
                                    v *= p.e.alpha;
                                }
                                v += cin[x];
                                const int64_t idx = rowbase + n0 + x;
                                if (p.e.c_fmt == NEMO_FMT_F32) {
                                    C32[idx] = v;
                                } else {
                                    const uint16_t hi = nb::f2bf(v);
                                    C16[idx] = hi;
                                    C16[idx + p.e.c_plane] = nb::f2bf(v - nb::bf2f(hi));
                                }
                                if (p.e.c32) p.e.c32[(int64_t)m * p.e.ldc32 + n0 + x] = v;
                            }
                        }
                    }
                    if (DEC) cur = nxt;
                    else epi_in(p, row_ok && jj0 + 16 < j0 + span, n_base + jj0 + 16, nout, rowbase, brow, ds, der, dbias, cur);
                }
                if (p.de.mode == 3 && row_ok) {
                    p.de.part_v[(int64_t)m * p.de.part_ld + 2 * wt + half] = amax;
                    p.de.part_i[(int64_t)m * p.de.part_ld + 2 * wt + half] = aidx;
                }
                if (w.parts > 1 && etid == 0) p.counters[tile] = 0;
            }
            sm100::tc_fence_before();
            sm100::named_barrier(1, 256);
            if (etid == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm100::smem_u32(&acc_empty[b])) : "memory");
            if (!ok) break;
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
    cudaFuncSetAttribute(gemm_tcr_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<128>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<256, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<256>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<128>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<256, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<256>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<224, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<224>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<224, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<224>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<208, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<208>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<208, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<208>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<80, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<80>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<80, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<80>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<160, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<160>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<160, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<160>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<112, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<112>::SMEM);
    cudaFuncSetAttribute(gemm_tcr_kernel<112, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgR<112>::SMEM);
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
    p.units = tiles * p.splits;
    p.dynM = a->dynM;
    p.rowoff = a->rowoff;
    p.e = nb::make_epi(a);
    p.ws = g_ws;
    p.counters = g_counters;
    const int grid = p.units < g_sms ? p.units : g_sms;
    nb::launch(gemm_tc_kernel<BN>, grid, THREADS, Cfg<BN>::SMEM, st, mw, mh, ml, p);
    return nb_check_launch("gemm_tc_kernel");
}

// Plan of an activation-major launch: BW weight rows per tile and the k-split. The estimate is
// fitted to measured launches on a B200 (shapes of this model, 64..14336 rows): a round of
// units costs ~0.27 us per k-block per 128 weight rows plus ~4 us of pipeline fill and
// epilogue, and a k-split adds ~6 us (partial tiles through L2, reduced by the tile's last CTA),
// so splits are only planned for long K (>= 32 k-blocks) over few tiles.
struct PlanR {
    int bw, tiles, splits, kb_per_split, units;
    int sk_q, slots, grid;  // stream-K share per CTA (0: k-split units), partial slots per tile, CTAs
    float est_us;
};

PlanR plan_r(const nemo_gemm_args_t *a, int bw, bool allow_split) {
    PlanR r;
    const bool glu = a->act == NEMO_ACT_GLU;
    const int kblocks = (a->K + BK - 1) / BK;
    const int n_wtiles = glu ? (a->N / 2) / (bw / 2) : (a->N + bw - 1) / bw;
    r.bw = bw;
    r.tiles = n_wtiles * ((a->M + 127) / 128);
    int splits = 1;
    if (allow_split && kblocks >= 32 && 2 * r.tiles < g_sms) {
        splits = g_sms / r.tiles;
        if (splits > kblocks / 16) splits = kblocks / 16;  // at least 16 k-blocks per split
        if (splits < 1) splits = 1;
        if ((size_t)r.tiles * splits * 128 * bw > g_ws_floats || r.tiles > g_ncounters) splits = 1;
    }
    r.kb_per_split = (kblocks + splits - 1) / splits;
    r.splits = (kblocks + r.kb_per_split - 1) / r.kb_per_split;
    r.units = r.tiles * r.splits;
    r.sk_q = 0;
    r.slots = r.splits;
    r.grid = r.units < g_sms ? r.units : g_sms;
    const int rounds = (r.units + g_sms - 1) / g_sms;
    r.est_us = rounds * (0.27f * ((float)bw / 128.0f) * r.kb_per_split + 4.0f) + (r.splits > 1 ? 6.0f : 0.0f);
    return r;
}

// Stream-K plan: every CTA gets an equal share q of the tiles' k-blocks, so no SM idles through
// a last, partly filled round of tiles; tiles cut between CTAs are summed through partial slots
// by the last of their pieces to finish. Needs a row count known at launch (no dynM). ok = 0
// when the partial slots would not fit the workspace.
PlanR plan_sk(const nemo_gemm_args_t *a, int bw, int *ok) {
    PlanR r = plan_r(a, bw, false);
    const int kb = (a->K + BK - 1) / BK, total = r.tiles * kb;
    const int q = (total + g_sms - 1) / g_sms;
    int parts = 1;
    for (int t = 0; t < r.tiles; ++t) {
        const int n = (t * kb + kb - 1) / q - (t * kb) / q + 1;
        parts = n > parts ? n : parts;
    }
    *ok = !a->dynM && (size_t)r.tiles * parts * 128 * bw <= g_ws_floats && r.tiles <= g_ncounters;
    r.sk_q = q;
    r.slots = parts;
    r.grid = (total + q - 1) / q;
    r.est_us = 0.27f * (bw / 128) * q + 4.0f + (parts > 1 ? 14.0f : 0.0f);
    return r;
}

// Stream-K is planned only on request (NEMO_GEMM_SK=1, or layout 3): measured on a B200 at this
// model's shapes (64..3584 rows) it was 1.1-2.4x slower than the best k-split plan, the partial
// tiles' round trip (store, fence, arrival, reload) costing more than the idle SMs it saves.
int sk_policy() {
    static int v = -2;
    if (v == -2) {
        const char *e = getenv("NEMO_GEMM_SK");
        v = e && atoi(e) == 1 ? 1 : 0;
    }
    return v;
}

// 16-byte epilogue accesses: every row start, plane offset and bias row of the output must keep
// a 16-column chunk on a 16-byte boundary.
int vec_ok(const nemo_gemm_args_t *a) {
    const bool f32 = a->c_fmt == NEMO_FMT_F32;
    const int64_t q = f32 ? 4 : 8;  // elements per 16 bytes
    const uintptr_t c = (uintptr_t)a->C;
    if (c & 15) return 0;
    if (a->ldc % q || a->gstride % q || (!f32 && a->c_plane % 8)) return 0;
    if (a->accumulate && !f32) return 0;
    if (a->bias && (((uintptr_t)a->bias & 15) || a->bias_gstride % 4 || (a->act == NEMO_ACT_GLU && (a->N / 2) % 4))) return 0;
    if (a->c32 && (((uintptr_t)a->c32 & 15) || a->ldc32 % 4)) return 0;
    return 1;
}

template <int BW>
int launch_r(const nemo_gemm_args_t *a, const PlanR &pl, cudaStream_t st, const NbDecEpi *de) {
    CUtensorMap mw, mh, ml;
    const bool glu = a->act == NEMO_ACT_GLU;
    if (make_map(&mw, a->W, a->K, a->N, a->ldw, glu ? BW / 2 : BW)) return -1;
    const uint16_t *A = (const uint16_t *)a->A;
    if (make_map(&mh, A, a->K, a->M, a->lda, 128) || make_map(&ml, A + a->a_plane, a->K, a->M, a->lda, 128)) return -1;
    TcArgs p;
    memset(&p, 0, sizeof p);
    p.M = a->M; p.N = a->N; p.K = a->K;
    p.kblocks = (a->K + BK - 1) / BK;
    p.glu = glu;
    p.n_wtiles = glu ? (a->N / 2) / (BW / 2) : (a->N + BW - 1) / BW;
    p.n_mtiles = (a->M + 127) / 128;
    p.splits = pl.splits;
    p.kb_per_split = pl.kb_per_split;
    p.units = pl.units;
    p.dynM = a->dynM;
    p.rowoff = a->rowoff;
    p.e = nb::make_epi(a);
    p.ws = g_ws;
    p.counters = g_counters;
    p.vec = vec_ok(a);
    if (de) p.de = *de;
    p.sk_q = pl.sk_q;
    p.slots = pl.slots;
    const int grid = pl.grid;
    // the widths other than 128 and 256: no k-splits (their partial tiles are laid out by halves
    // of BW / 2 columns) and no GLU (value and gate halves of BW / 4 columns per thread half)
    if (BW != 128 && BW != 256 && (pl.splits > 1 || pl.sk_q || glu)) return nb_set_error("tensor-core GEMM: %d-row tiles take unsplit plain GEMMs only", BW);
    if (de) nb::launch(gemm_tcr_kernel<BW, true>, grid, THREADS, CfgR<BW>::SMEM, st, mw, mh, ml, p);
    else nb::launch(gemm_tcr_kernel<BW, false>, grid, THREADS, CfgR<BW>::SMEM, st, mw, mh, ml, p);
    return nb_check_launch("gemm_tcr_kernel");
}

// sched: 0 = best estimate, 1 = k-split units only, 2 = stream-K (when the shape allows it)
int launch_rows(const nemo_gemm_args_t *a, cudaStream_t st, const NbDecEpi *de = nullptr, int sched = 0) {
    const bool glu = a->act == NEMO_ACT_GLU;
    const bool ok256 = !glu || (a->N / 2) % 128 == 0;
    PlanR best = plan_r(a, 128, false);
    // (224-row tiles without k-splits: with them the 1024 x 4096 FF-out shape measured 38 us per
    // CTA against 31 us with unsplit 128-row tiles)
    const PlanR cand[7] = { plan_r(a, 256, false), plan_r(a, 128, true), plan_r(a, 256, true), plan_r(a, 224, false), plan_r(a, 208, false), plan_r(a, 160, false),
                            plan_r(a, 112, false) };
    const int pol = sched == 1 ? 0 : sched == 2 ? 1 : sk_policy();
    if (pol != 1)
        for (const PlanR &p : cand) {
            const bool fits = p.bw == 128 || (p.bw == 256 && ok256) || ((p.bw == 224 || p.bw == 208 || p.bw == 160 || p.bw == 112) && !glu);
            if (fits && p.est_us < best.est_us) best = p;
        }
    if (pol != 0) {
        int ok128 = 0, ok2 = 0;
        const PlanR s128 = plan_sk(a, 128, &ok128), s256 = plan_sk(a, 256, &ok2);
        if (pol == 1 && ok128) best = s128;
        if (ok128 && s128.est_us < best.est_us) best = s128;
        if (ok2 && ok256 && s256.est_us < best.est_us) best = s256;
    }
    if (best.bw == 256) return launch_r<256>(a, best, st, de);
    if (best.bw == 224) return launch_r<224>(a, best, st, de);
    if (best.bw == 208) return launch_r<208>(a, best, st, de);
    if (best.bw == 160) return launch_r<160>(a, best, st, de);
    if (best.bw == 112) return launch_r<112>(a, best, st, de);
    return launch_r<128>(a, best, st, de);
}

}  // namespace

// One-time setup (driver entry point, split-K workspace): call before capturing a CUDA graph.
extern "C" int nb_gemm_tc_init(void) { return init_once(); }

// layout: 0 = by row count, 1 = weight-major tiles, 2 = activation-major tiles, 3 = activation-major
// tiles scheduled stream-K (falls back to the planner when the shape does not allow it)
int nb_gemm_tc_layout(const nemo_gemm_args_t *a, int layout, void *stream) {
    if (init_once()) return -1;
    if (a->act == NEMO_ACT_GLU && ((a->N / 2) % 64)) return nb_set_error("tensor-core GEMM: GLU needs N/2 to be a multiple of 64");
    if (a->K % 8) return nb_set_error("tensor-core GEMM: K must be a multiple of 8");
    cudaStream_t st = (cudaStream_t)stream;
    // activation-major above 32 rows (measured faster at 64 and more); up to 32 rows the weights
    // must stream through every SM with split-K, which the weight-major tiles do
    if (layout == 0) layout = a->M > 32 ? 2 : 1;
    if (layout == 2) return launch_rows(a, st);
    if (layout == 3) return launch_rows(a, st, nullptr, 2);
    if (a->M <= 16) return launch<16>(a, st);
    if (a->M <= 32) return launch<32>(a, st);
    if (a->M <= 64) return launch<64>(a, st);
    return launch<128>(a, st);
}

int nb_gemm_tc(const nemo_gemm_args_t *a, void *stream) { return nb_gemm_tc_layout(a, 0, stream); }

// Column-tile width of the joint GEMM with the argmax epilogue: 80 (faster, see below) while its
// partials (two per tile) fit the step kernel's one-warp reduction, else 128.
static int dec_joint_bw(int n) { return 2 * ((n + 79) / 80) <= 32 ? 80 : 128; }
extern "C" int nb_dec_joint_parts(int n) {
    const int bw = dec_joint_bw(n);
    return 2 * ((n + bw - 1) / bw);
}

extern "C" int nb_gemm_dec(const nemo_gemm_args_t *a, const NbDecEpi *de, void *stream) {
    if (init_once()) return -1;
    if (!de || de->mode < 1 || de->mode > 3) return nb_set_error("decoder GEMM: unknown epilogue mode");
    if (de->mode == 3) {
        // rows are streams (no row list); partials per (column tile, half): nb_dec_joint_parts(N) <= part_ld
        const int bw = dec_joint_bw(a->N);
        if (a->a_fmt != NEMO_FMT_BF16X2 || a->act != NEMO_ACT_NONE || a->accumulate || a->K % 8 || !a->bias || !de->part_v || !de->part_i ||
            de->part_ld < nb_dec_joint_parts(a->N) || a->dynM)
            return nb_set_error("decoder GEMM: argmax epilogue needs bf16 hi/lo activations, a bias, partial buffers of %d columns", nb_dec_joint_parts(a->N));
        if (bw == 80) return launch_r<80>(a, plan_r(a, 80, false), (cudaStream_t)stream, de);
        return launch_r<128>(a, plan_r(a, 128, false), (cudaStream_t)stream, de);
    }
    if (a->a_fmt != NEMO_FMT_BF16X2 || a->act != NEMO_ACT_NONE || a->accumulate || a->K % 8 || a->N % 16)
        return nb_set_error("decoder GEMM: needs bf16 hi/lo activations, no activation or accumulation, K %% 8 == 0 and N %% 16 == 0");
    const int ns = de->n_split;
    if (ns <= 0 || ns > a->N || ns % 16 || !de->need_idx || (ns < a->N && (!de->aux || ((uintptr_t)de->aux & 15) || ((uintptr_t)de->aux_bias & 15))))
        return nb_set_error("decoder GEMM: bad column split or aux output");
    if (de->mode == 1 && (!de->row || !de->c || !de->next || (((uintptr_t)de->row | (uintptr_t)de->c) & 15) || ((uintptr_t)de->next & 7) ||
                          de->next_ld % 4 || de->next_plane % 4))
        return nb_set_error("decoder GEMM: LSTM epilogue operands misaligned or missing");
    if (de->mode == 2 && (!a->bias || ((uintptr_t)a->bias & 15) || !de->enc || !de->erow || !de->pred || !de->X ||
                          (((uintptr_t)de->enc | (uintptr_t)de->pred | (uintptr_t)de->X) & 15) || de->x_plane % 8))
        return nb_set_error("decoder GEMM: joint epilogue operands misaligned or missing");
    // 80-row weight tiles: each CTA's time is its 128 rows of activation planes (K x 4 bytes per
    // row, the same for every width) plus its weight rows and an epilogue that grow with the width,
    // so more, narrower tiles finish sooner (256 streams, greedy decoder per config #4 step:
    // 4.39 / 3.94 / 3.47 / 3.15 / 3.12 / 2.93 / 2.83 ms with 256- / 208- / 160- / 128- / 112- /
    // 96- / 80-row tiles; 1024 streams: 8.57 ms with 112, 8.06 with 80)
    return launch_r<80>(a, plan_r(a, 80, false), (cudaStream_t)stream, de);
}

extern "C" int nb_attention_device_error(void);

// ---- bounded-wait self-test ---------------------------------------------------------------------
// One CTA (kind 0) or two (kind 1) wait on something nothing will ever complete, with a wait limit
// of `limit` clock cycles: kind 0 the mbarrier wait of the tensor-core kernels (an mbarrier that
// expects one arrival and gets none), kind 1 the grid barrier of the persistent kernels (a target
// one arrival above the grid). The wait gives up, records its code where the kernels record theirs
// and the kernel returns: nemo_gpu_check_device_errors then reports it.
__global__ void wait_selftest_kernel(int kind, long long limit, unsigned *bar) {
    __shared__ uint64_t mbar;
    if (kind == 0) {
        if (threadIdx.x == 0) {
            sm100::mbar_init(&mbar, 1);
            sm100::fence_mbar_init();
            if (!sm100::mbar_wait(&mbar, 0, limit)) atomicCAS(&g_tc_error, 0, 9);
        }
    } else {
        __syncthreads();
        if (threadIdx.x == 0) nb::grid_arrive_wait(bar, gridDim.x + 1, &g_tc_error, 10, limit);
        __syncthreads();
    }
}

extern "C" int nemo_gpu_wait_selftest(int kind, long long limit_cycles, void *stream) {
    if (kind != 0 && kind != 1) return nb_set_error("nemo_gpu_wait_selftest: kind %d (0 = mbarrier, 1 = grid barrier)", kind);
    if (limit_cycles < 1 || limit_cycles > 4000000000LL) return nb_set_error("nemo_gpu_wait_selftest: limit of %lld cycles", limit_cycles);
    static unsigned *bar[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nb_set_error("nemo_gpu_wait_selftest: no usable device");
    if (!bar[dev] && cudaMalloc((void **)&bar[dev], 2 * sizeof(unsigned)) != cudaSuccess) return nb_set_error("nemo_gpu_wait_selftest: out of memory");
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemsetAsync(bar[dev], 0, 2 * sizeof(unsigned), st) != cudaSuccess) return nb_set_error("nemo_gpu_wait_selftest: %s", cudaGetErrorString(cudaGetLastError()));
    wait_selftest_kernel<<<kind == 0 ? 1 : 2, 32, 0, st>>>(kind, limit_cycles, bar[dev]);
    return nb_check_launch("wait_selftest_kernel");
}

// Bumped each time a tensor-core wait failure is reported: split-K arrival counters may then have
// been left dirty, and the allocation-free entry clears its own again before its next launch.
static std::atomic<unsigned> g_tc_error_reports{0};

extern "C" int nemo_gpu_check_device_errors(void) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof v) != cudaSuccess) return nb_set_error("cannot read the device error flag");
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof z);  // reported once
        g_tc_error_reports.fetch_add(1);
        return nb_set_error("%s: a bounded device wait gave up (code %d)", v >= 9 ? "wait self-test" : "tensor-core GEMM", v);
    }
    const int a = nb_attention_device_error();
    if (a < 0) return nb_set_error("cannot read the attention error flag");
    if (a) return nb_set_error("attention: a bounded wait for the window's rows gave up");
    return 0;
}

// ---- allocation-free entry point -------------------------------------------------------------
// The same kernel and split-K plan as nb_gemm_tc for activation tiles of up to 32 rows (the
// single-stream and small-batch shapes, which are the ones that split K), with the partial tiles
// and arrival counters in a fixed array compiled into this module instead of the cudaMalloc'd
// workspace. It exists for hosts that must not allocate device memory once they are running: a
// real-time audio callback that drives one stream (cudaMalloc may synchronize the device and
// stall the callback), and servers that reserve their whole device-memory budget up front and
// refuse allocations afterwards.
//
// Limits: at most NA_MAX_ROWS activation rows; a plan that would need more partial-tile bytes
// or counters than the array holds is rejected with an error (with 148 SMs no shape of <= 32
// rows does). All calls on one device share the one array, so calls whose executions overlap
// (two streams, or two host threads without ordering) race on it and corrupt each other's sums:
// serialize them on one stream or order them with events.
//
// The first call on each device (with that device current) does the one-time set-up: the
// array's device address (cudaGetSymbolAddress), the kernels' shared-memory attribute, the
// driver's tensor-map encoder, and a blocking clear of the arrival counters. Make that first call
// before any stream capture. The kernel leaves every counter at zero when a tile finishes, so
// later calls do not clear them; only after nemo_gpu_check_device_errors has reported a failed
// wait (which can leave a counter dirty) does the next call clear them again, blocking.
constexpr int NA_MAX_ROWS = 32;
constexpr size_t NA_PART_BYTES = (size_t)5 << 20;  // split-K partial tiles: 5 MiB
constexpr int NA_COUNTERS = 1024;                  // one arrival counter per output tile
constexpr size_t NA_BYTES = NA_PART_BYTES + NA_COUNTERS * sizeof(int);
constexpr int NA_MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

namespace {

std::mutex g_na_mu;
EncodeTiled g_na_encode = nullptr;             // kept apart from g_encode, whose presence marks the workspace as allocated
unsigned char *g_na_ptr[NA_MAX_DEVICES] = {};  // device address of g_noalloc_scratch per device
int g_na_sms[NA_MAX_DEVICES] = {};
unsigned g_na_cleared[NA_MAX_DEVICES] = {};     // g_tc_error_reports when the counters were last cleared

int na_setup(unsigned char **scratch, int *sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nb_set_error("nemo_gemm_noalloc: no current CUDA device");
    if (dev < 0 || dev >= NA_MAX_DEVICES) return nb_set_error("nemo_gemm_noalloc: device %d beyond the %d supported", dev, NA_MAX_DEVICES);
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_ptr[dev]) {
        if (!g_na_encode) {
            void *fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
                return nb_set_error("nemo_gemm_noalloc: cuTensorMapEncodeTiled unavailable");
            g_na_encode = (EncodeTiled)fn;
        }
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return nb_set_error("nemo_gemm_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            return nb_set_error("nemo_gemm_noalloc: cannot read the SM count");
        if (cudaFuncSetAttribute(gemm_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<16>::SMEM) != cudaSuccess ||
            cudaFuncSetAttribute(gemm_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<32>::SMEM) != cudaSuccess)
            return nb_set_error("nemo_gemm_noalloc: cannot set the kernels' shared-memory size");
        if (cudaMemset((unsigned char *)p + NA_PART_BYTES, 0, NA_COUNTERS * sizeof(int)) != cudaSuccess)
            return nb_set_error("nemo_gemm_noalloc: cannot clear the arrival counters");
        g_na_sms[dev] = n;
        g_na_cleared[dev] = g_tc_error_reports.load();
        g_na_ptr[dev] = (unsigned char *)p;
    } else if (g_na_cleared[dev] != g_tc_error_reports.load()) {
        if (cudaMemset(g_na_ptr[dev] + NA_PART_BYTES, 0, NA_COUNTERS * sizeof(int)) != cudaSuccess)
            return nb_set_error("nemo_gemm_noalloc: cannot clear the arrival counters");
        g_na_cleared[dev] = g_tc_error_reports.load();
    }
    *scratch = g_na_ptr[dev];
    *sms = g_na_sms[dev];
    return 0;
}

int na_map(CUtensorMap *m, const void *base, int64_t cols, int64_t rows, int64_t ld_elems, int box_rows) {
    if (((uintptr_t)base & 15) || ((ld_elems * 2) & 15)) return nb_set_error("nemo_gemm_noalloc: base and row pitch must be 16-byte aligned");
    cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    cuuint64_t strides[1] = { (cuuint64_t)(ld_elems * 2) };
    cuuint32_t box[2] = { (cuuint32_t)BK, (cuuint32_t)box_rows };
    cuuint32_t es[2] = { 1, 1 };
    CUresult r = g_na_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return nb_set_error("nemo_gemm_noalloc: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

template <int BN>
int na_launch(const nemo_gemm_args_t *a, cudaStream_t st, unsigned char *scratch, int sms) {
    CUtensorMap mw, mh, ml;
    const bool glu = a->act == NEMO_ACT_GLU;
    if (na_map(&mw, a->W, a->K, a->N, a->ldw, glu ? 64 : BM)) return -1;
    const uint16_t *A = (const uint16_t *)a->A;
    if (na_map(&mh, A, a->K, a->M, a->lda, BN) || na_map(&ml, A + a->a_plane, a->K, a->M, a->lda, BN)) return -1;
    TcArgs p;
    memset(&p, 0, sizeof p);
    p.M = a->M; p.N = a->N; p.K = a->K;
    p.kblocks = (a->K + BK - 1) / BK;
    p.glu = glu;
    p.n_wtiles = glu ? (a->N / 2 + 63) / 64 : (a->N + BM - 1) / BM;
    p.n_mtiles = (a->M + BN - 1) / BN;
    const int tiles = p.n_wtiles * p.n_mtiles;
    int splits = 1;
    if (tiles < sms) {
        splits = (sms + tiles - 1) / tiles;
        if (splits > p.kblocks) splits = p.kblocks;
    }
    p.kb_per_split = (p.kblocks + splits - 1) / splits;
    p.splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split;
    p.units = tiles * p.splits;
    if (p.splits > 1) {
        const size_t need = (size_t)p.units * BN * BM * sizeof(float);
        if (need > NA_PART_BYTES || tiles > NA_COUNTERS)
            return nb_set_error("nemo_gemm_noalloc: this shape needs %zu bytes of split-K partials and %d counters; the static scratch holds %zu and %d",
                                need, tiles, NA_PART_BYTES, NA_COUNTERS);
    }
    p.dynM = a->dynM;
    p.rowoff = a->rowoff;
    p.e = nb::make_epi(a);
    p.ws = (float *)scratch;
    p.counters = (int *)(scratch + NA_PART_BYTES);
    const int grid = p.units < sms ? p.units : sms;
    nb::launch(gemm_tc_kernel<BN>, grid, THREADS, Cfg<BN>::SMEM, st, mw, mh, ml, p);
    return nb_check_launch("gemm_tc_kernel");
}

}  // namespace

extern "C" int nemo_gemm_noalloc(const nemo_gemm_args_t *a, void *stream) {
    // the checks nemo_gemm makes (null pointers, shape, GLU with an odd N, accumulate into a
    // non-fp32 output), then this entry's own limits
    if (nb_gemm_validate(a, "nemo_gemm_noalloc")) return -1;
    if (a->M == 0) return 0;
    if (a->M > NA_MAX_ROWS)
        return nb_set_error("nemo_gemm_noalloc: M=%d rows; the allocation-free GEMM takes 1..%d rows (its static scratch is sized for that)", a->M,
                            NA_MAX_ROWS);
    if (a->a_fmt != NEMO_FMT_BF16X2) return nb_set_error("nemo_gemm_noalloc: activations must be NEMO_FMT_BF16X2 planes");
    if (a->act == NEMO_ACT_GLU && ((a->N / 2) % 64)) return nb_set_error("nemo_gemm_noalloc: GLU needs N/2 to be a multiple of 64");
    if (a->K % 8) return nb_set_error("nemo_gemm_noalloc: K must be a multiple of 8");
    unsigned char *scratch = nullptr;
    int sms = 0;
    if (na_setup(&scratch, &sms)) return -1;
    cudaStream_t st = (cudaStream_t)stream;
    if (a->M <= 16) return na_launch<16>(a, st, scratch, sms);
    return na_launch<32>(a, st, scratch, sms);
}
