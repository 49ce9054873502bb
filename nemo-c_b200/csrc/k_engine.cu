// Kernels private to the streaming engine: per-epoch cache compaction (src/encoder.c:201-211)
// and the batched greedy RNNT loop bookkeeping (src/decoder.c:92-127), one frame per stream per
// iteration, every stream advancing independently.
#include "common.cuh"
#include "engine_dev.h"

namespace {

// Move kv rows [src_kv, src_kv + cache_len) to [0, cache_len) and din rows
// [src_din, src_din + conv_left) to [dst_din, dst_din + conv_left), every layer and stream.
// Source and destination never overlap (cap_rows >= 2 * att_left + cmax).
__global__ void compact_kernel(float *kv, float *din, int layers, int streams, int64_t cap, int D, int src_kv, int cache_len, int src_din,
                               int dst_din, int conv_left) {
    nb::pdl_wait();
    const int64_t kv_row = 3LL * D, per_kv = (int64_t)cache_len * kv_row, per_din = (int64_t)conv_left * D;
    const int64_t total = (int64_t)layers * streams * (per_kv + per_din);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ls = i / (per_kv + per_din), r = i - ls * (per_kv + per_din);
        if (r < per_kv) {
            float *base = kv + ls * cap * kv_row;
            base[r] = base[(int64_t)src_kv * kv_row + r];
        } else {
            const int64_t q = r - per_kv;
            float *base = din + ls * cap * D;
            base[(int64_t)dst_din * D + q] = base[(int64_t)src_din * D + q];
        }
    }
}

__global__ void dec_chunk_init_kernel(DecState d, int streams, int c) {
    nb::pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b == 0) { d.cnt[2] = 0; d.cnt[3] = 0; } // iterations run, blocks of dec_update done
    if (b >= streams) return;
    d.t[b] = 0;
    d.symbols[b] = 0;
    d.active[b] = c > 0;
    d.ntok[b] = 0;
}

// Streams that still have frames and whose prediction vector is stale get the prediction
// network this iteration (src/decoder.c:101); every active stream scores its current frame.
__global__ void dec_plan_kernel(DecState d, int streams, int c) {
    nb::pdl_wait();
    __shared__ int n_need;
    if (threadIdx.x == 0) n_need = 0;
    __syncthreads();
    for (int b = threadIdx.x; b < streams; b += blockDim.x) {
        const bool act = d.active[b];
        d.erow[b] = act ? b * c + d.t[b] : -1;
        int pos = -1;
        if (act && !d.pred_valid[b]) {
            pos = atomicAdd(&n_need, 1);
            d.need_idx[pos] = b;
        }
        d.need_pos[b] = pos;
    }
    __syncthreads();
    if (threadIdx.x == 0) { d.cnt[0] = n_need; d.cnt[1] = 0; }
}

// Prediction-network input for each listed stream: [embed(last token) (zeros for blank) | h0]
// for layer 0 and [. | h1] for layer 1 (src/decoder.c:61-70).
__global__ void dec_gather_kernel(DecState d, const uint16_t *__restrict__ embed, int PH, int blank) {
    nb::pdl_wait();
    const int i = blockIdx.x;
    if (i >= d.cnt[0]) return;
    const int b = d.need_idx[i];
    const int tok = d.last_token[b];
    const float *h0 = d.h + (int64_t)b * PH, *h1 = d.h + ((int64_t)d.streams + b) * PH;
    const int64_t r0 = (int64_t)i * 2 * PH;
    for (int j = threadIdx.x; j < PH; j += blockDim.x) {
        nb::store_act(d.A0, d.fmt, d.a_plane, r0 + j, tok == blank ? 0.0f : nb::bf2f(embed[(int64_t)tok * PH + j]));
        nb::store_act(d.A0, d.fmt, d.a_plane, r0 + PH + j, h0[j]);
        nb::store_act(d.A1, d.fmt, d.a_plane, r0 + PH + j, h1[j]);
    }
}

// LSTM cell (src/kernels.metal:475-486) from the committed cell state into the provisional
// state of each listed stream; h' also goes to `next` (the following GEMM's input row).
__global__ void dec_cell_kernel(DecState d, int layer, int PH, float *next, int64_t next_ld, int64_t next_plane) {
    nb::pdl_wait();
    const int i = blockIdx.x;
    if (i >= d.cnt[0]) return;
    const int b = d.need_idx[i];
    const float *g = d.gates + (int64_t)i * 4 * PH;
    const int64_t sb = ((int64_t)layer * d.streams + b) * PH;
    for (int j = threadIdx.x; j < PH; j += blockDim.x) {
        const float ig = nb::sigmoid_f(g[j]), fg = nb::sigmoid_f(g[PH + j]), gg = tanhf(g[2 * PH + j]), og = nb::sigmoid_f(g[3 * PH + j]);
        const float cc = fg * d.c[sb + j] + ig * gg;
        const float hh = og * tanhf(cc);
        d.cp[sb + j] = cc;
        d.hp[sb + j] = hh;
        nb::store_act(next, d.fmt, next_plane, (int64_t)i * next_ld + j, hh);
    }
}

__global__ void dec_scatter_pred_kernel(DecState d, int JH) {
    nb::pdl_wait();
    const int i = blockIdx.x;
    if (i >= d.cnt[0]) return;
    const int b = d.need_idx[i];
    for (int j = threadIdx.x; j < JH; j += blockDim.x) d.pred[(int64_t)b * JH + j] = d.predc[(int64_t)i * JH + j];
    if (threadIdx.x == 0) d.pred_valid[b] = 1;
}

// One decision per active stream (src/decoder.c:106-121): blank -> next frame, symbols = 0;
// token -> emit, commit the provisional LSTM state, re-score the same frame unless max_symbols
// tokens came from it.
// One greedy step per active stream (src/decoder.c:104-122). When the decoder runs as a CUDA
// graph WHILE loop (cond != 0), the last block to finish sets the loop condition: another
// iteration while some stream still has frames, at most max_it iterations per chunk.
// With logits: the decision is the argmax of the stream's row (ties to the lowest index,
// src/kernels.metal:521-550), taken here by warp 0; without, it was left in d.idx.
__global__ void dec_update_kernel(DecState d, int c, int PH, int blank, int max_symbols, int max_it, cudaGraphConditionalHandle cond,
                                  const float *__restrict__ logits, int64_t ldl, int V) {
    nb::pdl_wait();
    __shared__ int s_k;
    const int b = blockIdx.x;
    const bool live = d.active[b];
    if (threadIdx.x < 32) {
        int k0 = blank;
        if (live) {
            if (logits) {
                const float *l = logits + (int64_t)b * ldl;
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int n = threadIdx.x; n < V; n += 32) {
                    const float v = l[n];
                    if (v > bv) { bv = v; bi = n; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                }
                k0 = bi;
            } else {
                k0 = d.idx[b];
            }
        }
        if (threadIdx.x == 0) {
            s_k = k0;
            if (live) d.idx[b] = k0;
        }
    }
    __syncthreads();
    const int k = s_k;
    if (live && k != blank) {
        for (int l = 0; l < 2; ++l) {
            const int64_t sb = ((int64_t)l * d.streams + b) * PH;
            for (int j = threadIdx.x; j < PH; j += blockDim.x) { d.h[sb + j] = d.hp[sb + j]; d.c[sb + j] = d.cp[sb + j]; }
        }
    }
    if (threadIdx.x != 0) return;
    if (live) {
        int t = d.t[b], sym = d.symbols[b];
        if (k == blank) {
            sym = 0;
            ++t;
        } else {
            if (d.ntok[b] < d.tok_cap) d.tokens[(int64_t)b * d.tok_cap + d.ntok[b]] = k;
            d.ntok[b]++;
            d.last_token[b] = k;
            d.pred_valid[b] = 0;
            if (++sym >= max_symbols) { sym = 0; ++t; }
        }
        d.t[b] = t;
        d.symbols[b] = sym;
        const int act = t < c;
        d.active[b] = act;
        if (act) atomicAdd(&d.cnt[1], 1);
    }
    if (cond) {
        __threadfence();
        if (atomicAdd(&d.cnt[3], 1) == (int)gridDim.x - 1) {
            __threadfence();
            const int it = d.cnt[2] + 1;
            d.cnt[2] = it;
            d.cnt[3] = 0;
            cudaGraphSetConditional(cond, (atomicAdd(&d.cnt[1], 0) > 0 && it < max_it) ? 1u : 0u);
        }
    }
}

__global__ void dec_joint_in_kernel(DecState d, const float *__restrict__ enc, int JH, uint16_t *X, int64_t plane) {
    nb::pdl_wait();
    const int b = blockIdx.x;
    const int er = d.erow[b], pos = d.need_pos[b];
    const float *p = pos >= 0 ? d.predc + (int64_t)pos * JH : d.pred + (int64_t)b * JH;
    const float *e = enc + (int64_t)(er < 0 ? 0 : er) * JH;
    for (int i = threadIdx.x; i < JH; i += blockDim.x) {
        const float pv = p[i];
        if (pos >= 0) d.pred[(int64_t)b * JH + i] = pv;
        nb::store_act(X, NEMO_FMT_BF16X2, plane, (int64_t)b * JH + i, er < 0 ? 0.0f : fmaxf(e[i] + pv, 0.0f));
    }
    if (threadIdx.x == 0 && pos >= 0) d.pred_valid[b] = 1;
}

__global__ void dec_reset_kernel(DecState d, int PH, int blank) {
    nb::pdl_wait();
    const int b = blockIdx.x;
    for (int l = 0; l < 2; ++l) {
        const int64_t sb = ((int64_t)l * d.streams + b) * PH;
        for (int j = threadIdx.x; j < PH; j += blockDim.x) d.h[sb + j] = d.c[sb + j] = 0.0f;
    }
    if (threadIdx.x == 0) { d.last_token[b] = blank; d.pred_valid[b] = 0; d.active[b] = 0; d.ntok[b] = 0; }
}

}  // namespace

extern "C" int nb_compact(float *kv, float *din, int layers, int streams, int64_t cap, int D, int src_kv, int cache_len, int src_din, int dst_din,
                          int conv_left, void *stream) {
    nb::launch(compact_kernel, 148 * 8, 256, 0, (cudaStream_t)stream, kv, din, layers, streams, cap, D, src_kv, cache_len, src_din, dst_din, conv_left);
    return nb_check_launch("compact_kernel");
}
extern "C" int nb_dec_chunk_init(const DecState *d, int c, void *stream) {
    nb::launch(dec_chunk_init_kernel, (d->streams + 255) / 256, 256, 0, (cudaStream_t)stream, *d, d->streams, c);
    return nb_check_launch("dec_chunk_init_kernel");
}
extern "C" int nb_dec_plan(const DecState *d, int c, void *stream) {
    nb::launch(dec_plan_kernel, 1, 1024, 0, (cudaStream_t)stream, *d, d->streams, c);
    return nb_check_launch("dec_plan_kernel");
}
extern "C" int nb_dec_gather(const DecState *d, const uint16_t *embed, int PH, int blank, void *stream) {
    nb::launch(dec_gather_kernel, d->streams, 128, 0, (cudaStream_t)stream, *d, embed, PH, blank);
    return nb_check_launch("dec_gather_kernel");
}
extern "C" int nb_dec_cell(const DecState *d, int layer, int PH, float *next, int64_t next_ld, int64_t next_plane, void *stream) {
    nb::launch(dec_cell_kernel, d->streams, 128, 0, (cudaStream_t)stream, *d, layer, PH, next, next_ld, next_plane);
    return nb_check_launch("dec_cell_kernel");
}
extern "C" int nb_dec_scatter_pred(const DecState *d, int JH, void *stream) {
    nb::launch(dec_scatter_pred_kernel, d->streams, 128, 0, (cudaStream_t)stream, *d, JH);
    return nb_check_launch("dec_scatter_pred_kernel");
}
extern "C" int nb_dec_update(const DecState *d, int c, int PH, int blank, int max_symbols, int max_it, unsigned long long cond, const float *logits,
                             int64_t ldl, int V, void *stream) {
    nb::launch(dec_update_kernel, d->streams, 128, 0, (cudaStream_t)stream, *d, c, PH, blank, max_symbols, max_it, (cudaGraphConditionalHandle)cond, logits,
                                                                   ldl, V);
    return nb_check_launch("dec_update_kernel");
}
extern "C" int nb_dec_joint_in(const DecState *d, const float *enc, int JH, uint16_t *X, int64_t plane, void *stream) {
    nb::launch(dec_joint_in_kernel, d->streams, 128, 0, (cudaStream_t)stream, *d, enc, JH, X, plane);
    return nb_check_launch("dec_joint_in_kernel");
}
extern "C" int nb_dec_reset(const DecState *d, int PH, int blank, void *stream) {
    nb::launch(dec_reset_kernel, d->streams, 128, 0, (cudaStream_t)stream, *d, PH, blank);
    return nb_check_launch("dec_reset_kernel");
}
