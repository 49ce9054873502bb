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
        if (d.stats) {
            if (k != blank && sym == 0) atomicAdd(&d.stats[0], 1);
            atomicAdd(&d.stats[1], 1);
        }
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

// ---- fused batched greedy decoder -------------------------------------------------------------

constexpr int STEP_T = 160;  // threads of the per-stream kernels: 4 consecutive units / elements each for 640-wide rows

__device__ __forceinline__ float4 ld4(const float *p) { return *(const float4 *)p; }

// bf16 hi/lo planes of 4 consecutive values (idx a multiple of 4, plane a multiple of 4)
__device__ __forceinline__ void put4_planes(uint16_t *base, int64_t plane, int64_t idx, float4 v) {
    const uint16_t h0 = nb::f2bf(v.x), h1 = nb::f2bf(v.y), h2 = nb::f2bf(v.z), h3 = nb::f2bf(v.w);
    const uint16_t l0 = nb::f2bf(v.x - nb::bf2f(h0)), l1 = nb::f2bf(v.y - nb::bf2f(h1)), l2 = nb::f2bf(v.z - nb::bf2f(h2)), l3 = nb::f2bf(v.w - nb::bf2f(h3));
    *(uint2 *)(base + idx) = make_uint2((uint32_t)h0 | ((uint32_t)h1 << 16), (uint32_t)h2 | ((uint32_t)h3 << 16));
    *(uint2 *)(base + idx + plane) = make_uint2((uint32_t)l0 | ((uint32_t)l1 << 16), (uint32_t)l2 | ((uint32_t)l3 << 16));
}

__device__ __forceinline__ float4 relu_add4(float4 a, float4 b) {
    return make_float4(fmaxf(a.x + b.x, 0.0f), fmaxf(a.y + b.y, 0.0f), fmaxf(a.z + b.z, 0.0f), fmaxf(a.w + b.w, 0.0f));
}

// One LSTM unit (src/kernels.metal:475-486) from its gates i, f, g, o and cell state.
__device__ __forceinline__ float lstm_unit(float gi, float gf, float gg, float go, float &c) {
    const float ig = nb::sigmoid_f(gi), fg = nb::sigmoid_f(gf), g = tanhf(gg), og = nb::sigmoid_f(go);
    c = fg * c + ig * g;
    return og * tanhf(c);
}

// The next iteration's work of stream b. Listed (pos >= 0: it emitted, its prediction is stale):
// layer 0 of the prediction network, gates = T[token] + R0[b] (gate-interleaved), its cell state
// updated and h0' written to G1 input row pos. Otherwise, while active: its joint input row
// relu(enc[er] + pred[b]). The element loads are issued before the first store.
__device__ __forceinline__ void stream_rows(const DecState &d, const NbDecStep &s, int b, int tok, int pos, bool act, int er) {
    const int tid = threadIdx.x;
    if (pos >= 0) {
        const float *tr = s.T + (int64_t)tok * 4 * s.PH, *rr = s.R0 + (int64_t)b * 4 * s.PH;
        float *c0 = s.c0 + (int64_t)b * s.PH;
        for (int u = tid * 4; u < s.PH; u += STEP_T * 4) {
            float4 t[4], r[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) { t[q] = ld4(tr + 4 * u + 4 * q); r[q] = ld4(rr + 4 * u + 4 * q); }
            float4 c = ld4(c0 + u), h;
            h.x = lstm_unit(t[0].x + r[0].x, t[0].y + r[0].y, t[0].z + r[0].z, t[0].w + r[0].w, c.x);
            h.y = lstm_unit(t[1].x + r[1].x, t[1].y + r[1].y, t[1].z + r[1].z, t[1].w + r[1].w, c.y);
            h.z = lstm_unit(t[2].x + r[2].x, t[2].y + r[2].y, t[2].z + r[2].z, t[2].w + r[2].w, c.z);
            h.w = lstm_unit(t[3].x + r[3].x, t[3].y + r[3].y, t[3].z + r[3].z, t[3].w + r[3].w, c.w);
            *(float4 *)(c0 + u) = c;
            put4_planes(s.A, s.a_plane, (int64_t)pos * s.a_ld + u, h);
        }
    } else if (act) {
        const float *p = d.pred + (int64_t)b * s.JH, *e = s.enc + (int64_t)er * s.JH;
        for (int j = tid * 4; j < s.JH; j += STEP_T * 4) put4_planes(s.X, s.x_plane, (int64_t)b * s.JH + j, relu_add4(ld4(e + j), ld4(p + j)));
    }
}

// stream_rows for rows of exactly 4 * STEP_T units / columns, with the decision-independent
// operands (the recurrent gate part, the cell state, the kept prediction and the next frame's
// encoder row) loaded before the decision was known.
struct StreamPre {
    float4 r[4], c, p, e;
};
__device__ __forceinline__ void stream_pre_load(const DecState &d, const NbDecStep &s, int b, int er_next, StreamPre &P) {
    const int u = threadIdx.x * 4;
    const float *rr = s.R0 + (int64_t)b * 4 * s.PH + 4 * u;
#pragma unroll
    for (int q = 0; q < 4; ++q) P.r[q] = ld4(rr + 4 * q);
    P.c = ld4(s.c0 + (int64_t)b * s.PH + u);
    P.p = ld4(d.pred + (int64_t)b * s.JH + u);
    P.e = ld4(s.enc + (int64_t)er_next * s.JH + u);
}
__device__ __forceinline__ void stream_rows_pre(const NbDecStep &s, int b, int tok, int pos, bool act, const StreamPre &P) {
    const int u = threadIdx.x * 4;
    if (pos >= 0) {
        const float *tr = s.T + (int64_t)tok * 4 * s.PH + 4 * u;
        float4 t[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) t[q] = ld4(tr + 4 * q);
        float4 c = P.c, h;
        h.x = lstm_unit(t[0].x + P.r[0].x, t[0].y + P.r[0].y, t[0].z + P.r[0].z, t[0].w + P.r[0].w, c.x);
        h.y = lstm_unit(t[1].x + P.r[1].x, t[1].y + P.r[1].y, t[1].z + P.r[1].z, t[1].w + P.r[1].w, c.y);
        h.z = lstm_unit(t[2].x + P.r[2].x, t[2].y + P.r[2].y, t[2].z + P.r[2].z, t[2].w + P.r[2].w, c.z);
        h.w = lstm_unit(t[3].x + P.r[3].x, t[3].y + P.r[3].y, t[3].z + P.r[3].z, t[3].w + P.r[3].w, c.w);
        *(float4 *)(s.c0 + (int64_t)b * s.PH + u) = c;
        put4_planes(s.A, s.a_plane, (int64_t)pos * s.a_ld + u, h);
    } else if (act) {
        put4_planes(s.X, s.x_plane, (int64_t)b * s.JH + u, relu_add4(P.e, P.p));
    }
}

// Counts of this kernel's blocks: listed streams accumulate in cnt[4], active ones in cnt[6]; the
// last block to finish publishes them as cnt[0] / cnt[1] and clears the accumulators.
__device__ __forceinline__ void publish(const DecState &d, bool first, int max_it, cudaGraphConditionalHandle cond) {
    __threadfence();
    if (atomicAdd(&d.cnt[3], 1) != (int)gridDim.x - 1) return;
    __threadfence();
    const int n_need = atomicExch(&d.cnt[4], 0), n_act = atomicExch(&d.cnt[6], 0);
    d.cnt[0] = n_need;
    d.cnt[1] = n_act;
    d.cnt[3] = 0;
    const int it = first ? 0 : d.cnt[2] + 1;
    d.cnt[2] = it;
    if (cond) cudaGraphSetConditional(cond, (n_act > 0 && it < max_it) ? 1u : 0u);
}

__global__ void __launch_bounds__(STEP_T) dec_chunk_start_kernel(DecState d, NbDecStep s, int c) {
    nb::pdl_wait();
    __shared__ int s_pos;
    const int b = blockIdx.x;
    const bool act = c > 0;
    const bool need = act && !d.pred_valid[b];
    const int tok = d.last_token[b];
    if (threadIdx.x == 0) {
        s_pos = need ? atomicAdd(&d.cnt[4], 1) : -1;
        d.t[b] = 0;
        d.symbols[b] = 0;
        d.active[b] = act;
        d.ntok[b] = 0;
        d.erow[b] = act ? b * c : -1;
        d.need_pos[b] = s_pos;
        if (need) d.need_idx[s_pos] = b;
        if (act) atomicAdd(&d.cnt[6], 1);
    }
    __syncthreads();
    stream_rows(d, s, b, (tok >= 0 && tok < s.V) ? tok : s.blank, s_pos, act, b * c);
    if (threadIdx.x == 0) publish(d, true, 0, 0);
}

// One greedy step per active stream (src/decoder.c:104-122) from its logits row: argmax with ties
// to the lowest index (src/kernels.metal:521-550); blank -> next frame; token -> emit (its
// provisional LSTM state becomes the committed one), re-score the same frame unless max_symbols
// tokens came from it. Then the stream's work for the next iteration (stream_rows).
__global__ void __launch_bounds__(STEP_T) dec_step_kernel(DecState d, NbDecStep s, int c, int max_it, cudaGraphConditionalHandle cond) {
    nb::pdl_wait();
    __shared__ float rv[STEP_T / 32];
    __shared__ int ri[STEP_T / 32];
    __shared__ int s_k, s_pos;
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const bool live = d.active[b] != 0;
    if (!live) {
        if (tid == 0) {
            d.erow[b] = -1;
            d.need_pos[b] = -1;
            publish(d, false, max_it, cond);
        }
        return;
    }
    int t = d.t[b], sym = d.symbols[b];
    // the decision-independent operands of the next iteration, in flight during the argmax
    const bool pre = s.PH == 4 * STEP_T && s.JH == 4 * STEP_T;
    StreamPre P;
    if (pre) stream_pre_load(d, s, b, b * c + min(t + 1, c - 1), P);
    if (s.part_v) {
        // the joint GEMM left (value, column) partials per column tile: reduce them, ties to the
        // lowest column
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        if (tid < s.nparts) {
            bv = s.part_v[(int64_t)b * s.nparts + tid];
            bi = s.part_i[(int64_t)b * s.nparts + tid];
        }
        if (tid < 32) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (tid == 0) s_k = bi;
        }
        __syncthreads();
    } else {
        const float *l = s.logits + (int64_t)b * s.ldl;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll 2
        for (int n = tid * 4; n < s.V; n += STEP_T * 4) {
            const float4 v = ld4(l + n);  // the row pitch is a multiple of 4 floats
            // ascending indices within a thread: strict > keeps the lowest index of equal values
            if (v.x > bv) { bv = v.x; bi = n; }
            if (n + 1 < s.V && v.y > bv) { bv = v.y; bi = n + 1; }
            if (n + 2 < s.V && v.z > bv) { bv = v.z; bi = n + 2; }
            if (n + 3 < s.V && v.w > bv) { bv = v.w; bi = n + 3; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { rv[w] = bv; ri[w] = bi; }
        __syncthreads();
        if (tid == 0) {
            for (int i = 1; i < STEP_T / 32; ++i)
                if (rv[i] > bv || (rv[i] == bv && ri[i] < bi)) { bv = rv[i]; bi = ri[i]; }
            s_k = bi;
        }
        __syncthreads();
    }
    // an index outside the vocabulary (only if every logit were NaN) is taken as blank, so no
    // table row beyond the vocabulary is ever read
    const int k = (s_k >= 0 && s_k < s.V) ? s_k : s.blank;
    const bool emit = k != s.blank;
    if (tid == 0 && d.stats) {
        if (emit && sym == 0) atomicAdd(&d.stats[0], 1);
        atomicAdd(&d.stats[1], 1);
    }
    if (!emit) {
        sym = 0;
        ++t;
    } else if (++sym >= s.max_symbols) {
        sym = 0;
        ++t;
    }
    const bool act = t < c;
    const bool need = emit && act;
    if (tid == 0) {
        s_pos = need ? atomicAdd(&d.cnt[4], 1) : -1;
        d.idx[b] = k;
        if (emit) {
            if (d.ntok[b] < d.tok_cap) d.tokens[(int64_t)b * d.tok_cap + d.ntok[b]] = k;
            d.ntok[b]++;
            d.last_token[b] = k;
        }
        d.t[b] = t;
        d.symbols[b] = sym;
        d.active[b] = act;
        d.pred_valid[b] = !emit;
        d.erow[b] = act ? b * c + t : -1;
        d.need_pos[b] = s_pos;
        if (need) d.need_idx[s_pos] = b;
        if (act) atomicAdd(&d.cnt[6], 1);
    }
    __syncthreads();
    if (pre) stream_rows_pre(s, b, k, s_pos, act, P);
    else stream_rows(d, s, b, k, s_pos, act, b * c + t);
    if (tid == 0) publish(d, false, max_it, cond);
}

// Recurrent gate parts of a zero state: R0[b] = 0, R1[b] = b1 (both [streams][W]).
__global__ void dec_rows_init_kernel(float *R0, float *R1, const float *__restrict__ b1, int W) {
    nb::pdl_wait();
    const int b = blockIdx.x;
    for (int n = threadIdx.x; n < W; n += blockDim.x) {
        R0[(int64_t)b * W + n] = 0.0f;
        R1[(int64_t)b * W + n] = b1[n];
    }
}

// Gate-interleaved copy: row 4u + g of Wi is row g * PH + u of W.
__global__ void interleave_gates_kernel(const uint16_t *__restrict__ W, uint16_t *Wi, const float *__restrict__ bias, float *bi, int PH, int K) {
    nb::pdl_wait();
    const int r = blockIdx.x, u = r >> 2, g = r & 3;
    const int64_t src = (int64_t)g * PH + u;
    for (int k = threadIdx.x; k < K; k += blockDim.x) Wi[(int64_t)r * K + k] = W[src * K + k];
    if (bias && threadIdx.x == 0) bi[r] = bias[src];
}

__global__ void gate_table_kernel(const uint16_t *__restrict__ Wi, int64_t ldw, const uint16_t *__restrict__ embed, int PH, const float *__restrict__ bi,
                                  int blank, float *table, int N) {
    nb::pdl_wait();
    const int v = blockIdx.y, n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float acc = 0.0f;
    if (v != blank)
        for (int k = 0; k < PH; ++k) acc = fmaf(nb::bf2f(Wi[(int64_t)n * ldw + k]), nb::bf2f(embed[(int64_t)v * PH + k]), acc);
    table[(int64_t)v * N + n] = acc + bi[n];
}

__global__ void dec_reset_kernel(DecState d, int PH, int blank) {
    nb::pdl_wait();
    const int b = blockIdx.x;
    if (b == 0 && threadIdx.x < 8) d.cnt[threadIdx.x] = 0;
    if (b == 0 && threadIdx.x < 2 && d.stats) d.stats[threadIdx.x] = 0;
    for (int l = 0; l < 2; ++l) {
        const int64_t sb = ((int64_t)l * d.streams + b) * PH;
        for (int j = threadIdx.x; j < PH; j += blockDim.x) d.h[sb + j] = d.c[sb + j] = 0.0f;
    }
    if (threadIdx.x == 0) { d.last_token[b] = blank; d.pred_valid[b] = 0; d.active[b] = 0; d.ntok[b] = 0; }
}

}  // namespace

// The same with one block per (layer, stream): both moves are contiguous runs of whole rows, copied
// as float4 (every row start is 16-byte aligned when D % 4 == 0).
__global__ void __launch_bounds__(256) compact_rows_kernel(float *kv, float *din, int64_t cap, int D, int src_kv, int cache_len, int src_din, int dst_din,
                                                           int conv_left) {
    nb::pdl_wait();
    const int64_t ls = blockIdx.x, kv_row = 3LL * D;
    float4 *kd = (float4 *)(kv + ls * cap * kv_row);
    const float4 *ks = (const float4 *)(kv + ls * cap * kv_row + (int64_t)src_kv * kv_row);
    const int64_t nkv = (int64_t)cache_len * kv_row / 4;
    for (int64_t i = threadIdx.x; i < nkv; i += blockDim.x) kd[i] = ks[i];
    float4 *dd = (float4 *)(din + ls * cap * D + (int64_t)dst_din * D);
    const float4 *ds = (const float4 *)(din + ls * cap * D + (int64_t)src_din * D);
    const int64_t ndin = (int64_t)conv_left * D / 4;
    for (int64_t i = threadIdx.x; i < ndin; i += blockDim.x) dd[i] = ds[i];
}

extern "C" int nb_compact(float *kv, float *din, int layers, int streams, int64_t cap, int D, int src_kv, int cache_len, int src_din, int dst_din,
                          int conv_left, void *stream) {
    if (D % 4 == 0 && ((uintptr_t)kv & 15) == 0 && ((uintptr_t)din & 15) == 0 && (int64_t)layers * streams <= 0x7fffffff) {
        nb::launch(compact_rows_kernel, (unsigned)(layers * streams), 256, 0, (cudaStream_t)stream, kv, din, cap, D, src_kv, cache_len, src_din, dst_din,
                   conv_left);
        return nb_check_launch("compact_rows_kernel");
    }
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
extern "C" int nb_dec_chunk_start(const DecState *d, const NbDecStep *s, int c, void *stream) {
    nb::launch(dec_chunk_start_kernel, d->streams, STEP_T, 0, (cudaStream_t)stream, *d, *s, c);
    return nb_check_launch("dec_chunk_start_kernel");
}
extern "C" int nb_dec_step(const DecState *d, const NbDecStep *s, int c, int max_it, unsigned long long cond, void *stream) {
    nb::launch(dec_step_kernel, d->streams, STEP_T, 0, (cudaStream_t)stream, *d, *s, c, max_it, (cudaGraphConditionalHandle)cond);
    return nb_check_launch("dec_step_kernel");
}
extern "C" int nb_dec_interleave(const uint16_t *W, uint16_t *Wi, const float *bias, float *bi, int PH, int K, void *stream) {
    nb::launch(interleave_gates_kernel, 4 * PH, 256, 0, (cudaStream_t)stream, W, Wi, bias, bi, PH, K);
    return nb_check_launch("interleave_gates_kernel");
}
extern "C" int nb_dec_gate_table(const uint16_t *Wi, int64_t ldw, const uint16_t *embed, int V, int PH, const float *bi, int blank, float *table,
                                 void *stream) {
    const int N = 4 * PH;
    nb::launch(gate_table_kernel, dim3((N + 255) / 256, V), 256, 0, (cudaStream_t)stream, Wi, ldw, embed, PH, bi, blank, table, N);
    return nb_check_launch("gate_table_kernel");
}
extern "C" int nb_dec_rows_init(float *R0, float *R1, const float *b1, int streams, int W, void *stream) {
    nb::launch(dec_rows_init_kernel, streams, 256, 0, (cudaStream_t)stream, R0, R1, b1, W);
    return nb_check_launch("dec_rows_init_kernel");
}
