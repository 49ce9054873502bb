// GEMM epilogue shared by the CUDA-core and tensor-core GEMM kernels.
#pragma once
#include "common.cuh"

namespace nb {

struct Epi {
    const float *bias;
    int64_t bias_gstride;
    void *C;
    int64_t ldc, c_plane, gstride;
    int c_fmt, rpg, act, accumulate;
    float alpha;
    float *c32;      // optional fp32 copy of a bf16x2 output: c32[m * ldc32 + n]
    int64_t ldc32;
};

// Epilogue order bias -> act -> *alpha -> store/accumulate (src/kernels.metal:39-44, 106-114);
// GLU takes a * sigmoid(b) (src/kernels.metal:96-104). Row m of the GEMM goes to group
// g = m / rpg, row rowoff + m % rpg of that group.
__device__ __forceinline__ void epilogue(const Epi &e, int rowoff, int m, int n, int nb, float va, float vb) {
    const int g = m / e.rpg, r = m - g * e.rpg;
    const float *bias = e.bias ? e.bias + (int64_t)g * e.bias_gstride : nullptr;
    float v;
    if (e.act == NEMO_ACT_GLU) {
        if (bias) { va += bias[n]; vb += bias[nb]; }
        v = va * sigmoid_f(vb) * e.alpha;
    } else {
        v = va + (bias ? bias[n] : 0.0f);
        if (e.act == NEMO_ACT_SILU) v = silu_f(v);
        else if (e.act == NEMO_ACT_RELU) v = fmaxf(v, 0.0f);
        v *= e.alpha;
    }
    const int64_t idx = (int64_t)g * e.gstride + (int64_t)(rowoff + r) * e.ldc + n;
    if (e.accumulate) v += ((const float *)e.C)[idx];
    store_act(e.C, e.c_fmt, e.c_plane, idx, v);
    if (e.c32) e.c32[(int64_t)m * e.ldc32 + n] = v;
}

inline Epi make_epi(const nemo_gemm_args_t *a) {
    Epi e;
    e.bias = a->bias;
    e.bias_gstride = a->bias_gstride;
    e.C = a->C;
    e.ldc = a->ldc;
    e.c_plane = a->c_plane;
    e.gstride = a->gstride;
    e.c_fmt = a->c_fmt;
    e.rpg = a->rpg > 0 ? a->rpg : (a->M > 0 ? a->M : 1);
    e.act = a->act;
    e.accumulate = a->accumulate;
    e.alpha = a->alpha;
    e.c32 = a->c32;
    e.ldc32 = a->ldc32;
    return e;
}

}  // namespace nb
