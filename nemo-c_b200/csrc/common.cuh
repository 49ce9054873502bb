// Shared device helpers for the sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/nemo_gpu.h"

namespace nb {

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf2f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// round-to-nearest-even fp32 -> bf16 bits (inputs here are finite)
__device__ __forceinline__ uint16_t f2bf(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Metal-equivalent activations (src/kernels.metal:6-7), IEEE expf / division
__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }
__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// Store one activation either as fp32 or as a bf16 hi/lo pair (hi + lo == v to ~2^-17 relative).
__device__ __forceinline__ void store_act(void *base, int fmt, int64_t plane, int64_t idx, float v) {
    if (fmt == NEMO_FMT_F32) {
        ((float *)base)[idx] = v;
    } else {
        const uint16_t hi = f2bf(v);
        const uint16_t lo = f2bf(v - bf2f(hi));
        ((uint16_t *)base)[idx] = hi;
        ((uint16_t *)base)[idx + plane] = lo;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Butterfly of V values per lane over the warp (V a power of two, 2 <= V <= 128): at the step with
// lane offset O each lane keeps the half of its values selected by (lane & O) and adds its
// partner's copy of that half; once one value is left the remaining steps add it plainly. After it,
// lane l holds in x[j] (j < max(V / 32, 1)) the warp's total of value l * V / 32 + j (V >= 32) or,
// in x[0], of value l >> (5 - log2 V) (V < 32: l >> 1 for 16 values). (Templates, so that every
// index is a constant and the values stay in registers.)
template <int N, int O>
struct WarpFold {
    static __device__ __forceinline__ void run(float *x, int lane) {
        if constexpr (O > 0) {
            if constexpr (N > 1) {
                constexpr int H = N / 2;
                const bool up = (lane & O) != 0;
#pragma unroll
                for (int j = 0; j < H; ++j) {
                    const float send = up ? x[j] : x[j + H];
                    const float keep = up ? x[j + H] : x[j];
                    x[j] = keep + __shfl_xor_sync(0xffffffffu, send, O);
                }
                WarpFold<H, O / 2>::run(x, lane);
            } else {
                x[0] += __shfl_xor_sync(0xffffffffu, x[0], O);
                WarpFold<1, O / 2>::run(x, lane);
            }
        }
    }
};
template <int V>
__device__ __forceinline__ void warp_fold(float (&x)[V]) { WarpFold<V, 16>::run(x, threadIdx.x & 31); }

// Block-wide sum for blockDim.x == NT (multiple of 32); red must hold NT/32 floats.
template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) t += red[i];
    return t;
}

// Wait for the previous kernel in the stream when launched with programmatic dependent launch
// (a no-op otherwise: the launch itself waited), then let the next kernel be scheduled: it runs
// its own set-up on free SMs and blocks in its pdl_wait() until this grid has completed and its
// writes are visible. A grid is released only once all of its CTAs are resident, so waiting
// grids never keep their predecessor's CTAs from running.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
}
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

}  // namespace nb

// host side
extern "C" int nb_set_error(const char *fmt, ...);
extern "C" int nb_pdl_enabled(void);
extern "C" int nb_smem_attr(const void *func, size_t bytes);

namespace nb {
// Launch with programmatic dependent launch: the grid may be scheduled while its predecessor in
// the stream (or captured graph) drains, hiding the launch gap between dependent kernels. Every
// kernel launched this way calls pdl_wait() before its first global memory access, so it still
// sees all of the predecessor's writes and its writes never race the predecessor's reads.
// NEMO_PDL=0 launches plainly.
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = nb_pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}
}  // namespace nb
extern "C" void nb_count_launches(uint64_t n);
int nb_check_launch(const char *what);
