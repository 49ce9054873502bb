/* nemo_gpu: C-ABI of the B200 kernels (sm_100a). Plain pointers and sizes; device pointers
   unless stated; `stream` is a cudaStream_t (NULL = legacy default stream). Every entry point
   returns 0 on success or -1 after recording a message retrievable with nemo_gpu_last_error().

   These replace the reference's string-keyed Metal dispatch (src/gpu.h:20-41, src/gpu.m) and the
   kernel launchers of src/model.h:71-76 plus the direct dispatches in src/encoder.c and
   src/decoder.c. The math of each entry point is that of the Metal kernel it cites.

   Devices: a process drives one GPU through these entry points (nemo_gemm's split-K workspace is
   allocated once, on the device current at its first call). Per-kernel shared-memory limits are
   kept per device, and nemo_gemm_noalloc keeps its set-up per device. */
#ifndef NEMO_GPU_H
#define NEMO_GPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { NEMO_ACT_NONE = 0, NEMO_ACT_SILU = 1, NEMO_ACT_RELU = 2, NEMO_ACT_GLU = 3 };
enum { NEMO_FMT_F32 = 0, NEMO_FMT_BF16X2 = 1 };

/* C[row(m)][n] (= or +=) alpha * act(sum_k A[m][k] * W[n][k] + bias[g][n]).
   Replaces k_gemm (src/model.h:71, src/model.c:70-99) and its kernels gemm_bf16 / gemm_spec /
   gemm_mma (src/kernels.metal:12-208); like k_gemm it picks the kernel by row count:
   M <= 16 streams the weights through CUDA cores; larger M runs tcgen05 tensor-core tiles.
   Row mapping (new: lets one launch cover many streams and write into per-stream caches):
   m -> group g = m / rpg, r = m % rpg; C element at C + g*gstride + (rowoff + r)*ldc + n,
   bias at bias + g*bias_gstride + n. rowoff is read from device memory (NULL = 0).
   A formats: NEMO_FMT_F32 (fp32 [M][lda]) or NEMO_FMT_BF16X2 (two bf16 planes, hi at A and
   lo = A - hi at A + a_plane elements; hi + lo carries 16 mantissa bits). The C output may
   also be written as NEMO_FMT_BF16X2 planes (c_plane apart) for a following tensor-core GEMM. */
typedef struct {
    const void *A;
    int64_t lda, a_plane;
    int a_fmt;
    const uint16_t *W;
    int64_t ldw;
    const float *bias;
    int64_t bias_gstride;
    void *C;
    int64_t ldc, c_plane;
    int c_fmt;
    int rpg;
    int64_t gstride;
    const int *rowoff;
    const int *dynM; /* if non-NULL: rows actually processed = min(M, *dynM), read on the device */
    int M, N, K;
    int act, accumulate;
    float alpha;
    float *c32;      /* optional: also write the fp32 value at c32[m * ldc32 + n] (dense rows) */
    int64_t ldc32;
} nemo_gemm_args_t;
int nemo_gemm(const nemo_gemm_args_t *a, void *stream);
/* Force a kernel family for tests and the kernel sweep: 0 = by row count (default),
   1 = CUDA-core weight streaming, 2 = tcgen05 tensor cores (tile layout by row count),
   3 = CUDA-core tiled, 4 = tensor cores with weight-major tiles (weights on the MMA's 128-row
   side), 5 = tensor cores with activation-major tiles (128 activation rows x 128/256 weights),
   6 = activation-major tiles scheduled stream-K (every CTA an equal share of the k-blocks of all
   tiles; kind 5's plan when the row count is dynamic). */
int nemo_gemm_forced(const nemo_gemm_args_t *a, int kind, void *stream);
/* Allocation-free tensor-core GEMM (no counterpart in the reference, whose Metal GEMMs need no
   split-K scratch). Same arguments and results as nemo_gemm for NEMO_FMT_BF16X2 activations of
   1..32 rows; its split-K scratch is a fixed 5 MiB array inside the library, so it never
   allocates device memory. For hosts that cannot allocate once running: a real-time audio
   callback driving one stream (cudaMalloc may synchronize the device) and servers that reserve
   their device memory up front. It makes nemo_gemm's checks (null pointers, shape, GLU with an
   odd N, accumulate into a non-fp32 output; M = 0 does nothing) and returns -1 with
   nemo_gpu_last_error() set for more rows, other activation formats, or a plan that would exceed
   the scratch. The first call on each device (that device current) does the set-up, including a
   blocking clear of the split-K arrival counters; make it before any stream capture. Later calls
   clear nothing (the kernel leaves the counters at zero) unless nemo_gpu_check_device_errors has
   reported a failed device wait since, in which case the next call clears them again, blocking.
   Calls on one device share the scratch: calls that overlap in time race and must be serialized
   on one stream. */
int nemo_gemm_noalloc(const nemo_gemm_args_t *a, void *stream);

/* Row LayerNorm. Replaces k_layernorm (src/model.h:73; kernel src/kernels.metal:258-288).
   Y may be written as NEMO_FMT_BF16X2 planes (y_plane apart) for a tensor-core consumer. */
int nemo_layernorm(const float *X, const float *g, const float *b, void *Y, int y_fmt, int64_t y_plane,
                   int M, int D, float eps, void *stream);
/* Y1 = LN(X; g1, b1), Y2 = LN(Y1; g2, b2). Replaces k_layernorm2 (src/model.h:72; kernel
   src/kernels.metal:212-255). Y1 is fp32; Y2 may be BF16X2 planes. */
int nemo_layernorm2(const float *X, const float *g1, const float *b1, const float *g2, const float *b2,
                    float *Y1, void *Y2, int y2_fmt, int64_t y2_plane, int M, int D, float eps, void *stream);

/* Relative-position attention over a K/V cache window for `streams` independent streams.
   Replaces the attention_rel dispatch (src/encoder.c:161-165; kernel src/kernels.metal:293-348).
   Per stream s: queries are rows [*pos, *pos + c) of Q + s*q_sstride ([.][ldq]); keys/values
   rows [*pos - *cache_len, *pos + c) of K + s*kv_sstride / V + s*kv_sstride ([.][ldk]), so
   L = *cache_len + c (<= Lmax); pos and cache_len are read from device ints. P: [2*Lmax-1][D] position table. Output
   O + s*o_sstride ([c][D]) as fp32 or BF16X2 planes (o_plane apart). Limits: head dim 128, c <= 16,
   Lmax <= 96; Q, K, V, P, bias_u and bias_v 16-byte aligned; ldq, ldk, q_sstride, kv_sstride and D
   multiples of 4 floats (an error otherwise). */
int nemo_attention_rel(const float *Q, int64_t ldq, int64_t q_sstride, const float *K, const float *V, int64_t ldk,
                       int64_t kv_sstride, const int *pos, const int *cache_len, const float *P, const float *bias_u,
                       const float *bias_v, void *O, int o_fmt, int64_t o_plane, int64_t o_sstride,
                       int streams, int c, int Lmax, int H, int dh, int D, float scale, void *stream);

/* Causal depthwise conv (taps rows, history in place) + LayerNorm + SiLU, `streams` streams.
   Replaces the dwconv_ln_silu dispatch (src/encoder.c:172-174; kernel src/kernels.metal:361-409).
   din rows for stream s start at din + s*din_sstride + (*pos - (taps-1))*D. */
int nemo_dwconv_ln_silu(const float *din, int64_t din_sstride, const int *pos, const float *W, const float *g,
                        const float *b, void *Y, int y_fmt, int64_t y_plane, int streams, int c, int D, int taps,
                        float eps, void *stream);

/* 1 -> C channel 3x3 stride-2 conv + ReLU, causal padding, `streams` windows of [T][F] each
   (x_sstride apart). Replaces conv2d_c1_s2_relu (src/kernels.metal:413-432). Y: [s][T1][F1][C]. */
int nemo_conv2d_c1_s2_relu(const float *X, int64_t x_sstride, const float *W, const float *bias, float *Y,
                           int streams, int T, int F, int T1, int F1, int C, void *stream);
/* The first two subsampling stages in one pass: conv2d_c1_s2_relu followed by dwconv2d_s2
   (src/encoder.c:125-130), without the intermediate [T1][F1][C] map. X: `streams` windows of
   [T][F] (x_sstride apart); Y: [s][T2][F2][C] as fp32 or bf16 planes (y_plane apart). */
int nemo_subsample_front(const float *X, int64_t x_sstride, const float *W0, const float *b0, const float *W2, const float *b2, void *Y,
                         int y_fmt, int64_t y_plane, int streams, int T, int F, int C, void *stream);
/* Depthwise 3x3 stride-2 conv. Replaces dwconv2d_s2 (src/kernels.metal:435-454). X [s][T][F][C]. */
int nemo_dwconv2d_s2(const float *X, const float *W, const float *bias, float *Y, int streams, int T, int F,
                     int T1, int F1, int C, void *stream);
/* Gather rows [*lo, *lo + c) of each stream's [T][F][C] map and flatten them channel-major into
   [s*c][C*F] fp32 (flatten_cf, src/kernels.metal:457-462, restricted to the rows the chunk keeps
   at src/encoder.c:258). */
int nemo_flatten_rows(const float *X, float *Y, const int *lo, int streams, int T, int F, int C, int c, void *stream);

/* Log-mel frames (the transform of src/mel.c:115-173: Hann(400) centred in 512 points,
   double-precision FFT, power, 128 Slaney filters, log(x + 2^-24)) of `streams` sample spans:
   frame f of stream s reads span[s * span_stride + f * 160 .. + 512) (pre-emphasised samples,
   already reflected at the stream edges) and goes to out[s * out_stride + f * 128 ..]. */
int nemo_logmel_frames(const float *span, int64_t span_stride, int streams, int nframes, float *out, int64_t out_stride, void *stream);

/* Sample-rate conversion of `streams` streams at once: outputs [out0, out0 + count) of the
   windowed-sinc resampler of src/resample.c:34-82 (the sums of produce(), src/resample.c:52-71;
   the host keeps the FIFO bookkeeping). Output j is sum_k h(k - j r) x[k] / sum_k h(k - j r),
   r = in_rate / out_rate, over ceil(j r - half) <= k <= floor(j r + half), with x zero outside
   [0, nin). Row s of `in` (in_ld apart) holds input samples [in_start, in_start + in_len) of
   stream s, which must include every k in [0, nin) the outputs reach; output j of stream s goes
   to out[s * out_ld + j - out0]. Rates up to about 20x the output rate (shared-memory bound). */
int nemo_resample(const float *in, int64_t in_ld, int64_t in_start, int64_t in_len, int64_t nin, int64_t out0, int count, int in_rate,
                  int out_rate, float *out, int64_t out_ld, int streams, void *stream);

/* LSTM cell on gates [rows][4H] (i, f, g, o). Replaces lstm_cell (src/kernels.metal:475-486). */
int nemo_lstm_cell(const float *gates, const float *c_in, float *c_out, float *h_out, int rows, int H, void *stream);
/* Joint + argmax per row: logits = W . relu(enc[r] + pred[r]) + b (W bf16 [V][H]); ties ->
   lowest index. out_idx[r], out_val[r]. Replaces joint_partial + argmax_reduce
   (src/kernels.metal:490-550, dispatched at src/decoder.c:81-90). enc row r at enc + r*enc_ld,
   pred row r at pred + r*pred_ld (pred_ld 0 = one shared prediction vector). */
int nemo_joint_argmax(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, const uint16_t *W,
                      const float *bias, int V, int H, int rows, int *out_idx, float *out_val, void *stream);

const char *nemo_gpu_last_error(void);
/* 0 if no kernel has reported a device-side failure (a bounded wait that gave up instead of
   hanging); otherwise -1 with the message in nemo_gpu_last_error(). Synchronous (reads a flag);
   each failure is reported once. */
int nemo_gpu_check_device_errors(void);
/* Diagnostic: launch a wait that nothing completes, bounded by limit_cycles clock cycles, to show
   that a device wait which runs out returns an error status instead of hanging or trapping.
   kind 0 = the tensor-core kernels' mbarrier wait, kind 1 = the persistent kernels' grid barrier.
   The next nemo_gpu_check_device_errors (and the next nemoasr_feed / batch step, through err)
   reports it, once. The reference surfaces Metal command-buffer errors the same way through
   err/errlen (src/gpu.m:131-134); it has no such self-test. */
int nemo_gpu_wait_selftest(int kind, long long limit_cycles, void *stream);
/* Number of CUDA kernels this library has launched (directly or by graph launch) since load. */
uint64_t nemo_gpu_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
