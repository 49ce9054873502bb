/* Device-side decoder state of the streaming engine (structure of arrays over streams). Shared by
   engine.c (host) and k_engine.cu (kernels). */
#ifndef NB_ENGINE_DEV_H
#define NB_ENGINE_DEV_H
#include <stddef.h>
#include <stdint.h>
#include "../../include/nemo_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int streams, tok_cap;
    int *t, *symbols, *active, *pred_valid, *last_token, *ntok, *tokens;
    int *need_pos;                    /* [streams] compact row of a stream in need_idx, -1 if not listed */
    int *need_idx, *erow, *idx, *cnt; /* cnt[0] streams needing the prediction net, cnt[1] still active,
                                         cnt[2] iterations this chunk, cnt[3] dec_update blocks done */
    float *h, *c, *hp, *cp;           /* [2][streams][PH] committed / provisional LSTM state */
    float *pred;                      /* [streams][JH] joint prediction projection */
    float *A0, *A1, *gates, *hp1c, *predc; /* compact per-iteration work rows */
    int fmt;                          /* format of A0 / A1 / hp1c (GEMM inputs): fp32 or bf16 hi/lo planes */
    int64_t a_plane, h_plane;         /* plane offsets (elements) of A0/A1 and of hp1c */
    uint16_t *jx;                     /* joint GEMM input planes [streams][JH] */
    float *logits;                    /* [streams][num_classes] */
    int *stats;                       /* [0] frames whose first decision emitted a token, [1] decisions
                                         (since reset; kept by the several-stream iterations) */
} DecState;

/* Persistent single-stream encoder (k_encoder1.cu): one conformer block's weights and caches. */
typedef struct {
    const uint16_t *ff1_w1, *ff1_w2, *wqkv, *wo, *pw1, *pw2, *ff2_w1, *ff2_w2;
    const float *ln_ff1_g, *ln_ff1_b, *ln_att_g, *ln_att_b, *ln_conv_g, *ln_conv_b, *ln_ff2_g, *ln_ff2_b, *ln_out_g, *ln_out_b;
    const float *bn_g, *bn_b, *dw_w, *bias_u, *bias_v, *ptab;
    float *kv, *din; /* [cap][3D] and [cap][D] cache rows of the stream */
} NbEnc1Layer;

#define NB_ENC1_MAX_LAYERS 32
typedef struct {
    NbEnc1Layer L[NB_ENC1_MAX_LAYERS]; /* by value: the kernel reads it from its parameter space */
    int layers, D, FF, H, taps, Lmax, c, ring_bytes;
    int left;                   /* attention history rows at most: windows of left + c rows */
    float eps, scale;
    const int *pos, *cache_len; /* device words */
    float *h;                   /* [c][D] residual stream: pre-encode output in, last block's output out */
    float *h2;                  /* [c][D] the residual stream between the two halves of a block */
    const uint8_t *image;       /* the weights laid out per CTA (nb_encoder1_repack) */
    const float *fold;          /* LayerNorm fold constants (nb_encoder1_repack) */
    float *ff, *att;            /* [c][FF], [c][D] scratch */
    uint16_t *xout;             /* LN_out(h) as bf16 hi / lo planes [c][D], xout_plane elements apart */
    int64_t xout_plane;
    unsigned *bar;              /* [2] grid-barrier arrivals, abort flag (zeroed before each launch) */
    int *err;                   /* nonzero after a bounded wait gave up */
    /* the encoder's tail as three more stages of the launch (tail = 1; src/encoder.c:189-194):
       ph = relu(LN_out(h) pw0^T + pb0) [c][PRH], prompted = ph pw2^T + pb2 [c][D] (fp32),
       joint = prompted jw^T + jb [c][JH]; pw0 rows are pw0_ld bf16 apart (its language columns are
       folded into pb0). With tail = 0 the launch ends with xout and these are unused. */
    int tail, PRH, JH, pw0_ld;
    const uint16_t *pw0, *pw2, *jw;
    const float *pb0, *pb2, *jb;
    float *ph, *prompted, *joint;
} NbEnc1Args;

/* Persistent single-stream greedy decoder (k_decoder1.cu). */
typedef struct {
    DecState d;                           /* stream 0's greedy state (read at start, written back) */
    const uint16_t *W0, *W1, *Wp, *Wo, *embed;  /* LSTM [4PH][2PH] x2, prediction [JH][PH], joint out [V][JH], embed [V][PH] */
    const float *b0, *b1, *bp, *bo;
    const float *enc;                     /* [c][JH] joint encoder rows of the chunk */
    float *H0, *H1;                       /* [2][PH] committed / provisional hidden state (roles swap on emission) */
    float *PRED;                          /* [JH] */
    float *part_v;                        /* [16][grid] per-CTA best logit per frame */
    int *part_i;                          /* [16][grid] and its vocabulary index */
    unsigned *bar;                        /* [2] grid-barrier arrivals, abort flag (zeroed before each launch) */
    int *err;
    int PH, JH, V, blank, max_symbols, c;
} NbDec1Args;

int nb_decoder1(const NbDec1Args *args, int grid, void *stream);
int nb_decoder1_fits(int PH, int JH, int V, int grid, int cmax, size_t smem_optin);
size_t nb_decoder1_smem(int PH, int JH, int V, int grid, int c);

int nb_encoder1(const NbEnc1Args *args, int grid, void *stream);
int nb_encoder1_ring_bytes(int D, int FF, int grid, size_t smem_optin, int c, int Lw);
size_t nb_encoder1_smem(int ring_bytes, int c, int Lw);
size_t nb_encoder1_image_bytes(int D, int FF, int layers);
size_t nb_encoder1_tail_image_bytes(int D, int PRH, int JH);
size_t nb_encoder1_fold_bytes(int D, int FF, int layers);
int nb_encoder1_repack(const NbEnc1Args *args, int grid, uint8_t *image, float *fold, void *stream);

/* log-mel frames of sample spans (k_mel.cu) into rows out_row0.. of each stream's frame block */
int nb_logmel_frames(const float *span, int64_t span_stride, int streams, int nframes, float *out, int64_t out_stride, int64_t out_row0,
                     void *stream);

/* nonzero if nemo_resample (k_resample.cu) takes this rate pair */
int nb_resample_smem_ok(int in_rate, int out_rate);

int nb_set_error(const char *fmt, ...);
int nb_gemm_validate(const nemo_gemm_args_t *a, const char *who);
int nb_gemm_tc_init(void);
void nb_set_launch_counting(int on);
void nb_count_launches(uint64_t n);
int nb_compact(float *kv, float *din, int layers, int streams, int64_t cap, int D, int src_kv, int cache_len, int src_din, int dst_din,
               int conv_left, void *stream);
int nb_dec_chunk_init(const DecState *d, int c, void *stream);
int nb_dec_plan(const DecState *d, int c, void *stream);
int nb_dec_gather(const DecState *d, const uint16_t *embed, int PH, int blank, void *stream);
int nb_dec_cell(const DecState *d, int layer, int PH, float *next, int64_t next_ld, int64_t next_plane, void *stream);
int nb_dec_scatter_pred(const DecState *d, int JH, void *stream);
/* cond: handle of the CUDA graph WHILE loop this launch belongs to (0 outside such a loop); the
   last block sets it to "another iteration" while streams remain active and fewer than max_it
   iterations ran. cnt[2] counts the iterations of the chunk. */
int nb_dec_update(const DecState *d, int c, int PH, int blank, int max_symbols, int max_it, unsigned long long cond, const float *logits,
                  int64_t ldl, int V, void *stream);
/* Joint input of every stream: X[b] = relu(enc[erow[b]] + pred_b) as bf16 hi/lo planes (zeros for
   inactive streams), where pred_b is the freshly computed compact row of a listed stream (also
   stored as its prediction) or its kept prediction. */
int nb_dec_joint_in(const DecState *d, const float *enc, int JH, uint16_t *X, int64_t plane, void *stream);
int nb_dec_reset(const DecState *d, int PH, int blank, void *stream);

/* ---- fused batched greedy decoder (activation-major tensor-core GEMMs with decoder epilogues) --
   The LSTM weights are gate-interleaved (row 4u + g holds gate g of unit u, gates i, f, g, o), so
   each 16-column epilogue chunk holds all four gates of 4 units. A stream runs the prediction
   network only right after it emitted a token, and the state it then commits is the provisional
   state of its last prediction run; so the recurrent halves W0h . h0 and W1h . h1 of its next
   run are computed as soon as that state exists, by the GEMMs that read h0' and h1' anyway
   (their weight rows concatenated), and kept per stream as R0 = W0h . h0, R1 = b1 + W1h . h1.
   One iteration, for the streams listed (rows of the compact GEMMs):
     step kernel:  gates0 = T[token] + R0[b] -> cell 0 (c0)        -> h0' into the G1 input row
     G1:  [W1x ; W0h] . h0'   -> gates1 = . + R1[b] -> cell 1 (c1) -> h1' into the G2 input row
                              -> R0[b] = W0h . h0'
     G2:  [Wp ; W1h] . h1'    -> pred[b] = bp + ., X[b] = relu(enc[erow[b]] + pred[b])
                              -> R1[b] = b1 + W1h . h1'
     G3:  Wo . X              -> logits; the step kernel takes each active stream's argmax.
   T[v] = b0 + W0x . embed[v] (blank's row is b0: blank feeds zeros). The cell state c of each
   layer is kept once per stream: it is read and rewritten by the same run, which always follows
   the commit of the previous run's state. */
typedef struct {
    int mode;                 /* 1: LSTM cell; 2: prediction + joint input; 3: per-row argmax of bias + product */
    int n_split;              /* columns [0, n_split) take the cell / prediction; [n_split, N) go to aux */
    const int *need_idx;      /* GEMM row -> stream */
    const int *last_token;    /* mode 1: if set, the gate row of stream b is row[last_token[b]], else row[b] */
    const float *row;         /* mode 1: [.][n_split] gate rows added to the product (bias included) */
    float *c;                 /* mode 1: [streams][n_split / 4] cell state, read and rewritten */
    uint16_t *next;           /* mode 1: next GEMM input, row m, columns [0, n_split / 4): bf16 hi/lo planes */
    int64_t next_ld, next_plane;
    const float *enc;         /* mode 2: [rows][n_split] joint encoder rows; erow[b] selects the row */
    const int *erow;
    float *pred;              /* mode 2: [streams][n_split] */
    uint16_t *X;              /* mode 2: [streams][n_split] joint input, bf16 hi/lo planes */
    int64_t x_plane;
    float *aux;               /* [streams][N - n_split]: aux[b][n - n_split] = product (+ aux_bias) */
    const float *aux_bias;
    float *part_v;            /* mode 3: [rows][part_ld] best value of each (column tile, half), ties to */
    int *part_i;              /*         the lowest column; and its column */
    int part_ld;
} NbDecEpi;

/* Tensor-core GEMM (activation-major tiles) with a decoder epilogue instead of the plain one. */
int nb_gemm_dec(const nemo_gemm_args_t *a, const NbDecEpi *de, void *stream);
/* Argmax partials per row of the mode-3 (joint output) GEMM over n columns: two per column tile. */
int nb_dec_joint_parts(int n);

typedef struct {
    const float *logits;      /* [streams][ldl] */
    int64_t ldl;
    int V, blank, max_symbols, PH, JH;
    const float *enc;         /* [streams * c][JH] joint encoder rows of the chunk */
    const float *part_v;      /* if set: the logits' argmax comes as nparts partial (value, index) pairs per stream */
    const int *part_i;
    int nparts;
    const float *T, *R0;      /* [V][4PH] token gate rows of layer 0, [streams][4PH] recurrent part */
    float *c0;                /* [streams][PH] layer-0 cell state */
    uint16_t *A, *X;          /* G1 input rows (h0', compact) and joint input rows (per stream) */
    int64_t a_ld, a_plane, x_plane;
} NbDecStep;

/* Chunk start: per-stream counters, layer 0 of the streams whose prediction is stale (their G1
   input rows) and the joint input of the others. cnt[0] = streams listed, cnt[1] = streams
   active, cnt[2] = 0. */
int nb_dec_chunk_start(const DecState *d, const NbDecStep *s, int c, void *stream);
/* One greedy decision per active stream from its logits row, then the next iteration's rows as
   at chunk start; the last block publishes cnt[0], cnt[1], counts the iteration in cnt[2] and
   sets the WHILE condition (cond != 0). */
int nb_dec_step(const DecState *d, const NbDecStep *s, int c, int max_it, unsigned long long cond, void *stream);
/* R0[b] = 0 and R1[b] = b1 for every stream (the recurrent gate parts of a zero state). */
int nb_dec_rows_init(float *R0, float *R1, const float *b1, int streams, int W, void *stream);
/* Gate-interleaved copy of an LSTM layer [4PH][K] (and its bias when given). */
int nb_dec_interleave(const uint16_t *W, uint16_t *Wi, const float *bias, float *bi, int PH, int K, void *stream);
/* table[v][n] = bi[n] + sum_{k < PH} Wi[n][k] * embed[v][k] (fp32, k ascending); row blank = bi. */
int nb_dec_gate_table(const uint16_t *Wi, int64_t ldw, const uint16_t *embed, int V, int PH, const float *bi, int blank, float *table,
                      void *stream);
int nb_joint_argmax_rows(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, int pred_rpg, const uint16_t *W,
                         const float *bias, int V, int H, int rows, const int *enc_row_of, int *out_idx, float *out_val, void *stream);
int nb_joint_argmax_gemm(const float *enc, int64_t enc_ld, const float *pred, int64_t pred_ld, const uint16_t *W, const float *bias, int V, int H,
                         int rows, const int *enc_row_of, uint16_t *X, float *logits, int64_t ldl, int *out_idx, float *out_val, void *stream);
int nb_dwconv2d_s2_fmt(const float *X, const float *W, const float *bias, void *Y, int y_fmt, int64_t y_plane, int streams, int T, int F,
                       int T1, int F1, int C, void *stream);
int nb_flatten_rows_fmt(const float *X, void *Y, int y_fmt, int64_t y_plane, const int *lo, int streams, int T, int F, int C, int c, void *stream);

#ifdef __cplusplus
}
#endif
#endif
