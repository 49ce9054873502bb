/* Model weights resident in HBM (one arena per device) and the vocabulary / prompt tables.
   Layout choices differ from the reference's arena (src/model.c:205-284) where the B200 kernels
   want them: q|k|v rows back to back as one [3D][D] matrix (as src/model.c:241-242), each LSTM
   layer's Wx and Wh side by side as one [4H][2H] matrix so one GEMM yields all gates, and small
   tensors widened to fp32 (as src/model.c:59-67). */
#ifndef NB_MODEL_H
#define NB_MODEL_H
#include "nb.h"

typedef struct {
    uint16_t *ff1_w1, *ff1_w2, *ff2_w1, *ff2_w2, *wqkv, *wo, *pw1, *pw2;
    float *ln_ff1_g, *ln_ff1_b, *ln_att_g, *ln_att_b, *ln_conv_g, *ln_conv_b, *ln_ff2_g, *ln_ff2_b, *ln_out_g, *ln_out_b;
    float *bn_g, *bn_b, *dw_w, *bias_u, *bias_v, *ptab;
} nb_layer_t;

typedef struct nb_model {
    nb_config_t g;
    int device;
    char gpu_name[256];
    void *arena;
    size_t arena_bytes, arena_used;
    float *conv0_w, *conv0_b, *conv2_w, *conv2_b, *conv5_w, *conv5_b, *conv3_b, *conv6_b, *pre_out_b;
    uint16_t *conv3_w, *conv6_w, *pre_out_w;
    nb_layer_t *L;
    uint16_t *prompt_w0, *prompt_w2;
    float *prompt_b2;
    uint16_t *lstm_w[2];
    float *lstm_b[2];
    uint16_t *embed;
    uint16_t *joint_enc_w, *joint_pred_w, *joint_out_w;
    float *joint_enc_b, *joint_pred_b, *joint_out_b;
    /* host tables */
    uint16_t *prompt_b0_host;     /* [PH] */
    uint16_t *prompt_onehot_host; /* [PH][NP]: columns D.. D+NP-1 of prompt_kernel.0.weight */
    char **pieces;
    int n_pieces;
    char **lang_keys;
    int *lang_idx;
    int n_lang;
    double load_ms;
    /* the encoder weights laid out for the persistent single-stream encoder on a grid of
       enc1_grid CTAs (built by the first single-stream engine, shared by all of the model's) */
    uint8_t *enc1_image;
    float *enc1_fold;  /* and the LayerNorm fold constants of the persistent encoder */
    int enc1_grid;
} nb_model_t;

nb_model_t *nb_model_load(nb_source_t *src, char *err, size_t errlen);
void nb_model_free(nb_model_t *m);
int nb_model_prompt_index(const nb_model_t *m, const char *lang);
/* b_eff[n] = b0[n] + W0[n][D + idx] (src/model.c:312-322), fp32 into out[PH]. */
void nb_model_prompt_bias(const nb_model_t *m, int idx, float *out);
int nb_model_right_trained(const nb_model_t *m, int right);
/* Text of one token: "" for specials and language tags, U+2581 -> ' ' (src/tokenizer.c:34-50). */
char *nb_model_token_text(const nb_model_t *m, int id);

#endif
