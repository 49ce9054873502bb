/* Where the model's tensors come from: a checkpoint directory in the reference's format
   (config.json + model.safetensors, read the way src/safetensors.c:11-56 and src/model.c:185-200
   read them) or the in-memory synthetic generator. Also the config parser (src/model.c:125-172). */
#include "nb.h"
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

double nb_now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1000.0 + (double)ts.tv_nsec / 1e6;
}

typedef struct { char *name; int bf16; size_t offset, nbytes, numel; } st_entry;

struct nb_source {
    nbj_t *config;
    /* checkpoint file */
    void *map;
    size_t map_len;
    st_entry *t;
    size_t nt;
    /* synthetic */
    int synth;
    nemoasr_synth_spec_t spec;
};

static char *slurp(const char *path, size_t *len) {
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (n < 0) { fclose(f); return NULL; }
    char *b = malloc((size_t)n + 1);
    if (fread(b, 1, (size_t)n, f) != (size_t)n) { fclose(f); free(b); return NULL; }
    fclose(f);
    b[n] = 0;
    *len = (size_t)n;
    return b;
}

nb_source_t *nb_source_open_dir(const char *dir, char *err, size_t errlen) {
    nb_source_t *s = calloc(1, sizeof *s);
    char path[4096];
    size_t len;
    snprintf(path, sizeof path, "%s/config.json", dir);
    char *txt = slurp(path, &len);
    if (!txt) { snprintf(err, errlen, "cannot read %s", path); free(s); return NULL; }
    char jerr[256];
    s->config = nbj_parse(txt, len, jerr, sizeof jerr);
    free(txt);
    if (!s->config) { snprintf(err, errlen, "config.json: %s", jerr); free(s); return NULL; }

    snprintf(path, sizeof path, "%s/model.safetensors", dir);
    int fd = open(path, O_RDONLY);
    if (fd < 0) { snprintf(err, errlen, "cannot open %s", path); nb_source_close(s); return NULL; }
    struct stat sb;
    if (fstat(fd, &sb) != 0) { close(fd); snprintf(err, errlen, "fstat %s failed", path); nb_source_close(s); return NULL; }
    void *map = mmap(NULL, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { snprintf(err, errlen, "mmap %s failed", path); nb_source_close(s); return NULL; }
    s->map = map;
    s->map_len = (size_t)sb.st_size;
    uint64_t hl = 0;
    if (s->map_len < 8) { snprintf(err, errlen, "%s: file too small", path); nb_source_close(s); return NULL; }
    memcpy(&hl, map, 8);
    if (hl > s->map_len - 8) { snprintf(err, errlen, "%s: bad header length", path); nb_source_close(s); return NULL; }
    nbj_t *hdr = nbj_parse((const char *)map + 8, (size_t)hl, jerr, sizeof jerr);
    if (!hdr || hdr->type != NBJ_OBJ) { snprintf(err, errlen, "%s header: %s", path, jerr); nbj_free(hdr); nb_source_close(s); return NULL; }
    const size_t data0 = 8 + (size_t)hl;
    s->t = calloc(hdr->count, sizeof *s->t);
    for (size_t i = 0; i < hdr->count; ++i) {
        if (!strcmp(hdr->keys[i], "__metadata__")) continue;
        const nbj_t *e = hdr->items[i];
        st_entry *T = &s->t[s->nt];
        T->name = strdup(hdr->keys[i]);
        T->bf16 = !strcmp(nbj_str(nbj_get(e, "dtype"), ""), "BF16");
        const nbj_t *shape = nbj_get(e, "shape");
        T->numel = 1;
        for (size_t d = 0; d < nbj_len(shape); ++d) T->numel *= (size_t)nbj_num(nbj_at(shape, d), 0);
        const nbj_t *off = nbj_get(e, "data_offsets");
        const size_t a = (size_t)nbj_num(nbj_at(off, 0), 0), b = (size_t)nbj_num(nbj_at(off, 1), 0);
        T->offset = data0 + a;
        T->nbytes = b >= a ? b - a : 0;
        s->nt++;
        if (b < a || T->offset + T->nbytes > s->map_len) {
            snprintf(err, errlen, "tensor %s out of file bounds", T->name);
            nbj_free(hdr);
            nb_source_close(s);
            return NULL;
        }
    }
    nbj_free(hdr);
    return s;
}

nb_source_t *nb_source_open_synth(const nemoasr_synth_spec_t *spec, char *err, size_t errlen) {
    if (spec->d_model <= 0 || spec->d_model % 128 || spec->n_layers <= 0 || spec->vocab_size <= 0) {
        snprintf(err, errlen, "bad synthetic spec (d_model must be a positive multiple of 128)");
        return NULL;
    }
    nb_source_t *s = calloc(1, sizeof *s);
    s->synth = 1;
    s->spec = *spec;
    char *txt = nb_synth_config_json(spec);
    char jerr[256];
    s->config = nbj_parse(txt, strlen(txt), jerr, sizeof jerr);
    free(txt);
    if (!s->config) { snprintf(err, errlen, "synthetic config: %s", jerr); free(s); return NULL; }
    return s;
}

void nb_source_close(nb_source_t *s) {
    if (!s) return;
    if (s->map) munmap(s->map, s->map_len);
    for (size_t i = 0; i < s->nt; ++i) free(s->t[i].name);
    free(s->t);
    nbj_free(s->config);
    free(s);
}
const nbj_t *nb_source_config(const nb_source_t *s) { return s->config; }

int nb_source_bf16(nb_source_t *s, const char *name, size_t numel, uint16_t *dst, char *err, size_t errlen) {
    if (s->synth) {
        if (nb_synth_tensor(&s->spec, name, numel, dst)) { snprintf(err, errlen, "missing tensor %s (or unexpected size %zu)", name, numel); return -1; }
        return 0;
    }
    for (size_t i = 0; i < s->nt; ++i) {
        if (strcmp(s->t[i].name, name)) continue;
        if (!s->t[i].bf16) { snprintf(err, errlen, "tensor %s is not bf16", name); return -1; }
        if (s->t[i].numel != numel || s->t[i].nbytes != numel * 2) {
            snprintf(err, errlen, "tensor %s has %zu elements, expected %zu", name, s->t[i].numel, numel);
            return -1;
        }
        memcpy(dst, (const char *)s->map + s->t[i].offset, numel * 2);
        return 0;
    }
    snprintf(err, errlen, "missing tensor %s", name);
    return -1;
}

/* Same defaults and checks as src/model.c:125-172. */
int nb_parse_config(const nbj_t *c, nb_config_t *g, char *err, size_t errlen) {
    const nbj_t *enc = nbj_get(c, "encoder"), *pre = nbj_get(c, "preprocessor"), *pr = nbj_get(c, "prompt");
    const nbj_t *dec = nbj_get(c, "decoder"), *jo = nbj_get(c, "joint");
    if (!enc || !pre || !pr || !dec || !jo) { snprintf(err, errlen, "config.json missing sections"); return -1; }
    memset(g, 0, sizeof *g);
    g->feat_in = (int)nbj_num(nbj_get(enc, "feat_in"), 128);
    g->n_layers = (int)nbj_num(nbj_get(enc, "n_layers"), 24);
    g->d_model = (int)nbj_num(nbj_get(enc, "d_model"), 1024);
    g->n_heads = (int)nbj_num(nbj_get(enc, "n_heads"), 8);
    g->head_dim = g->n_heads > 0 ? g->d_model / g->n_heads : 0;
    g->d_ff = g->d_model * (int)nbj_num(nbj_get(enc, "ff_expansion_factor"), 4);
    g->subsampling = (int)nbj_num(nbj_get(enc, "subsampling_factor"), 8);
    g->sub_channels = (int)nbj_num(nbj_get(enc, "subsampling_conv_channels"), 256);
    g->conv_kernel = (int)nbj_num(nbj_get(enc, "conv_kernel_size"), 9);
    g->num_prompts = (int)nbj_num(nbj_get(pr, "num_prompts"), 128);
    g->prompt_hidden = (int)nbj_num(nbj_get(pr, "prompt_hidden"), 2048);
    g->pred_hidden = (int)nbj_num(nbj_get(dec, "pred_hidden"), 640);
    g->pred_layers = (int)nbj_num(nbj_get(dec, "pred_rnn_layers"), 2);
    g->vocab_size = (int)nbj_num(nbj_get(dec, "vocab_size"), 13087);
    g->blank_id = g->vocab_size;
    g->joint_hidden = (int)nbj_num(nbj_get(jo, "joint_hidden"), 640);
    g->num_classes = (int)nbj_num(nbj_get(jo, "num_classes"), 13087) + 1;
    g->max_symbols = (int)nbj_num(nbj_get(c, "max_symbols"), 10);
    g->ln_eps = 1e-5f;
    const nbj_t *acs = nbj_get(enc, "att_context_size");
    for (size_t i = 0; i < nbj_len(acs) && i < 8; ++i) {
        const nbj_t *pair = nbj_at(acs, i);
        g->att_left = (int)nbj_num(nbj_at(pair, 0), 56);
        g->trained_right[g->n_trained++] = (int)nbj_num(nbj_at(pair, 1), 13);
    }
    g->att_right_default = (int)nbj_num(nbj_at(nbj_get(c, "default_att_context_size"), 1), 13);
    if (g->pred_layers != 2) { snprintf(err, errlen, "only 2 LSTM layers supported"); return -1; }
    if (g->head_dim != 128 || g->joint_hidden > 1024 || g->conv_kernel != 9 || g->subsampling != 8 || g->d_model % 128 ||
        g->pred_hidden % 32 || g->joint_hidden % 32 || g->sub_channels % 32 || g->d_ff % 128 || g->prompt_hidden % 128) {
        snprintf(err, errlen, "unexpected architecture dims");
        return -1;
    }
    if ((int)nbj_num(nbj_get(pre, "sample_rate"), 16000) != 16000 || (int)nbj_num(nbj_get(pre, "features"), 128) != 128 || g->feat_in != 128) {
        snprintf(err, errlen, "unexpected preprocessor config");
        return -1;
    }
    if (g->num_classes != g->vocab_size + 1) { snprintf(err, errlen, "num_classes must be vocab_size + 1"); return -1; }
    int maxr = 0;
    for (int i = 0; i < g->n_trained; ++i) if (g->trained_right[i] > maxr) maxr = g->trained_right[i];
    g->Lmax = g->att_left + maxr + 1 + 2;
    int f = g->feat_in;
    for (int i = 0; i < 3; ++i) f = f / 2 + 1;
    g->sub_freq_out = f;
    return 0;
}
