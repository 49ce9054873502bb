/* Public API (include/nemoasr.h): the reference's session surface (src/nemoasr.c) over the B200
   engine, plus the synthetic-model and batched-stream entry points. */
#include "engine.h"
#include <cuda_runtime_api.h>
#include <dirent.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

static const int LAT_MS[] = { 80, 160, 320, 560, 1120 }; /* src/nemoasr.c:58-59 */
static const int LAT_R[] = { 0, 1, 3, 6, 13 };
static int lat_index(int right) {
    for (int i = 0; i < 5; ++i) if (LAT_R[i] == right) return i;
    return -1;
}
static int right_for(int latency_ms) {
    for (int i = 0; i < 5; ++i) if (LAT_MS[i] == latency_ms) return LAT_R[i];
    return -1;
}

struct nemoasr {
    nb_model_t *m;
    nb_engine_t *eng;
    nb_engine_t *warm[5];  /* engines warmed by nemoasr_prepare_latency for other latencies (LAT_MS order) */
    int prompt;            /* language prompt index of the session (kept across latency changes) */
    nb_mel_t *mel;
    nb_resampler_t *rs;
    int input_rate, latency_ms, finished, printed_any;
    float *tmp;
    size_t tmp_cap;
    char *text;
    size_t text_len, text_cap;
    int *tok;
    int tok_cap;
    double load_ms;
    nemoasr_stats_t stats;
};

int nemoasr_default_model_dir(char *out, size_t n) {
    const char *home = getenv("HOME");
    char snaps[1024];
    snprintf(snaps, sizeof snaps, "%s/.cache/huggingface/hub/models--mlx-community--nemotron-3.5-asr-streaming-0.6b/snapshots", home ? home : ".");
    DIR *d = opendir(snaps);
    if (!d) return -1;
    struct dirent *ent;
    int found = 0;
    while ((ent = readdir(d))) {
        if (ent->d_name[0] == '.') continue;
        snprintf(out, n, "%s/%s", snaps, ent->d_name);
        char probe[2048];
        snprintf(probe, sizeof probe, "%s/model.safetensors", out);
        struct stat sb;
        if (stat(probe, &sb) == 0) { found = 1; break; }
    }
    closedir(d);
    return found ? 0 : -1;
}

static nb_model_t *load_model(const char *model_dir, const nemoasr_synth_spec_t *spec, char *err, size_t errlen) {
    nb_source_t *src;
    nemoasr_synth_spec_t sp;
    if (spec) src = nb_source_open_synth(spec, err, errlen);
    else if (model_dir && !strncmp(model_dir, "synthetic:", 10)) {
        nemoasr_synth_default(&sp);
        sp.seed = strtoull(model_dir + 10, NULL, 10);
        src = nb_source_open_synth(&sp, err, errlen);
    } else if (model_dir) src = nb_source_open_dir(model_dir, err, errlen);
    else { snprintf(err, errlen, "no model"); return NULL; }
    if (!src) return NULL;
    nb_model_t *m = nb_model_load(src, err, errlen);
    nb_source_close(src);
    return m;
}

/* Feed through the GPU log-mel: every stream's samples (after resampling, `count` each) in pieces
   whose frames fit one staged span; each piece is staged (host bookkeeping), transformed on the
   GPU into the engine's frame queue, and stepped. Steps see final only on the last piece. */
static int feed_gpu_mel(nb_engine_t *eng, nb_mel_t **mel, const float *const *in, size_t count, int B, int final, int *tokens, int max_tokens,
                        int *counts, size_t *chunks, char *err, size_t errlen) {
    const size_t piece = (size_t)(NB_SPAN_FRAMES - 3) * NB_MEL_HOP;
    size_t *nf = malloc((size_t)B * sizeof *nf);
    size_t off = 0;
    int rc = 0;
    do {
        const size_t len = count - off < piece ? count - off : piece;
        const int last = final && off + len >= count;
        if (nb_engine_span_wait(eng)) { snprintf(err, errlen, "span staging: device error"); rc = -1; break; }
        /* streams staged in groups, each group's upload in flight while the next is staged */
        const int G = B >= 64 ? 4 : 1;
        for (int grp = 0; grp < G && !rc; ++grp) {
            const int s0 = (int)((int64_t)B * grp / G), s1 = (int)((int64_t)B * (grp + 1) / G);
#pragma omp parallel for schedule(static) if (s1 - s0 > 1)
            for (int s = s0; s < s1; ++s) {
                size_t cap;
                float *span = nb_engine_span(eng, s, &cap);
                /* a stream that never saw a sample has no frames, not a reflected empty one */
                nf[s] = (last && len == 0 && nb_mel_total_samples(mel[s]) == 0) ? 0 : nb_mel_stage(mel[s], in[s] + off, len, last, span, cap);
            }
            for (int s = s0; s < s1; ++s)
                if (nf[s] != nf[0] || nf[s] == (size_t)-1) { snprintf(err, errlen, "streams produced different frame counts (%zu vs %zu)", nf[s], nf[0]); rc = -1; break; }
            if (!rc && nf[0] && nb_engine_upload_spans(eng, s0, s1, nf[0], err, errlen)) rc = -1;
        }
        if (rc) break;
        if (nf[0] && nb_engine_finish_spans(eng, nf[0], err, errlen)) { rc = -1; break; }
        int r, rows;
        while ((r = nb_engine_step(eng, last, tokens, max_tokens, counts, &rows, err, errlen)) == 1)
            if (rows > 0) ++*chunks;
        if (r < 0) { rc = -1; break; }
        off += len;
    } while (off < count);
    free(nf);
    return rc;
}

static nemoasr_t *open_common(nb_model_t *m, const char *language, int latency_ms, int input_rate, double t0, char *err, size_t errlen) {
    const int right = right_for(latency_ms);
    nemoasr_t *s = calloc(1, sizeof *s);
    s->m = m;
    if (!nb_model_right_trained(m, right)) { snprintf(err, errlen, "latency %d ms not trained for this checkpoint", latency_ms); nemoasr_close(s); return NULL; }
    const int idx = nb_model_prompt_index(m, language ? language : "auto");
    if (idx < 0) { snprintf(err, errlen, "unknown language prompt %s", language ? language : "auto"); nemoasr_close(s); return NULL; }
    s->eng = nb_engine_create(m, 1, right, err, errlen);
    if (!s->eng) { nemoasr_close(s); return NULL; }
    if (nb_engine_set_prompt(s->eng, 0, idx, err, errlen)) { nemoasr_close(s); return NULL; }
    s->prompt = idx;
    s->mel = nb_mel_create();
    s->input_rate = input_rate;
    s->latency_ms = latency_ms;
    if (input_rate != NB_MEL_SR) s->rs = nb_resampler_create(input_rate, NB_MEL_SR);
    s->tok_cap = 4096;
    s->tok = malloc((size_t)s->tok_cap * sizeof(int));
    s->load_ms = nb_now_ms() - t0;
    return s;
}

nemoasr_t *nemoasr_open(const char *model_dir, const char *language, int latency_ms, int input_rate, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    if (right_for(latency_ms) < 0) { snprintf(err, errlen, "latency must be one of 80, 160, 320, 560, 1120 ms"); return NULL; }
    if (input_rate <= 0) { snprintf(err, errlen, "input_rate must be positive"); return NULL; }
    const double t0 = nb_now_ms();
    nb_model_t *m = load_model(model_dir, NULL, err, errlen);
    if (!m) return NULL;
    return open_common(m, language, latency_ms, input_rate, t0, err, errlen);
}

nemoasr_t *nemoasr_open_synthetic(const nemoasr_synth_spec_t *spec, const char *language, int latency_ms, int input_rate, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    if (right_for(latency_ms) < 0) { snprintf(err, errlen, "latency must be one of 80, 160, 320, 560, 1120 ms"); return NULL; }
    if (input_rate <= 0) { snprintf(err, errlen, "input_rate must be positive"); return NULL; }
    const double t0 = nb_now_ms();
    nb_model_t *m = load_model(NULL, spec, err, errlen);
    if (!m) return NULL;
    return open_common(m, language, latency_ms, input_rate, t0, err, errlen);
}

void nemoasr_close(nemoasr_t *s) {
    if (!s) return;
    nb_engine_destroy(s->eng);
    for (int i = 0; i < 5; ++i) nb_engine_destroy(s->warm[i]);
    nb_mel_destroy(s->mel);
    nb_resampler_destroy(s->rs);
    nb_model_free(s->m);
    free(s->tmp);
    free(s->text);
    free(s->tok);
    free(s);
}

static void append_text(nemoasr_t *s, const char *t) {
    const size_t n = strlen(t);
    if (!n) return;
    if (s->text_len + n + 1 > s->text_cap) {
        s->text_cap = (s->text_len + n + 1) * 2;
        s->text = realloc(s->text, s->text_cap);
    }
    memcpy(s->text + s->text_len, t, n + 1);
    s->text_len += n;
}

/* resample -> mel -> engine; appends token ids (up to max) and returns their count, -1 on error */
static int feed_tokens(nemoasr_t *s, const float *samples, size_t n, int final, int *out, int max, char *err, size_t errlen) {
    if (s->finished) return 0;
    const float *in = samples;
    size_t count = n;
    if (s->rs && nb_engine_gpu_resample(s->eng, s->input_rate)) {
        nb_resample_job_t job;
        nb_resampler_plan(s->rs, samples, n, final, &job);
        if (nb_engine_resample(s->eng, &job, &in, err, errlen)) return -1;
        nb_resampler_commit(s->rs, job.count);
        count = job.count;
    } else if (s->rs) {
        const size_t need = (size_t)((double)n * NB_MEL_SR / s->input_rate) + 4096;
        if (need > s->tmp_cap) { s->tmp_cap = need * 2; s->tmp = realloc(s->tmp, s->tmp_cap * sizeof(float)); }
        count = n ? nb_resampler_process(s->rs, samples, n, s->tmp, s->tmp_cap) : 0;
        if (final) count += nb_resampler_flush(s->rs, s->tmp + count, s->tmp_cap - count);
        in = s->tmp;
    }
    s->stats.audio_seconds += (double)count / NB_MEL_SR;
    int got = 0;
    if (nb_engine_gpu_mel(s->eng)) {
        size_t chunks = 0;
        const float *ins[1] = { in };
        if (feed_gpu_mel(s->eng, &s->mel, ins, count, 1, final, out, max, &got, &chunks, err, errlen)) return -1;
        s->stats.chunks += chunks;
    } else if (!(final && count == 0 && nb_mel_total_samples(s->mel) == 0)) {
        const float *frames;
        size_t nf;
        nb_mel_push(s->mel, in, count, final, &frames, &nf);
        if (nf && nb_engine_push(s->eng, &frames, nf, err, errlen)) return -1;
        int rc, rows;
        while ((rc = nb_engine_step(s->eng, final, out, max, &got, &rows, err, errlen)) == 1)
            if (rows > 0) s->stats.chunks++;
        if (rc < 0) return -1;
    }
    if (final) s->finished = 1;
    s->stats.tokens += (size_t)got;
    double enc, dec;
    size_t ch;
    nb_engine_times(s->eng, &enc, &dec, &ch);
    s->stats.encoder_ms = enc;
    s->stats.decoder_ms = dec;
    return got;
}

char *nemoasr_feed(nemoasr_t *s, const float *samples, size_t n, int final, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    const int got = feed_tokens(s, samples, n, final, s->tok, s->tok_cap, err, errlen);
    if (got < 0) return NULL;
    for (int i = 0; i < got; ++i) {
        char *txt = nb_model_token_text(s->m, s->tok[i]);
        const char *p = txt;
        if (!s->printed_any) while (*p == ' ') p++;
        if (*p) { append_text(s, p); s->printed_any = 1; }
        free(txt);
    }
    if (!s->text_len) return NULL;
    char *out = s->text;
    s->text = NULL;
    s->text_len = s->text_cap = 0;
    return out;
}

/* Token ids instead of text (parity tests and callers with their own detokenizer). */
int nemoasr_feed_tokens(nemoasr_t *s, const float *samples, size_t n, int final, int *tokens, int max_tokens, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    return feed_tokens(s, samples, n, final, tokens, max_tokens, err, errlen);
}

void nemoasr_free(char *text) { free(text); }

static int check_latency(const nemoasr_t *s, int latency_ms, char *err, size_t errlen) {
    const int right = right_for(latency_ms);
    if (right < 0) { snprintf(err, errlen, "latency must be one of 80, 160, 320, 560, 1120 ms"); return -1; }
    if (!nb_model_right_trained(s->m, right)) { snprintf(err, errlen, "latency %d ms not trained for this checkpoint", latency_ms); return -1; }
    return right;
}

/* src/nemoasr.c:162-172 + src/warmup.c: the reference builds every GPU pipeline a stream at this
   latency can hit and runs a dummy stream. Here the per-chunk work is a CUDA graph per chunk
   shape, so the warm-up captures the graph of every shape the latency can produce (nothing runs):
   on the session's engine when it already has this latency, else on an engine kept for it, which
   a later nemoasr_reset to this latency takes over with its graphs. */
int nemoasr_prepare_latency(nemoasr_t *s, int latency_ms, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    const int right = check_latency(s, latency_ms, err, errlen);
    if (right < 0) return -1;
    if (nb_engine_right(s->eng) == right) return nb_engine_prepare(s->eng, err, errlen);
    const int li = lat_index(right);
    if (!s->warm[li]) {
        s->warm[li] = nb_engine_create(s->m, 1, right, err, errlen);
        if (!s->warm[li]) return -1;
    }
    return nb_engine_prepare(s->warm[li], err, errlen);
}

int nemoasr_graphs_captured(const nemoasr_t *s) { return nb_engine_graphs(s->eng); }

int nemoasr_reset(nemoasr_t *s, const char *language, int latency_ms, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    const int right = check_latency(s, latency_ms, err, errlen);
    if (right < 0) return -1;
    int idx = s->prompt;  /* no language given: keep the session's (the reference keeps it in the model) */
    if (language) {
        idx = nb_model_prompt_index(s->m, language);
        if (idx < 0) { snprintf(err, errlen, "unknown language prompt %s", language); return -1; }
    }
    if (nb_engine_right(s->eng) == right) {
        if (nb_engine_reset(s->eng, err, errlen)) return -1;
    } else {
        const int li = lat_index(right), cur = lat_index(nb_engine_right(s->eng));
        nb_engine_t *e = s->warm[li];
        s->warm[li] = NULL;
        if (!e) e = nb_engine_create(s->m, 1, right, err, errlen);
        if (!e) return -1;
        if (nb_engine_reset(e, err, errlen)) { nb_engine_destroy(e); return -1; }
        /* the engine being replaced keeps its graphs for a later switch back */
        nb_engine_destroy(s->warm[cur]);
        s->warm[cur] = s->eng;
        s->eng = e;
    }
    if (nb_engine_set_prompt(s->eng, 0, idx, err, errlen)) return -1;
    s->prompt = idx;
    nb_mel_destroy(s->mel);
    s->mel = nb_mel_create();
    if (s->rs) { nb_resampler_destroy(s->rs); s->rs = nb_resampler_create(s->input_rate, NB_MEL_SR); }
    free(s->text);
    s->text = NULL;
    s->text_len = s->text_cap = 0;
    s->finished = 0;
    s->printed_any = 0;
    s->latency_ms = latency_ms;
    return 0;
}

double nemoasr_load_ms(const nemoasr_t *s) { return s->load_ms; }
const char *nemoasr_gpu_name(const nemoasr_t *s) { return s->m->gpu_name; }
int nemoasr_latency_ms(const nemoasr_t *s) { return s->latency_ms; }
void nemoasr_stats(const nemoasr_t *s, nemoasr_stats_t *out) { *out = s->stats; }

/* Parity taps (like the reference CLI's --dump-enc, src/main.c:99): encoder rows from now on. */
void nemoasr_set_taps(nemoasr_t *s, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks) {
    nb_engine_set_taps(s->eng, prompted, joint_enc, cap_rows, chunk_rows, cap_chunks);
}
void nemoasr_tap_counts(const nemoasr_t *s, size_t *rows, size_t *chunks) { nb_engine_tap_counts(s->eng, rows, chunks); }

/* ---- batched streams ------------------------------------------------------------------------ */
struct nemoasr_batch {
    nb_model_t *m;
    nb_engine_t *eng;
    int B, input_rate, finished;
    nb_mel_t **mel;
    nb_resampler_t **rs;
    float **tmp;
    size_t tmp_cap;
    const float **frames;
    nemoasr_stats_t stats;
};

nemoasr_batch_t *nemoasr_batch_open(const char *model_dir, const nemoasr_synth_spec_t *synth, int n_streams, const char *const *languages,
                                    int latency_ms, int input_rate, char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    const int right = right_for(latency_ms);
    if (right < 0) { snprintf(err, errlen, "latency must be one of 80, 160, 320, 560, 1120 ms"); return NULL; }
    if (input_rate <= 0 || n_streams <= 0) { snprintf(err, errlen, "input_rate and n_streams must be positive"); return NULL; }
    nb_model_t *m = load_model(model_dir, synth, err, errlen);
    if (!m) return NULL;
    nemoasr_batch_t *b = calloc(1, sizeof *b);
    b->m = m;
    b->B = n_streams;
    b->input_rate = input_rate;
    if (!nb_model_right_trained(m, right)) { snprintf(err, errlen, "latency %d ms not trained for this checkpoint", latency_ms); nemoasr_batch_close(b); return NULL; }
    b->eng = nb_engine_create(m, n_streams, right, err, errlen);
    if (!b->eng) { nemoasr_batch_close(b); return NULL; }
    b->mel = calloc((size_t)n_streams, sizeof *b->mel);
    b->rs = calloc((size_t)n_streams, sizeof *b->rs);
    b->tmp = calloc((size_t)n_streams, sizeof *b->tmp);
    b->frames = calloc((size_t)n_streams, sizeof *b->frames);
    for (int s = 0; s < n_streams; ++s) {
        const char *lang = languages && languages[s] ? languages[s] : "auto";
        const int idx = nb_model_prompt_index(m, lang);
        if (idx < 0) { snprintf(err, errlen, "unknown language prompt %s", lang); nemoasr_batch_close(b); return NULL; }
        if (nb_engine_set_prompt(b->eng, s, idx, err, errlen)) { nemoasr_batch_close(b); return NULL; }
        b->mel[s] = nb_mel_create();
        if (input_rate != NB_MEL_SR) b->rs[s] = nb_resampler_create(input_rate, NB_MEL_SR);
    }
    return b;
}

void nemoasr_batch_close(nemoasr_batch_t *b) {
    if (!b) return;
    nb_engine_destroy(b->eng);
    for (int s = 0; b->mel && s < b->B; ++s) { nb_mel_destroy(b->mel[s]); nb_resampler_destroy(b->rs[s]); free(b->tmp[s]); }
    free(b->mel);
    free(b->rs);
    free(b->tmp);
    free(b->frames);
    nb_model_free(b->m);
    free(b);
}

/* Batch feed at an input rate other than 16 kHz through the GPU resampler, in passes of at most
   one second of input per stream so that the staging buffers stay bounded whatever the feed size
   (the streaming resampler and log-mel give the same outputs under any split of the input). */
static int batch_feed_resampled(nemoasr_batch_t *b, const float *const *samples, size_t n, int final, int *tokens, int max_tokens, int *counts,
                                char *err, size_t errlen) {
    const int B = b->B;
    const size_t piece = (size_t)b->input_rate;
    nb_resample_job_t *jobs = calloc((size_t)B, sizeof *jobs);
    const float **ins = calloc((size_t)B, sizeof *ins);
    size_t off = 0;
    int rc = 0;
    do {
        const size_t len = n - off < piece ? n - off : piece;
        const int last = final && off + len >= n;
#pragma omp parallel for schedule(static) if (B > 1)
        for (int s = 0; s < B; ++s) nb_resampler_plan(b->rs[s], len ? samples[s] + off : NULL, len, last, &jobs[s]);
        if ((rc = nb_engine_resample(b->eng, jobs, ins, err, errlen))) break;
        const size_t count = jobs[0].count;
        for (int s = 0; s < B; ++s) nb_resampler_commit(b->rs[s], jobs[s].count);
        b->stats.audio_seconds += (double)count / NB_MEL_SR * B;
        if ((rc = feed_gpu_mel(b->eng, b->mel, ins, count, B, last, tokens, max_tokens, counts, &b->stats.chunks, err, errlen))) break;
        off += len;
    } while (off < n);
    free(jobs);
    free(ins);
    return rc;
}

int nemoasr_batch_feed(nemoasr_batch_t *b, const float *const *samples, size_t n, int final, int *tokens, int max_tokens, int *counts, char *err,
                       size_t errlen) {
    if (errlen) err[0] = 0;
    for (int s = 0; s < b->B; ++s) counts[s] = 0;
    if (b->finished) return 0;
    const int B = b->B;
    if (b->rs[0] && nb_engine_gpu_resample(b->eng, b->input_rate)) {
        const int rc = batch_feed_resampled(b, samples, n, final, tokens, max_tokens, counts, err, errlen);
        if (final) b->finished = 1;
        for (int s = 0; s < B; ++s) b->stats.tokens += (size_t)counts[s];
        double enc, dec;
        size_t ch;
        nb_engine_times(b->eng, &enc, &dec, &ch);
        b->stats.encoder_ms = enc;
        b->stats.decoder_ms = dec;
        return rc;
    }
    size_t *nf = calloc((size_t)B, sizeof *nf);
    size_t *cnt = calloc((size_t)B, sizeof *cnt);
    const size_t need = (size_t)((double)n * NB_MEL_SR / b->input_rate) + 4096;
    if (b->input_rate != NB_MEL_SR && need > b->tmp_cap) {
        b->tmp_cap = need * 2;
        for (int s = 0; s < B; ++s) b->tmp[s] = realloc(b->tmp[s], b->tmp_cap * sizeof(float));
    }
    const int gpu_mel = nb_engine_gpu_mel(b->eng);
    const float **ins = calloc((size_t)B, sizeof *ins);
#pragma omp parallel for schedule(dynamic, 4) if (!gpu_mel || b->rs[0])  /* with the GPU log-mel and no resampler the loop only copies pointers */
    for (int s = 0; s < B; ++s) {
        const float *in = samples[s];
        size_t c = n;
        if (b->rs[s]) {
            c = n ? nb_resampler_process(b->rs[s], samples[s], n, b->tmp[s], b->tmp_cap) : 0;
            if (final) c += nb_resampler_flush(b->rs[s], b->tmp[s] + c, b->tmp_cap - c);
            in = b->tmp[s];
        }
        cnt[s] = c;
        ins[s] = in;
        if (gpu_mel) continue;
        if (final && c == 0 && nb_mel_total_samples(b->mel[s]) == 0) { nf[s] = 0; b->frames[s] = NULL; continue; }
        nb_mel_push(b->mel[s], in, c, final, &b->frames[s], &nf[s]);
    }
    int rc = 0;
    if (gpu_mel) {
        for (int s = 1; s < B; ++s)
            if (cnt[s] != cnt[0]) { snprintf(err, errlen, "streams resampled to different lengths (%zu vs %zu)", cnt[s], cnt[0]); rc = -1; break; }
        b->stats.audio_seconds += (double)cnt[0] / NB_MEL_SR * B;
        if (!rc) rc = feed_gpu_mel(b->eng, b->mel, ins, cnt[0], B, final, tokens, max_tokens, counts, &b->stats.chunks, err, errlen);
        free(ins);
        free(nf);
        free(cnt);
        if (final) b->finished = 1;
        for (int s = 0; s < B; ++s) b->stats.tokens += (size_t)counts[s];
        double enc, dec;
        size_t ch;
        nb_engine_times(b->eng, &enc, &dec, &ch);
        b->stats.encoder_ms = enc;
        b->stats.decoder_ms = dec;
        return rc;
    }
    free(ins);
    for (int s = 1; s < B; ++s)
        if (nf[s] != nf[0]) { snprintf(err, errlen, "streams produced different frame counts (%zu vs %zu)", nf[s], nf[0]); rc = -1; break; }
    b->stats.audio_seconds += (double)cnt[0] / NB_MEL_SR * B;
    if (!rc && nf[0]) rc = nb_engine_push(b->eng, b->frames, nf[0], err, errlen);
    if (!rc) {
        int r, rows;
        while ((r = nb_engine_step(b->eng, final, tokens, max_tokens, counts, &rows, err, errlen)) == 1)
            if (rows > 0) b->stats.chunks++;
        if (r < 0) rc = -1;
    }
    free(nf);
    free(cnt);
    if (final) b->finished = 1;
    for (int s = 0; s < B; ++s) b->stats.tokens += (size_t)counts[s];
    double enc, dec;
    size_t ch;
    nb_engine_times(b->eng, &enc, &dec, &ch);
    b->stats.encoder_ms = enc;
    b->stats.decoder_ms = dec;
    return rc;
}

int nemoasr_batch_reset(nemoasr_batch_t *b, char *err, size_t errlen) {
    if (nb_engine_reset(b->eng, err, errlen)) return -1;
    for (int s = 0; s < b->B; ++s) {
        nb_mel_destroy(b->mel[s]);
        b->mel[s] = nb_mel_create();
        if (b->rs[s]) { nb_resampler_destroy(b->rs[s]); b->rs[s] = nb_resampler_create(b->input_rate, NB_MEL_SR); }
    }
    b->finished = 0;
    return 0;
}

void nemoasr_batch_stats(const nemoasr_batch_t *b, nemoasr_stats_t *out) {
    *out = b->stats;
    size_t chunks = 0;
    nb_engine_times(b->eng, &out->encoder_ms, &out->decoder_ms, &chunks); /* also covers steps driven by nemoasr_batch_step */
}
int nemoasr_batch_decode_counts(nemoasr_batch_t *b, long long out[4], char *err, size_t errlen) {
    if (errlen) err[0] = 0;
    return nb_engine_decode_counts(b->eng, out, err, errlen);
}
void nemoasr_batch_set_taps(nemoasr_batch_t *b, float *prompted, float *joint_enc, size_t cap_rows, int *chunk_rows, size_t cap_chunks) {
    nb_engine_set_taps(b->eng, prompted, joint_enc, cap_rows, chunk_rows, cap_chunks);
}
nb_engine_t *nb_batch_engine(nemoasr_batch_t *b) { return b->eng; }
