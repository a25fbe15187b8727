/*
 * compat/mistral_model.h -- drop-in for the model-level entry points of the reference's mistral/mistral_model.h
 * on the decode path, backed by the B200 engine (one sd_ctx holds the repacked weights and the fp16 KV ring).
 *
 *   MistralModel                    mistral/mistral_model.h:30-52    cfg, gguf and the host logits row; the
 *                                                                      per-layer host tensors are replaced by
 *                                                                      `ctx` (weights in HBM)
 *   mistral_load / mistral_free     mistral/mistral_model.h:262-357, :1253-1268
 *   embed_token                     mistral/mistral_model.h:125-157  -> sd_embed_token
 *   mistral_layer_decode_parallel   mistral/mistral_model.h:818-899  -> sd_layer_decode (the layer's K/V goes to
 *                                                                      the engine's ring; kv->len is kept as :856-858)
 *   mistral_logits                  mistral/mistral_model.h:1110-1122 -> sd_logits into m->logits
 *   SampleParams, sample_argmax,    mistral/mistral_model.h:1125-1250 -> sd_sample_token (temp 0: argmax, first
 *   sample_token, sample_temperature                                      index on ties)
 * The reference draws its uniforms from arc4random(); here they come from one Philox stream per process (seed
 * set by spec_rng_seed, default 0), shared with compat/speculative.h, so runs are reproducible.
 * sample_token, sample_argmax and spec_accept take no model argument: they run on the device of the model
 * loaded last (or the one given to spec_bind_model).
 */
#ifndef SPECDEC_COMPAT_MISTRAL_MODEL_H
#define SPECDEC_COMPAT_MISTRAL_MODEL_H
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "gguf_loader.h"
#include "kv_cache.h"

typedef struct {
    MistralConfig cfg;
    GGUFFile *gguf;
    float *logits;  /* [vocab] host: the last mistral_logits result */
    sd_ctx *ctx;    /* the engine: weights and KV ring in HBM */
} MistralModel;

/* The model the argument-less calls run on, and the process's Philox stream (seed, next counter). */
static MistralModel *spec_bound_model_ = NULL;
static uint64_t spec_rng_seed_ = 0, spec_rng_counter_ = 0;

static inline void spec_bind_model(MistralModel *m) { spec_bound_model_ = m; }
static inline void spec_rng_seed(uint64_t seed) {
    spec_rng_seed_ = seed;
    spec_rng_counter_ = 0;
}

/* mistral_load with the KV ring's slot count (the reference's --context, mistral_infer.m:518-523). */
static inline MistralModel *mistral_load_context(const char *path, int max_seq) {
    MistralModel *m = (MistralModel *)calloc(1, sizeof(MistralModel));
    if (!m) return NULL;
    m->gguf = gguf_open(path);
    if (!m->gguf) {
        free(m);
        return NULL;
    }
    m->cfg = m->gguf->cfg;
    sd_ctx_opts o;
    sd_ctx_opts_default(&o);
    o.max_seq = max_seq;
    if (sd_ctx_create(m->gguf->mmap_base, m->gguf->mmap_len, &o, &m->ctx) != SD_OK) {
        fprintf(stderr, "mistral_load: %s\n", sd_last_error());
        gguf_close(m->gguf);
        free(m);
        return NULL;
    }
    m->logits = (float *)calloc((size_t)m->cfg.vocab_size, sizeof(float));
    spec_bound_model_ = m;
    return m;
}

/* The reference's default ring: 65536 slots (mistral_infer.m:518-520). */
static inline MistralModel *mistral_load(const char *path) { return mistral_load_context(path, 65536); }

static inline void mistral_free(MistralModel *m) {
    if (!m) return;
    if (spec_bound_model_ == m) spec_bound_model_ = NULL;
    sd_ctx_free(m->ctx);
    gguf_close(m->gguf);
    free(m->logits);
    free(m);
}

static inline void embed_token(MistralModel *m, int token_id, float *out) {
    if (sd_embed_token(m->ctx, token_id, out) != SD_OK) fprintf(stderr, "embed_token: %s\n", sd_last_error());
}

static inline void mistral_layer_decode_parallel(MistralModel *m, KVCache *kv, float *x, int layer, int pos) {
    if (sd_layer_decode(m->ctx, x, layer, pos) != SD_OK) {
        fprintf(stderr, "mistral_layer_decode_parallel: %s\n", sd_last_error());
        return;
    }
    if (kv && kv->len < kv->max_seq && pos + 1 > kv->len) kv->len = pos + 1;
}

static inline void mistral_logits(MistralModel *m, const float *x) {
    if (sd_logits(m->ctx, x, 1, m->logits) != SD_OK) fprintf(stderr, "mistral_logits: %s\n", sd_last_error());
}

typedef struct {
    float temp;
    int top_k;
    float top_p;
    float rep_penalty;
    const int *prev_tokens;
    int n_prev;
} SampleParams;

static inline int sample_token(float *logits, int n, SampleParams *p) {
    if (!spec_bound_model_) return 0;
    const int t = sd_sample_token(spec_bound_model_->ctx, logits, n, p->temp, p->top_k, p->top_p, p->rep_penalty,
                                  (const int32_t *)p->prev_tokens, p->prev_tokens ? p->n_prev : 0, spec_rng_seed_,
                                  &spec_rng_counter_);
    if (t < 0) {
        fprintf(stderr, "sample_token: %s\n", sd_last_error());
        return 0;
    }
    return t;
}

static inline int sample_argmax(const float *logits, int n) {
    float *copy = (float *)malloc(sizeof(float) * (size_t)n);
    if (!copy) return 0;
    memcpy(copy, logits, sizeof(float) * (size_t)n);
    SampleParams p = {0.0f, 40, 0.9f, 1.0f, NULL, 0};
    const int t = sample_token(copy, n, &p);
    free(copy);
    return t;
}

static inline int sample_temperature(const float *logits_in, int n, float temp) {
    float *copy = (float *)malloc(sizeof(float) * (size_t)n);
    if (!copy) return 0;
    memcpy(copy, logits_in, sizeof(float) * (size_t)n);
    SampleParams p = {temp, 40, 0.9f, 1.0f, NULL, 0};
    const int t = sample_token(copy, n, &p);
    free(copy);
    return t;
}

#endif
