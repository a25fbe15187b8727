/*
 * compat/speculative.h -- drop-in for the reference's mistral/speculative.h, backed by the B200 engine.
 * The model and its KV ring are one sd_ctx (the ring lives in HBM, so the KVCache argument of the
 * reference signatures is accepted and ignored).
 *
 *   SpeculativeState, spec_state_init     speculative.h:14-28
 *   spec_verify                           speculative.h:81-105  -> sd_forward (batched, one weight read)
 *   spec_accept                           speculative.h:121-198 -> sd_spec_accept on the device of the
 *                                         context bound by spec_bind_context (bonus from row n_draft,
 *                                         the callers' override of speculative.h:312-317)
 *   NGramDraft, ngram_draft_init/push/push_n/free/fn   speculative.h:387-464 -> device scan
 *   spec_decode_loop                      speculative.h:217-379 -> sd_decode (whole loop on the device)
 */
#ifndef SPECDEC_COMPAT_SPECULATIVE_H
#define SPECDEC_COMPAT_SPECULATIVE_H
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include "../specdec_b200.h"

#define SPEC_MAX_DRAFT 8

typedef struct {
    int draft_tokens[SPEC_MAX_DRAFT];
    float draft_probs[SPEC_MAX_DRAFT];
    int64_t total_draft;
    int64_t total_accepted;
    int64_t total_iterations;
} SpeculativeState;

static inline void spec_state_init(SpeculativeState *s) { memset(s, 0, sizeof(*s)); }

/* spec_accept has no model argument in the reference; it runs on the context bound here. */
static sd_ctx *spec_bound_ctx_ = NULL;
static inline void spec_bind_context(sd_ctx *ctx) { spec_bound_ctx_ = ctx; }

static inline int spec_verify(sd_ctx *model, void *kv_unused, const int *tokens, int n, int start_pos,
                              float *target_logits) {
    (void)kv_unused;
    sd_model_info in;
    if (sd_ctx_info(model, &in) != SD_OK) return -1;
    for (int i = 0; i < n; i += 8) {
        int S = n - i < 8 ? n - i : 8;
        if (sd_forward(model, (const int32_t *)tokens + i, S, start_pos + i, target_logits + (size_t)i * in.vocab_size,
                       NULL) != SD_OK)
            return -1;
    }
    return 0;
}

/* target_logits: [n_draft + 1][vocab] (row n_draft feeds the bonus token). */
static inline int spec_accept(const float *draft_probs, const float *target_logits, const int *draft_tokens,
                              int n_draft, int vocab_size, float temperature, int *accepted_tokens) {
    static uint64_t counter = 0;
    (void)vocab_size;
    if (!spec_bound_ctx_) return -1;
    int n = sd_spec_accept(spec_bound_ctx_, draft_probs, target_logits, (const int32_t *)draft_tokens, n_draft,
                           temperature, SD_BONUS_ARGMAX, 0, &counter, (int32_t *)accepted_tokens);
    return n;
}

typedef struct {
    int *history;
    int history_len;
    int history_cap;
    int ngram_n;
    int max_draft;
} NGramDraft;

static inline NGramDraft *ngram_draft_init(const int *prompt_tokens, int n_prompt, int ngram_n, int max_draft) {
    NGramDraft *d = (NGramDraft *)calloc(1, sizeof(NGramDraft));
    d->ngram_n = ngram_n > 0 ? ngram_n : 3;
    d->max_draft = max_draft > 0 ? max_draft : 4;
    if (d->max_draft > SPEC_MAX_DRAFT) d->max_draft = SPEC_MAX_DRAFT;
    d->history_cap = n_prompt + 4096;
    d->history = (int *)malloc(sizeof(int) * d->history_cap);
    memcpy(d->history, prompt_tokens, sizeof(int) * n_prompt);
    d->history_len = n_prompt;
    return d;
}

static inline void ngram_draft_push(NGramDraft *d, int token) {
    if (d->history_len >= d->history_cap) {
        d->history_cap *= 2;
        d->history = (int *)realloc(d->history, sizeof(int) * d->history_cap);
    }
    d->history[d->history_len++] = token;
}

static inline void ngram_draft_push_n(NGramDraft *d, const int *tokens, int n) {
    for (int i = 0; i < n; i++) ngram_draft_push(d, tokens[i]);
}

static inline void ngram_draft_free(NGramDraft *d) {
    if (d) {
        free(d->history);
        free(d);
    }
}

static inline int ngram_draft_fn(void *draft_ctx, void *model, void *kv, int current_token, int pos, float temperature,
                                 SpeculativeState *spec) {
    (void)model; (void)kv; (void)pos; (void)temperature;
    NGramDraft *d = (NGramDraft *)draft_ctx;
    int match = -1;
    int n = sd_ngram_draft((const int32_t *)d->history, d->history_len, d->ngram_n, d->max_draft, current_token,
                           (int32_t *)spec->draft_tokens, &match);
    if (n < 0) return 0;
    for (int i = 0; i < n; i++) spec->draft_probs[i] = 0.9f;
    return n;
}

/* Whole decode loop on the device; the prompt's K/V must already be in the context's ring. */
static inline int spec_decode_loop(sd_ctx *model, const int *history, int n_hist, int first_token, int max_tokens,
                                   float temperature, int mode, int spec_k, int *out_tokens, int out_cap,
                                   SpeculativeState *spec) {
    sd_gen_params p;
    sd_gen_params_default(&p);
    p.mode = mode;
    p.max_tokens = max_tokens;
    p.temp = temperature;
    p.spec_k = spec_k;
    sd_gen_stats st;
    int n = sd_decode(model, &p, (const int32_t *)history, n_hist, first_token, (int32_t *)out_tokens, out_cap, &st);
    if (spec && n >= 0) {
        spec->total_draft = st.total_draft;
        spec->total_accepted = st.total_accepted;
        spec->total_iterations = st.total_iterations;
    }
    return n;
}

#endif
