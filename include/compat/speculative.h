/*
 * compat/speculative.h -- drop-in for the reference's mistral/speculative.h, backed by the B200 engine.  Same
 * type names, fields and signatures; MistralModel, KVCache and Tokenizer come from the compat headers beside
 * this one (the model's weights and KV ring live in HBM, in model->ctx).
 *
 *   SpeculativeState, spec_state_init      speculative.h:14-28
 *   spec_softmax, spec_sample_probs        speculative.h:37-68   -> sd_spec_softmax / sd_spec_sample_probs
 *   spec_verify                            speculative.h:81-105  -> sd_forward (one batched forward per 16 tokens)
 *   spec_accept                            speculative.h:121-198 -> sd_spec_accept (the bonus from row n_draft-1
 *                                                                   when every draft is accepted, as the reference)
 *   SpecDraftFn                            speculative.h:206-208
 *   spec_decode_loop                       speculative.h:217-379 (see below)
 *   NGramDraft, ngram_draft_init/push/push_n/free/fn   speculative.h:387-464 -> device scan (sd_ngram_draft)
 *   SelfSpecDraft, self_spec_draft_init/free/fn        speculative.h:479-538 -> sd_forward_layers (the first
 *                                                       draft_layers layers + the LM head, greedy)
 * spec_decode_loop runs the reference's loop -- draft, verify [current, drafts], accept, bonus from the last
 * verify row, emit, advance -- with every step on the device.  At temp 0 with ngram_draft_fn whose history is
 * the prompt already in the ring (history_len == start_pos) the whole loop runs on the device (sd_decode; its
 * n-gram history also grows with the emitted tokens, the prompt-lookup wiring; temp-0 output is the same
 * either way).  Random draws come from the Philox stream of compat/mistral_model.h (spec_rng_seed).
 * At temp 0 the bonus is the argmax of the last verify row; the reference's own loop draws it uniformly
 * (spec_softmax at temperature 0 is flat, speculative.h:312-317): spec_set_bonus_mode(SD_BONUS_REFERENCE)
 * reproduces that.
 */
#ifndef SPECDEC_COMPAT_SPECULATIVE_H
#define SPECDEC_COMPAT_SPECULATIVE_H
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include "mistral_model.h"
#include "tokenizer.h"

#define SPEC_MAX_DRAFT 8

typedef struct {
    int draft_tokens[SPEC_MAX_DRAFT];
    float draft_probs[SPEC_MAX_DRAFT];
    int64_t total_draft;
    int64_t total_accepted;
    int64_t total_iterations;
} SpeculativeState;

static inline void spec_state_init(SpeculativeState *s) { memset(s, 0, sizeof(*s)); }

static int spec_bonus_mode_ = SD_BONUS_ARGMAX;
static inline void spec_set_bonus_mode(int mode) { spec_bonus_mode_ = mode; }

static inline double spec_time_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

static inline void spec_softmax(const float *logits, float *probs, int n, float temperature) {
    if (!spec_bound_model_ || sd_spec_softmax(spec_bound_model_->ctx, logits, probs, n, temperature) != SD_OK)
        fprintf(stderr, "spec_softmax: %s\n", spec_bound_model_ ? sd_last_error() : "no model loaded");
}

static inline int spec_sample_probs(const float *probs, int n) {
    if (!spec_bound_model_) return n - 1;
    const int t = sd_spec_sample_probs(spec_bound_model_->ctx, probs, n, spec_rng_seed_, &spec_rng_counter_);
    return t < 0 ? n - 1 : t;
}

static inline int spec_verify(MistralModel *model, KVCache *kv, const int *draft_tokens, int n_draft, int start_pos,
                              float *target_logits) {
    const int vocab = model->cfg.vocab_size;
    for (int i = 0; i < n_draft; i += SD_MAX_VERIFY) {
        const int S = n_draft - i < SD_MAX_VERIFY ? n_draft - i : SD_MAX_VERIFY;
        if (sd_forward(model->ctx, (const int32_t *)draft_tokens + i, S, start_pos + i,
                       target_logits + (size_t)i * vocab, NULL) != SD_OK)
            return -1;
    }
    if (kv && kv->len < kv->max_seq && start_pos + n_draft > kv->len) kv->len = start_pos + n_draft;
    return 0;
}

/* target_logits: [n_draft][vocab_size] (speculative.h:121-198). */
static inline int spec_accept(const float *draft_probs, const float *target_logits, const int *draft_tokens,
                              int n_draft, int vocab_size, float temperature, int *accepted_tokens) {
    if (!spec_bound_model_ || n_draft < 1) return 0;
    /* the device rule takes the bonus from row n_draft: repeat row n_draft-1 there */
    float *rows = (float *)malloc(sizeof(float) * (size_t)(n_draft + 1) * vocab_size);
    if (!rows) return 0;
    memcpy(rows, target_logits, sizeof(float) * (size_t)n_draft * vocab_size);
    memcpy(rows + (size_t)n_draft * vocab_size, target_logits + (size_t)(n_draft - 1) * vocab_size,
           sizeof(float) * (size_t)vocab_size);
    const int n = sd_spec_accept(spec_bound_model_->ctx, draft_probs, rows, (const int32_t *)draft_tokens, n_draft,
                                 temperature, SD_BONUS_ARGMAX, spec_rng_seed_, &spec_rng_counter_,
                                 (int32_t *)accepted_tokens);
    free(rows);
    if (n < 0) fprintf(stderr, "spec_accept: %s\n", sd_last_error());
    return n < 0 ? 0 : n;
}

typedef int (*SpecDraftFn)(void *draft_ctx, MistralModel *model, KVCache *kv, int current_token, int pos,
                           float temperature, SpeculativeState *spec);

/* ---- n-gram drafter ---------------------------------------------------------------------------------------- */
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

static inline int ngram_draft_fn(void *draft_ctx, MistralModel *model, KVCache *kv, int current_token, int pos,
                                 float temperature, SpeculativeState *spec) {
    (void)model; (void)kv; (void)pos; (void)temperature;
    NGramDraft *d = (NGramDraft *)draft_ctx;
    int match = -1;
    const int n = sd_ngram_draft((const int32_t *)d->history, d->history_len, d->ngram_n, d->max_draft, current_token,
                                 (int32_t *)spec->draft_tokens, &match);
    if (n < 0) return 0;
    for (int i = 0; i < n; i++) spec->draft_probs[i] = 0.9f;
    return n;
}

/* ---- self-speculative drafter: the first draft_layers layers of the target + its LM head ------------------ */
typedef struct {
    MistralModel *model;
    KVCache kv;         /* metadata: the drafter's K/V of layers < draft_layers are the target's ring slots,
                           which the verify forward of the same positions overwrites */
    float *x;
    int draft_layers;
    int max_draft;
} SelfSpecDraft;

static inline SelfSpecDraft *self_spec_draft_init(MistralModel *model, int draft_layers, int max_draft, int max_seq) {
    SelfSpecDraft *d = (SelfSpecDraft *)calloc(1, sizeof(SelfSpecDraft));
    d->model = model;
    d->draft_layers = draft_layers;
    d->max_draft = max_draft > SPEC_MAX_DRAFT ? SPEC_MAX_DRAFT : max_draft;
    d->kv = kv_alloc(draft_layers, model->cfg.n_kv_heads, model->cfg.head_dim, max_seq);
    d->x = (float *)calloc((size_t)model->cfg.dim, sizeof(float));
    return d;
}

static inline void self_spec_draft_free(SelfSpecDraft *d) {
    if (!d) return;
    kv_free(&d->kv);
    free(d->x);
    free(d);
}

static inline int self_spec_draft_fn(void *draft_ctx, MistralModel *model, KVCache *kv, int current_token, int pos,
                                     float temperature, SpeculativeState *spec) {
    (void)kv; (void)temperature;
    SelfSpecDraft *d = (SelfSpecDraft *)draft_ctx;
    if (d->kv.len > pos) d->kv.len = pos;
    int tok = current_token;
    for (int k = 0; k < d->max_draft; k++) {
        int32_t t32 = tok, next = 0;
        if (sd_forward_layers(model->ctx, d->draft_layers, &t32, 1, pos + k, NULL, &next) != SD_OK) {
            fprintf(stderr, "self_spec_draft_fn: %s\n", sd_last_error());
            return k;
        }
        spec->draft_tokens[k] = next;
        spec->draft_probs[k] = 1.0f;
        tok = next;
    }
    return d->max_draft;
}

/* ---- the decode loop --------------------------------------------------------------------------------------- */
static inline void spec_print_piece_(Tokenizer *tok, int t) {
    if (!tok) return;
    const char *piece = tokenizer_decode_token(tok, t);
    if (piece) {
        printf("%s", piece);
        fflush(stdout);
    }
}

static inline void spec_print_stats_(const SpeculativeState *spec, int generated, double t_total, double t_draft,
                                     double t_verify) {
    fprintf(stderr, "\n--- Speculative Decoding Stats ---\n");
    fprintf(stderr, "Generated tokens:     %d\n", generated);
    fprintf(stderr, "Draft iterations:     %lld\n", (long long)spec->total_iterations);
    if (spec->total_iterations > 0) {
        fprintf(stderr, "Avg draft/iter:       %.1f\n", (double)spec->total_draft / spec->total_iterations);
        fprintf(stderr, "Avg accepted/iter:    %.1f\n", (double)spec->total_accepted / spec->total_iterations);
        const int64_t pure = spec->total_accepted - spec->total_iterations;
        fprintf(stderr, "Acceptance rate:      %.1f%%\n", spec->total_draft > 0 ? 100.0 * pure / spec->total_draft : 0.0);
    }
    fprintf(stderr, "Draft time:           %.1f ms (%.1f%%)\n", t_draft, t_total > 0 ? 100.0 * t_draft / t_total : 0.0);
    fprintf(stderr, "Verify time:          %.1f ms (%.1f%%)\n", t_verify, t_total > 0 ? 100.0 * t_verify / t_total : 0.0);
    fprintf(stderr, "Total decode:         %.1f ms\n", t_total);
    if (generated > 0) {
        fprintf(stderr, "Effective tok/s:      %.2f\n", generated / (t_total / 1000.0));
        fprintf(stderr, "Per-token (effective): %.1f ms\n", t_total / generated);
    }
}

static inline void spec_decode_loop(MistralModel *model, KVCache *kv, Tokenizer *tok, SpeculativeState *spec,
                                    SpecDraftFn draft_fn, void *draft_ctx, int first_token, int start_pos,
                                    int max_tokens, float temperature) {
    const int vocab = model->cfg.vocab_size;
    sd_model_info info;
    sd_ctx_info(model->ctx, &info);
    const int eos = tok ? tok->eos_id : info.eos_id;
    spec_bound_model_ = model;
    const double t_start = spec_time_ms();
    double t_draft_total = 0, t_verify_total = 0;
    int tokens_generated = 0;

    if (draft_fn == ngram_draft_fn && temperature <= 0.0f && ((NGramDraft *)draft_ctx)->history_len == start_pos) {
        /* the whole loop on the device */
        NGramDraft *d = (NGramDraft *)draft_ctx;
        int32_t *hist = (int32_t *)malloc(sizeof(int32_t) * (size_t)(start_pos + 1));
        int32_t *out = (int32_t *)malloc(sizeof(int32_t) * (size_t)(max_tokens + 2 * SD_MAX_VERIFY + 4));
        for (int i = 0; i < start_pos; i++) hist[i] = d->history[i];
        hist[start_pos] = first_token;
        sd_gen_params p;
        sd_gen_params_default(&p);
        p.mode = SD_GEN_NGRAM;
        p.max_tokens = max_tokens + 1;  /* sd_decode counts the first token as generated; this loop does not */
        p.temp = 0.0f;
        p.rep_penalty = 1.0f;
        p.spec_k = d->max_draft;
        p.ngram_n = d->ngram_n;
        p.bonus_mode = spec_bonus_mode_;
        p.seed = spec_rng_seed_;
        sd_gen_stats st;
        const int n = first_token == eos ? 0
                                         : sd_decode(model->ctx, &p, hist, start_pos + 1, first_token, out,
                                                     max_tokens + 2 * SD_MAX_VERIFY + 4, &st);
        if (n < 0) {
            fprintf(stderr, "spec_decode_loop: %s\n", sd_last_error());
        } else {
            for (int i = 0; i < n; i++) {
                spec_print_piece_(tok, out[i]);
                tokens_generated++;
                if (out[i] == eos) break;
            }
            if (n > 0) {
                spec->total_draft += st.total_draft;
                spec->total_accepted += st.total_accepted;
                spec->total_iterations += st.total_iterations;
                t_verify_total = st.ms_decode;
                if (kv && kv->len < kv->max_seq && start_pos + n > kv->len) kv->len = start_pos + n;
            }
        }
        free(hist);
        free(out);
        spec_print_stats_(spec, tokens_generated, spec_time_ms() - t_start, t_draft_total, t_verify_total);
        return;
    }

    int accepted[SPEC_MAX_DRAFT + 1];
    int current_token = first_token, pos = start_pos;
    float *all_logits = (float *)malloc(sizeof(float) * (size_t)(SPEC_MAX_DRAFT + 1) * vocab);
    while (tokens_generated < max_tokens) {
        if (current_token == eos) break;
        const double t0 = spec_time_ms();
        int n_draft = draft_fn(draft_ctx, model, kv, current_token, pos, temperature, spec);
        if (n_draft <= 0) {
            /* no draft: one target forward and sample_temperature (speculative.h:240-260) */
            int32_t cur32 = current_token;
            if (sd_forward(model->ctx, &cur32, 1, pos, all_logits, NULL) != SD_OK) break;
            current_token = sample_temperature(all_logits, vocab, temperature);
            spec_print_piece_(tok, current_token);
            pos++;
            tokens_generated++;
            spec->total_iterations++;
            continue;
        }
        if (n_draft > SPEC_MAX_DRAFT) n_draft = SPEC_MAX_DRAFT;
        const double t_draft_end = spec_time_ms();
        t_draft_total += t_draft_end - t0;
        const int n_verify = n_draft + 1;
        int verify_tokens[SPEC_MAX_DRAFT + 1];
        verify_tokens[0] = current_token;
        memcpy(verify_tokens + 1, spec->draft_tokens, sizeof(int) * (size_t)n_draft);
        if (spec_verify(model, kv, verify_tokens, n_verify, pos, all_logits) != 0) break;
        t_verify_total += spec_time_ms() - t_draft_end;
        const int n_accepted = spec_accept(spec->draft_probs, all_logits, spec->draft_tokens, n_draft, vocab,
                                           temperature, accepted);
        if (n_accepted < 1) break;
        if (n_accepted == n_draft + 1) {
            /* the bonus comes from the last verify row (speculative.h:312-317) */
            const float *row = all_logits + (size_t)n_draft * vocab;
            if (temperature <= 0.0f && spec_bonus_mode_ == SD_BONUS_ARGMAX) {
                accepted[n_draft] = sample_argmax(row, vocab);
            } else {
                float *bp = (float *)malloc(sizeof(float) * (size_t)vocab);
                spec_softmax(row, bp, vocab, temperature);
                accepted[n_draft] = spec_sample_probs(bp, vocab);
                free(bp);
            }
        }
        int stop = 0;
        for (int i = 0; i < n_accepted; i++) {
            spec_print_piece_(tok, accepted[i]);
            if (accepted[i] == eos) {
                tokens_generated += i + 1;
                stop = 1;
                break;
            }
        }
        if (stop) break;
        spec->total_draft += n_draft;
        spec->total_accepted += n_accepted;
        spec->total_iterations++;
        pos += n_accepted;
        current_token = accepted[n_accepted - 1];
        tokens_generated += n_accepted;
    }
    free(all_logits);
    spec_print_stats_(spec, tokens_generated, spec_time_ms() - t_start, t_draft_total, t_verify_total);
}

#endif
