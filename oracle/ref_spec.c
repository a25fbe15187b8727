/*
 * ref_spec.c -- TEST INFRASTRUCTURE.  Compiles the reference's own mistral/speculative.h (included from the
 * reference tree at build time, never copied) against the stand-ins in ref_stub/ and exports its n-gram drafter,
 * spec_softmax, spec_sample_probs and spec_accept as plain C entry points for tests/test_ref_spec.py, which holds
 * the parity oracle (oracle/oracle.c) to them.  Randomness: arc4random draws from a table set by ref_set_draws.
 */
#include "speculative.h"

#define REF_API __attribute__((visibility("default")))

const uint32_t *g_ref_draws = NULL;
int g_ref_n_draws = 0, g_ref_next_draw = 0;

REF_API void ref_set_draws(const uint32_t *draws, int n) {
    g_ref_draws = draws;
    g_ref_n_draws = n;
    g_ref_next_draw = 0;
}

REF_API int ref_draws_used(void) { return g_ref_next_draw; }

/* speculative.h:395-464: a drafter over history[0..hlen), then one ngram_draft_fn call. */
REF_API int ref_ngram_draft(const int *history, int hlen, int ngram_n, int max_draft, int current_token,
                            int *draft_tokens, float *draft_probs) {
    NGramDraft *d = ngram_draft_init(history, hlen, ngram_n, max_draft);
    SpeculativeState s;
    spec_state_init(&s);
    const int n = ngram_draft_fn(d, NULL, NULL, current_token, 0, 0.0f, &s);
    for (int i = 0; i < n; i++) {
        draft_tokens[i] = s.draft_tokens[i];
        draft_probs[i] = s.draft_probs[i];
    }
    ngram_draft_free(d);
    return n;
}

/* speculative.h:408-418 then :425: history pushed token by token after a prompt. */
REF_API int ref_ngram_draft_pushed(const int *prompt, int n_prompt, const int *pushed, int n_pushed, int ngram_n,
                                   int max_draft, int current_token, int *draft_tokens, float *draft_probs) {
    NGramDraft *d = ngram_draft_init(prompt, n_prompt, ngram_n, max_draft);
    ngram_draft_push_n(d, pushed, n_pushed);
    SpeculativeState s;
    spec_state_init(&s);
    const int n = ngram_draft_fn(d, NULL, NULL, current_token, 0, 0.0f, &s);
    for (int i = 0; i < n; i++) {
        draft_tokens[i] = s.draft_tokens[i];
        draft_probs[i] = s.draft_probs[i];
    }
    ngram_draft_free(d);
    return n;
}

REF_API void ref_spec_softmax(const float *logits, float *probs, int n, float temperature) {
    spec_softmax(logits, probs, n, temperature);
}

REF_API int ref_spec_sample_probs(const float *probs, int n) { return spec_sample_probs(probs, n); }

REF_API int ref_spec_accept(const float *draft_probs, const float *target_logits, const int *draft_tokens, int n_draft,
                            int vocab_size, float temperature, int *accepted_tokens) {
    return spec_accept(draft_probs, target_logits, draft_tokens, n_draft, vocab_size, temperature, accepted_tokens);
}
