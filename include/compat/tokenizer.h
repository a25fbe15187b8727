/*
 * compat/tokenizer.h -- drop-in for the reference's mistral/tokenizer.h, backed by the library's tokenizer
 * (sd_tokenizer_*: the same ids as the reference for every text).
 *
 *   Tokenizer                 mistral/tokenizer.h:21-30   (tokens / scores / types / vocab_size / bos_id / eos_id;
 *                                                          the hash table is inside the library)
 *   tokenizer_init            mistral/tokenizer.h:121-153
 *   tokenizer_encode          mistral/tokenizer.h:200-346
 *   tokenizer_decode_token    mistral/tokenizer.h:348-373
 *   tokenizer_decode          mistral/tokenizer.h:375-412 (free the result with free())
 *   tokenizer_apply_chat      mistral/tokenizer.h:416-429 (free the result with free())
 *   tokenizer_free            mistral/tokenizer.h:431-442
 */
#ifndef SPECDEC_COMPAT_TOKENIZER_H
#define SPECDEC_COMPAT_TOKENIZER_H
#include <stdlib.h>
#include <string.h>
#include "gguf_loader.h"

enum { TOK_NORMAL = 1, TOK_UNKNOWN = 2, TOK_CONTROL = 3, TOK_UNUSED = 4, TOK_BYTE = 6 };

typedef struct {
    char **tokens;
    float *scores;
    int *types;
    int vocab_size;
    int bos_id, eos_id;
    sd_tokenizer *impl;
} Tokenizer;

static inline Tokenizer *tokenizer_init(GGUFFile *gguf) {
    if (!gguf) return NULL;
    Tokenizer *t = (Tokenizer *)calloc(1, sizeof(Tokenizer));
    if (!t) return NULL;
    if (sd_tokenizer_create(gguf->mmap_base, gguf->mmap_len, &t->impl) != SD_OK) {
        free(t);
        return NULL;
    }
    sd_tokenizer_info(t->impl, &t->vocab_size, &t->bos_id, &t->eos_id);
    t->tokens = (char **)calloc((size_t)t->vocab_size, sizeof(char *));
    t->scores = (float *)calloc((size_t)t->vocab_size, sizeof(float));
    t->types = (int *)calloc((size_t)t->vocab_size, sizeof(int));
    for (int i = 0; i < t->vocab_size; i++) {
        const char *p = "";
        sd_tokenizer_entry(t->impl, i, &p, &t->scores[i], &t->types[i]);
        t->tokens[i] = strdup(p);
    }
    return t;
}

static inline int tokenizer_encode(Tokenizer *t, const char *text, int *out, int max_tokens, int add_bos) {
    int n = sd_tokenizer_encode(t->impl, text, (int32_t *)out, max_tokens, add_bos);
    return n < 0 ? 0 : n;
}

static inline const char *tokenizer_decode_token(Tokenizer *t, int token_id) { return sd_tokenizer_piece(t->impl, token_id); }

static inline char *tokenizer_decode(Tokenizer *t, const int *tokens, int n_tokens) {
    char *s = sd_tokenizer_decode(t->impl, (const int32_t *)tokens, n_tokens);
    if (!s) return NULL;
    char *r = strdup(s);
    sd_free(s);
    return r;
}

static inline char *tokenizer_apply_chat(const char *user_msg) {
    char *s = sd_tokenizer_apply_chat(user_msg);
    if (!s) return NULL;
    char *r = strdup(s);
    sd_free(s);
    return r;
}

static inline void tokenizer_free(Tokenizer *t) {
    if (!t) return;
    if (t->tokens)
        for (int i = 0; i < t->vocab_size; i++) free(t->tokens[i]);
    free(t->tokens);
    free(t->scores);
    free(t->types);
    sd_tokenizer_free(t->impl);
    free(t);
}

#endif
