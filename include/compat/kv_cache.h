/*
 * compat/kv_cache.h -- drop-in for the reference's mistral/kv_cache.h.
 *
 *   KVCache    mistral/kv_cache.h:10-20  (same fields)
 *   kv_alloc   mistral/kv_cache.h:22-35  -> metadata only: the fp16 ring [n_layers][max_seq][kv_dim] lives in the
 *                                           model's device memory (sd_ctx), so k_cache / v_cache stay NULL and host
 *                                           code reads only n_layers .. kv_dim, pos and len, as after the
 *                                           reference's metal_wire_kv_cache (mistral/metal_matvec.h:297-310)
 *   kv_free    mistral/kv_cache.h:69-75
 * The ring's contents can be read back with sd_kv_read.
 */
#ifndef SPECDEC_COMPAT_KV_CACHE_H
#define SPECDEC_COMPAT_KV_CACHE_H
#include <stdint.h>
#include <stdlib.h>

typedef struct {
    int n_layers;
    int n_kv_heads;
    int head_dim;
    int max_seq;
    int kv_dim;
    uint16_t *k_cache;  /* fp16 bits; NULL: in device memory */
    uint16_t *v_cache;
    int pos;
    int len;
} KVCache;

static inline KVCache kv_alloc(int n_layers, int n_kv_heads, int head_dim, int max_seq) {
    KVCache c;
    c.n_layers = n_layers;
    c.n_kv_heads = n_kv_heads;
    c.head_dim = head_dim;
    c.max_seq = max_seq;
    c.kv_dim = n_kv_heads * head_dim;
    c.k_cache = NULL;
    c.v_cache = NULL;
    c.pos = 0;
    c.len = 0;
    return c;
}

static inline void kv_free(KVCache *cache) {
    free(cache->k_cache);
    free(cache->v_cache);
    cache->k_cache = NULL;
    cache->v_cache = NULL;
}

#endif
