/*
 * TEST INFRASTRUCTURE.  Stand-in for mistral/mistral_model.h when the reference's mistral/speculative.h is
 * compiled on x86-64 with gcc (oracle/Makefile, target _ref/libspec_ref.so).  The real header pulls in
 * Accelerate, Metal, GCD and NEON; speculative.h needs from it only the model and KV types, a few model calls
 * (which the functions under test -- the n-gram drafter, spec_softmax, spec_sample_probs, spec_accept -- never
 * make) and the Accelerate vector routines below.  The vector routines are restated with libm exactly as the
 * parity oracle restates them (oracle/oracle.c), so a comparison against the oracle checks the reference's own
 * control flow and arithmetic around them.  arc4random draws from a table the harness fills, so both sides
 * consume the same uniforms.
 */
#pragma once
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#include <math.h>
#include "gguf_loader.h"

typedef struct {
    int n_layers, n_kv_heads, head_dim, max_seq, kv_dim;
    uint16_t *k_cache, *v_cache;
    int pos, len;
} KVCache;

typedef struct {
    MistralConfig cfg;
    float *logits;
} MistralModel;

/* Model calls: never reached by the functions under test. */
static void stub_unreachable(const char *what) {
    fprintf(stderr, "reference stub: %s is not available in this build\n", what);
    abort();
}
static void embed_token(MistralModel *m, int t, float *o) { (void)m; (void)t; (void)o; stub_unreachable("embed_token"); }
static void mistral_layer_decode_parallel(MistralModel *m, KVCache *kv, float *x, int l, int p) {
    (void)m; (void)kv; (void)x; (void)l; (void)p;
    stub_unreachable("mistral_layer_decode_parallel");
}
static void mistral_logits(MistralModel *m, const float *x) { (void)m; (void)x; stub_unreachable("mistral_logits"); }
static int sample_argmax(const float *l, int n) { (void)l; (void)n; stub_unreachable("sample_argmax"); return 0; }
static int sample_temperature(const float *l, int n, float t) {
    (void)l; (void)n; (void)t;
    stub_unreachable("sample_temperature");
    return 0;
}
static KVCache kv_alloc(int n_layers, int n_kv_heads, int head_dim, int max_seq) {
    KVCache c;
    memset(&c, 0, sizeof c);
    c.n_layers = n_layers;
    c.n_kv_heads = n_kv_heads;
    c.head_dim = head_dim;
    c.max_seq = max_seq;
    c.kv_dim = n_kv_heads * head_dim;
    return c;
}
static void kv_free(KVCache *c) { (void)c; }

/* Accelerate (vDSP / vForce) routines used by speculative.h, restated as the oracle restates them. */
typedef unsigned long vDSP_Length;
typedef long vDSP_Stride;
static void vDSP_maxv(const float *a, vDSP_Stride ia, float *c, vDSP_Length n) {
    float m = a[0];
    for (vDSP_Length i = 1; i < n; i++)
        if (a[i * ia] > m) m = a[i * ia];
    *c = m;
}
static void vDSP_vsadd(const float *a, vDSP_Stride ia, const float *b, float *c, vDSP_Stride ic, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] + *b;
}
static void vDSP_vsmul(const float *a, vDSP_Stride ia, const float *b, float *c, vDSP_Stride ic, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] * *b;
}
static void vDSP_sve(const float *a, vDSP_Stride ia, float *c, vDSP_Length n) {
    float s = 0.0f;
    for (vDSP_Length i = 0; i < n; i++) s += a[i * ia];
    *c = s;
}
static void vvexpf(float *y, const float *x, const int *n) {
    for (int i = 0; i < *n; i++) y[i] = expf(x[i]);
}

/* arc4random: the next value of the table set by ref_set_draws (harness); 0 once it runs out.  glibc declares its
 * own arc4random, so the reference's calls are renamed to the stand-in. */
extern const uint32_t *g_ref_draws;
extern int g_ref_n_draws, g_ref_next_draw;
static uint32_t ref_arc4random(void) {
    return g_ref_next_draw < g_ref_n_draws ? g_ref_draws[g_ref_next_draw++] : 0u;
}
#define arc4random ref_arc4random
