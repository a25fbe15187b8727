/*
 * compat/metal_matvec.h -- drop-in for the context API of the reference's GPU backend
 * (mistral/metal_matvec.h), backed by the B200 engine.  MetalContext is an sd_ctx.
 *
 *   metal_context_init        mistral/metal_matvec.h:134-225  -> sd_ctx_create on the mmap'd GGUF image
 *   metal_set_theta_inv       mistral/metal_matvec.h:228-234  -> no-op: θ_inv is computed from the GGUF
 *   metal_set_rmsnorm_bufs    mistral/metal_matvec.h:237-249  -> no-op: norms are uploaded from the GGUF
 *   metal_alloc_batch_buffers mistral/metal_matvec.h:253-293  -> 0 if S fits one verify forward, else -1
 *   metal_wire_kv_cache       mistral/metal_matvec.h:297-310  -> the KV ring lives in HBM; the host
 *                                                                struct keeps only its metadata
 *   metal_context_free        mistral/metal_matvec.h:540-565
 * The reference's metal_encode_* helpers take Metal encoder objects; their stream-ordered replacement is
 * sd_forward_dev (one forward of S tokens, all layers, plus the LM head).
 */
#ifndef SPECDEC_COMPAT_METAL_MATVEC_H
#define SPECDEC_COMPAT_METAL_MATVEC_H
#include <stdio.h>
#include <stdlib.h>
#include "../specdec_b200.h"

typedef sd_ctx MetalContext;

/* A model loaded through compat/mistral_model.h from the same mmap'd image already holds the weights and the
 * KV ring in HBM: metal_context_init then returns that context (shared, not freed by metal_context_free). */
#ifdef SPECDEC_COMPAT_MISTRAL_MODEL_H
#define SPECDEC_COMPAT_SHARED_CTX_ (spec_bound_model_ ? spec_bound_model_->ctx : NULL)
#define SPECDEC_COMPAT_SHARED_BASE_ (spec_bound_model_ ? spec_bound_model_->gguf->mmap_base : NULL)
#else
#define SPECDEC_COMPAT_SHARED_CTX_ NULL
#define SPECDEC_COMPAT_SHARED_BASE_ NULL
#endif

static inline MetalContext *metal_context_init(void *mmap_base, size_t mmap_len, int dim, int kv_dim, int hidden,
                                               int vocab, int n_heads, int n_layers, int max_seq) {
    sd_ctx *c = NULL;
    if (SPECDEC_COMPAT_SHARED_CTX_ && SPECDEC_COMPAT_SHARED_BASE_ == mmap_base) {
        c = SPECDEC_COMPAT_SHARED_CTX_;
    } else {
        sd_ctx_opts o;
        sd_ctx_opts_default(&o);
        o.max_seq = max_seq;
        if (sd_ctx_create(mmap_base, mmap_len, &o, &c) != SD_OK) {
            fprintf(stderr, "specdec_b200: context init failed: %s\n", sd_last_error());
            return NULL;
        }
    }
    sd_model_info in;
    sd_ctx_info(c, &in);
    if (in.dim != dim || in.n_kv_heads * in.head_dim != kv_dim || in.hidden_dim != hidden || in.vocab_size != vocab ||
        in.n_heads != n_heads || in.n_layers != n_layers) {
        fprintf(stderr, "specdec_b200: GGUF shape differs from the caller's arguments\n");
        if (c != SPECDEC_COMPAT_SHARED_CTX_) sd_ctx_free(c);
        return NULL;
    }
    return c;
}

static inline void metal_set_theta_inv(MetalContext *ctx, const float *theta_inv, int half_dim) {
    (void)ctx; (void)theta_inv; (void)half_dim;
}

static inline void metal_set_rmsnorm_bufs(MetalContext *ctx, int layer, const float *rms_att, const float *rms_ffn,
                                          int dim) {
    (void)ctx; (void)layer; (void)rms_att; (void)rms_ffn; (void)dim;
}

static inline int metal_alloc_batch_buffers(MetalContext *ctx, int S, int dim, int kv_dim, int hidden, int n_heads,
                                            int max_att_len) {
    (void)dim; (void)kv_dim; (void)hidden; (void)n_heads;
    sd_model_info in;
    if (!ctx || sd_ctx_info(ctx, &in) != SD_OK) return -1;
    return (S >= 1 && S <= SD_MAX_VERIFY && max_att_len <= in.max_seq) ? 0 : -1;
}

/* The ring stays in device memory; host code may still read kv->len / kv->max_seq.  Pass the
 * reference's KVCache (or any struct whose first pointer fields are k_cache / v_cache) to drop the
 * host copies, as the reference does when it wires Metal buffers. */
static inline void metal_wire_kv_cache(MetalContext *ctx, void *kv_ptr) {
    (void)ctx;
    typedef struct { int a, b, c, d, e; void *k; void *v; int f, g; } kv_layout;
    kv_layout *kv = (kv_layout *)kv_ptr;
    if (!kv) return;
    free(kv->k);
    free(kv->v);
    kv->k = NULL;
    kv->v = NULL;
}

static inline void metal_context_free(MetalContext *ctx) {
    if (ctx != SPECDEC_COMPAT_SHARED_CTX_) sd_ctx_free(ctx);
}

#endif
