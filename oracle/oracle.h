/*
 * oracle.h -- CPU restatement of m0at/ANEtransformers' Mistral Q4_0 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * product in anetransformers_b200/ and the timed CPU baseline in bench.py.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * may load it.  The product never links, imports or calls it.
 *
 * Every function restates one reference function in portable C (x86-64, gcc);
 * the reference itself needs arm_neon.h, clang blocks, GCD and Accelerate and
 * does not compile here.  Each definition cites the reference file:line it
 * follows (paths relative to the reference repository root).
 *
 * Parity pinning: the reference's own known-answer tests (Q4_0 dequant values,
 * RoPE pos-0 identity and norm preservation, GQA head broadcast, RMSNorm /
 * SiLU / softmax KATs; tests/test_mistral.m:414-518,742-779,921-983) are
 * replayed against this code in tests/test_oracle_kat.py.  The quantizer codes,
 * SDOT block sums, n-gram drafts and acceptance have no golden vectors in the
 * reference: for those the restatement follows the code line by line and is the
 * only oracle.  Apple Accelerate calls (vDSP_dotpr, vvexpf, vvsincosf) are
 * restated with libm, so values behind those calls are pinned only to within
 * floating-point tolerance.
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* mistral/dequant.h:17-21 -- 18-byte Q4_0 block: fp16 scale bits + 16 nibble bytes.
 * Nibble layout (dequant.h:611-612): low nibble of qs[j] = element j,
 * high nibble = element j+16.  Value = d * (q - 8). */
typedef struct { uint16_t d; uint8_t qs[16]; } or_block_q4_0;

/* mistral/dequant.h:537-541 -- 36-byte Q8_0 activation block: fp32 scale + 32 int8.
 * (Not ggml's 34-byte fp16-scale layout.) */
typedef struct { float d; int8_t qs[32]; } or_block_q8_0;

/* Quantizer rounding variant.  The reference compiles with -ffast-math
 * (mistral/Makefile:2), which may turn amax/127.0f into a multiply by the
 * rounded reciprocal of 127.  OR_QUANT_IEEE follows the source text exactly;
 * OR_QUANT_RECIP models the reciprocal rewrite. */
enum { OR_QUANT_IEEE = 0, OR_QUANT_RECIP = 1 };

/* Matvec accumulation form: OR_ACC_FMA = sumf = fmaf(wd*xd, (float)isum, sumf)
 * (fp-contract under -ffast-math); OR_ACC_MULADD = separate multiply and add. */
enum { OR_ACC_FMA = 0, OR_ACC_MULADD = 1 };

typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab_size;
    float rope_theta, rms_eps;
} or_config;

typedef struct {
    const void *wq, *wk, *wv, *wo, *w1, *w2, *w3;   /* Q4_0 AoS, [rows][in/32] */
    const float *rms_att, *rms_ffn;                  /* [dim] */
} or_layer;

#define OR_MAX_LAYERS 64

typedef struct {
    or_config cfg;
    or_layer layers[OR_MAX_LAYERS];
    const void *tok_embd;    /* Q4_0 [vocab][dim] */
    const float *rms_final;  /* [dim] */
    const void *lm_head;     /* [vocab][dim] of type lm_head_type */
    int tok_embd_type;       /* OR_TYPE_Q4_0 (default 0 is read as Q4_0) or OR_TYPE_Q4_K */
    int lm_head_type;        /* OR_TYPE_Q4_0 (default), OR_TYPE_Q4_K or OR_TYPE_Q6_K */
    float *theta_inv;        /* [head_dim/2] */
    /* scratch (mistral/mistral_model.h:339-350) */
    float *xb, *xb2, *q, *k, *v, *att, *hb, *hb2, *logits;
    or_block_q8_0 *xb_q8, *hb_q8;
    int att_cap;
} or_model;

/* mistral/kv_cache.h:10-20 -- fp16 sequence-major ring, [layer][max_seq][kv_dim]. */
typedef struct {
    int n_layers, n_kv_heads, head_dim, max_seq, kv_dim;
    uint16_t *k, *v;
    int pos, len;
} or_kv;

/* ---- threading (stand-in for GCD dispatch_apply, dequant.h:1037) ---- */
void or_set_threads(int n);
int  or_get_threads(void);

/* ---- fp16 helpers ---- */
float    or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);

/* ---- kernels ---- */
void or_quantize_q8_0(const float *x, or_block_q8_0 *out, int n, int variant);
void or_q4q8_block_sums(const void *W, const or_block_q8_0 *x, int32_t *isum,
                        int out_dim, int in_dim);
void or_matvec_q4_0_q8_0(const void *W, const or_block_q8_0 *x, float *y,
                         int out_dim, int in_dim);
void or_set_acc_mode(int mode);
void or_dequant_q4_0(const void *blocks, float *out, int n);

/* K-quant super-blocks of 256 values (GGML type ids) -- mistral/dequant.h:15-30, :280-290. */
enum { OR_TYPE_Q4_0 = 2, OR_TYPE_Q4_K = 12, OR_TYPE_Q6_K = 14 };
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[128]; } or_block_q4_K;            /* 144 B */
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } or_block_q6_K; /* 210 B */
/* Q6_K -> fp32 (dequant_q6_K_block, mistral/dequant.h:292-306); n a multiple of 256. */
void or_dequant_q6_K(const void *blocks, float *out, int n);
/* Q4_K -> fp16 values (bits) in the reference's fp16 arithmetic (dequant_q4_K_block_neon, :63-113). */
void or_dequant_q4_K_f16(const void *blocks, uint16_t *out, int n);
/* y[r] = W[r] . x with fp32 activations, the reference's fp32 path for K-quant matrices (q4_matvec,
 * mistral/mistral_model.h:211-242 -> q6_K_matvec_f32_neon, dequant.h:349-520; Q4_K: fp16 dequant then sgemv).
 * Accumulation: value i goes into lane i % 4 by fused multiply-add, the four lanes are added pairwise. */
void or_matvec_kq_f32(int type, const void *W, const float *x, float *y, int rows, int in_dim);
void or_rmsnorm(float *out, const float *x, const float *w, int dim, float eps);
void or_rope_theta(float *theta_inv, int head_dim, float theta);
void or_apply_rope(float *q, float *k, int pos, const float *theta_inv,
                   int n_heads, int n_kv_heads, int head_dim);
void or_silu_mul(float *gate, const float *up, int n);
void or_softmax(float *x, int n);
void or_attention(float *q, float *att, float *out, const uint16_t *kc,
                  const uint16_t *vc, int n_heads, int heads_per_kv, int hd,
                  int max_seq, int pos);

/* ---- model ---- */
int  or_model_init(or_model *m, int max_seq);   /* allocs scratch + theta_inv */
void or_model_free(or_model *m);
int  or_kv_alloc(or_kv *kv, int n_layers, int n_kv_heads, int head_dim, int max_seq);
void or_kv_free(or_kv *kv);
void or_embed_token(const or_model *m, int token, float *out);
void or_layer_decode(or_model *m, or_kv *kv, float *x, int layer, int pos);
void or_logits(or_model *m, const float *x);
void or_forward_token(or_model *m, or_kv *kv, int token, int pos, int n_layers);

/* ---- sampling ---- */
typedef struct {
    float temp;
    int   top_k;
    float top_p;
    float rep_penalty;
    const int *prev_tokens;
    int   n_prev;
} or_sample_params;

/* Seeded replacement for arc4random(): Philox4x32-10 keyed by seed; draw k is
 * word 0 of philox(counter = {k, 0, 0, 0}). */
typedef struct { uint64_t seed; uint64_t counter; } or_rng;
uint32_t or_philox_u32(uint64_t seed, uint64_t counter);
uint32_t or_rng_next(or_rng *r);
float    or_rng_uniform(or_rng *r);   /* (float)u / (float)UINT32_MAX */

int or_sample_argmax(const float *logits, int n);
int or_sample_token(float *logits, int n, const or_sample_params *p, or_rng *rng);

/* ---- speculative ---- */
#define OR_SPEC_MAX_DRAFT 8
void or_spec_softmax(const float *logits, float *probs, int n, float temperature);
int  or_spec_sample_probs(const float *probs, int n, or_rng *rng);
int  or_spec_accept(const float *draft_probs, const float *target_logits,
                    const int *draft_tokens, int n_draft, int vocab, float temperature,
                    int *accepted, or_rng *rng);

typedef struct {
    int *history; int history_len; int history_cap;
    int ngram_n; int max_draft;
} or_ngram;
int  or_ngram_init(or_ngram *d, const int *prompt, int n_prompt, int ngram_n, int max_draft);
void or_ngram_push(or_ngram *d, int token);
void or_ngram_free(or_ngram *d);
int  or_ngram_draft(const or_ngram *d, int current_token, int *draft_tokens, float *draft_probs);
/* pure scan over a history array (same semantics as or_ngram_draft) */
int  or_ngram_scan(const int *history, int hlen, int ngram_n, int max_draft,
                   int current_token, int *draft_tokens, int *match_pos_out);

/* ---- generation loops ---- */
enum { OR_BONUS_ARGMAX = 0, OR_BONUS_REFERENCE = 1 };
typedef struct {
    int max_tokens;       /* --tokens */
    float temp, top_p; int top_k; float rep_penalty; int rep_window;
    int ignore_eos; int eos_id;
    int spec_k;           /* drafts per iteration */
    int ngram_n;
    int draft_layers;     /* self-spec */
    int history_has_current;   /* 1 = reference n-gram wiring (quirk), 0 = prompt lookup */
    int bonus_mode;            /* OR_BONUS_ARGMAX (fixed) or OR_BONUS_REFERENCE */
    uint64_t seed;
    int max_seq;
} or_gen_opts;

typedef struct {
    int n_generated;
    int64_t total_draft, total_accepted, total_iterations;
} or_gen_stats;

/* out_tokens must hold max_tokens + SPEC_MAX_DRAFT + 2 entries. */
int or_generate_greedy(or_model *m, const int *prompt, int n_prompt,
                       const or_gen_opts *o, int *out_tokens, or_gen_stats *st);
int or_generate_ngram(or_model *m, const int *prompt, int n_prompt,
                      const or_gen_opts *o, int *out_tokens, or_gen_stats *st);
int or_generate_self_spec(or_model *m, const int *prompt, int n_prompt,
                          const or_gen_opts *o, int *out_tokens, or_gen_stats *st);

/* Prefill by sequential single-token decode (mistral_infer.m:594-599). */
void or_prefill(or_model *m, or_kv *kv, const int *tokens, int n, int n_layers, float *x_out);

#ifdef __cplusplus
}
#endif
