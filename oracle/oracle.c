/*
 * oracle.c -- CPU restatement of the reference's Mistral Q4_0 W4A8 decode path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker + timed CPU baseline); see oracle.h.
 * Compiled with -O2 -ffp-contract=off so that the only fused multiply-adds are
 * the explicit fmaf() calls that model the reference's NEON vfmaq / clang
 * fp-contract behaviour.
 */
#define _GNU_SOURCE
#include "oracle.h"
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>

/* ------------------------------------------------------------------------- */
/* fp16 <-> fp32 (IEEE binary16, round-to-nearest-even)                       */
/* ------------------------------------------------------------------------- */
float or_f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

uint16_t or_f32_to_f16(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

/* ------------------------------------------------------------------------- */
/* Row-chunk thread pool: stand-in for GCD dispatch_apply with an atomic chunk  */
/* counter (mistral/dequant.h:1037-1042).  Workers persist between calls.      */
/* ------------------------------------------------------------------------- */
typedef void (*or_chunk_fn)(void *ctx, int chunk);

static struct {
    int n_threads;           /* total including caller */
    pthread_t th[128];
    int started;
    pthread_mutex_t mu;
    pthread_cond_t go, done;
    unsigned gen;
    int busy;                /* workers still running current job */
    or_chunk_fn fn;
    void *ctx;
    int n_chunks;
    int next;                /* atomic */
    int quit;
} g_pool = { .n_threads = 1, .mu = PTHREAD_MUTEX_INITIALIZER,
             .go = PTHREAD_COND_INITIALIZER, .done = PTHREAD_COND_INITIALIZER };

static void pool_drain(void) {
    int c;
    while ((c = __atomic_fetch_add(&g_pool.next, 1, __ATOMIC_RELAXED)) < g_pool.n_chunks)
        g_pool.fn(g_pool.ctx, c);
}

static void *pool_worker(void *arg) {
    (void)arg;
    unsigned seen = 0;
    pthread_mutex_lock(&g_pool.mu);
    for (;;) {
        while (g_pool.gen == seen && !g_pool.quit)
            pthread_cond_wait(&g_pool.go, &g_pool.mu);
        if (g_pool.quit) break;
        seen = g_pool.gen;
        pthread_mutex_unlock(&g_pool.mu);
        pool_drain();
        pthread_mutex_lock(&g_pool.mu);
        if (--g_pool.busy == 0) pthread_cond_signal(&g_pool.done);
    }
    pthread_mutex_unlock(&g_pool.mu);
    return NULL;
}

static void pool_stop(void) {
    if (!g_pool.started) return;
    pthread_mutex_lock(&g_pool.mu);
    g_pool.quit = 1;
    pthread_cond_broadcast(&g_pool.go);
    pthread_mutex_unlock(&g_pool.mu);
    for (int i = 0; i < g_pool.n_threads - 1; i++) pthread_join(g_pool.th[i], NULL);
    g_pool.started = 0;
    g_pool.quit = 0;
}

void or_set_threads(int n) {
    if (n < 1) n = 1;
    if (n > 128) n = 128;
    pool_stop();
    g_pool.n_threads = n;
    if (n > 1) {
        for (int i = 0; i < n - 1; i++) pthread_create(&g_pool.th[i], NULL, pool_worker, NULL);
        g_pool.started = 1;
    }
}

int or_get_threads(void) { return g_pool.n_threads; }

static void parallel_chunks(int n_chunks, or_chunk_fn fn, void *ctx) {
    if (g_pool.n_threads <= 1 || n_chunks <= 1) {
        for (int c = 0; c < n_chunks; c++) fn(ctx, c);
        return;
    }
    pthread_mutex_lock(&g_pool.mu);
    g_pool.fn = fn;
    g_pool.ctx = ctx;
    g_pool.n_chunks = n_chunks;
    g_pool.next = 0;
    g_pool.busy = g_pool.n_threads - 1;
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.go);
    pthread_mutex_unlock(&g_pool.mu);
    pool_drain();
    pthread_mutex_lock(&g_pool.mu);
    while (g_pool.busy > 0) pthread_cond_wait(&g_pool.done, &g_pool.mu);
    pthread_mutex_unlock(&g_pool.mu);
}

/* ------------------------------------------------------------------------- */
/* Q8_0 activation quantizer -- mistral/dequant.h:545-599                      */
/* ------------------------------------------------------------------------- */
void or_quantize_q8_0(const float *x, or_block_q8_0 *out, int n, int variant) {
    const int nb = n / 32;
    for (int i = 0; i < nb; i++) {
        const float *src = x + 32 * i;
        /* amax = max |x| over the block (dequant.h:553-568); max is order-free. */
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(src[j]);
            if (a > amax) amax = a;
        }
        /* d = amax / 127 (dequant.h:570); RECIP models -ffast-math's rewrite. */
        float d = (variant == OR_QUANT_RECIP) ? amax * (1.0f / 127.0f) : amax / 127.0f;
        out[i].d = d;
        if (amax == 0.0f) {                       /* dequant.h:573-576 */
            memset(out[i].qs, 0, 32);
            continue;
        }
        float id = 1.0f / d;                      /* dequant.h:578 */
        for (int j = 0; j < 32; j++) {
            /* vcvtnq_s32_f32: round to nearest, ties to even, saturating, NaN -> 0
             * (dequant.h:587-588); a denormal amax makes id = inf, so the saturating
             * form matters there;
             * vqmovn s32->s16->s8: saturate to [-128, 127] (dequant.h:591-595). */
            float v = src[j] * id;
            long r;
            if (v != v) r = 0;                          /* NaN -> 0 (FCVTNS) */
            else if (v >= 2147483648.0f) r = 2147483647L;
            else if (v <= -2147483648.0f) r = -2147483647L - 1;
            else r = lrintf(v);
            if (r > 127) r = 127;
            if (r < -128) r = -128;
            out[i].qs[j] = (int8_t)r;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Q4_0 x Q8_0 exact int32 block dot -- the SDOT inner step of                 */
/* mistral/dequant.h:1068-1087: isum = sum_j (q_lo_j - 8) * x_j                */
/*                                   + (q_hi_j - 8) * x_{j+16}                 */
/* ------------------------------------------------------------------------- */
static inline int32_t block_isum(const or_block_q4_0 *w, const or_block_q8_0 *x) {
    int32_t s = 0;
    for (int j = 0; j < 16; j++) {
        int lo = (int)(w->qs[j] & 0x0F) - 8;
        int hi = (int)(w->qs[j] >> 4) - 8;
        s += lo * (int)x->qs[j] + hi * (int)x->qs[j + 16];
    }
    return s;
}

void or_q4q8_block_sums(const void *W, const or_block_q8_0 *x, int32_t *isum,
                        int out_dim, int in_dim) {
    const int bpr = in_dim / 32;
    const or_block_q4_0 *blk = (const or_block_q4_0 *)W;
    for (int r = 0; r < out_dim; r++)
        for (int b = 0; b < bpr; b++)
            isum[(size_t)r * bpr + b] = block_isum(&blk[(size_t)r * bpr + b], &x[b]);
}

static int g_acc_mode = OR_ACC_FMA;
void or_set_acc_mode(int mode) { g_acc_mode = mode; }

/* One output row, blocks in order b = 0..bpr-1 with a sequential fp32 sum:
 * sumf += (wd * xd) * (float)isum  (mistral/dequant.h:1085, per 4-row unroll
 * and tail :1118), contracted to an FMA under -ffast-math. */
static inline float row_dot(const or_block_q4_0 *row, const or_block_q8_0 *x, int bpr) {
    float sumf = 0.0f;
    for (int b = 0; b < bpr; b++) {
        float wd = or_f16_to_f32(row[b].d);
        float xd = x[b].d;
        float s = wd * xd;
        float fi = (float)block_isum(&row[b], &x[b]);
        if (g_acc_mode == OR_ACC_FMA) sumf = fmaf(s, fi, sumf);
        else sumf = sumf + s * fi;
    }
    return sumf;
}

typedef struct {
    const or_block_q4_0 *W;
    const or_block_q8_0 *x;
    float *y;
    int out_dim, bpr, chunk_rows;
} mv_ctx;

static void mv_chunk(void *p, int chunk) {
    mv_ctx *c = (mv_ctx *)p;
    int r0 = chunk * c->chunk_rows;
    int r1 = r0 + c->chunk_rows;
    if (r1 > c->out_dim) r1 = c->out_dim;
    for (int r = r0; r < r1; r++)
        c->y[r] = row_dot(c->W + (size_t)r * c->bpr, c->x, c->bpr);
}

/* Row-parallel matvec -- mistral/dequant.h:1022-1137 (64-row chunks, 32 when
 * in_dim > 8192, atomic work stealing).  The fused QKV / gate-up variants
 * (mistral/mistral_model.h:676-814) compute the same per-row expression. */
void or_matvec_q4_0_q8_0(const void *W, const or_block_q8_0 *x, float *y,
                         int out_dim, int in_dim) {
    mv_ctx c;
    c.W = (const or_block_q4_0 *)W;
    c.x = x;
    c.y = y;
    c.out_dim = out_dim;
    c.bpr = in_dim / 32;
    c.chunk_rows = (in_dim > 8192) ? 32 : 64;
    int n_chunks = (out_dim + c.chunk_rows - 1) / c.chunk_rows;
    parallel_chunks(n_chunks, mv_chunk, &c);
}

/* Q4_0 dequant -- tests/test_cpu_ref.h:236-250 and the Q4_0 branch of
 * embed_token (mistral/mistral_model.h:134-145). */
void or_dequant_q4_0(const void *blocks, float *out, int n) {
    const or_block_q4_0 *b = (const or_block_q4_0 *)blocks;
    for (int i = 0; i < n / 32; i++) {
        float d = or_f16_to_f32(b[i].d);
        for (int j = 0; j < 16; j++) {
            uint8_t v = b[i].qs[j];
            out[i * 32 + j] = d * ((float)(v & 0x0F) - 8.0f);
            out[i * 32 + j + 16] = d * ((float)(v >> 4) - 8.0f);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* RMSNorm -- mistral/mistral_model.h:202-208.  vDSP_dotpr's internal order is  */
/* Apple's; restated as a sequential fused dot.                                */
/* ------------------------------------------------------------------------- */
void or_rmsnorm(float *out, const float *x, const float *w, int dim, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < dim; i++) ss = fmaf(x[i], x[i], ss);
    ss = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = 0; i < dim; i++) out[i] = x[i] * ss;        /* vDSP_vsmul */
    for (int i = 0; i < dim; i++) out[i] = out[i] * w[i];    /* vDSP_vmul */
}

/* RoPE inverse frequencies -- mistral/mistral_model.h:69-74. */
void or_rope_theta(float *theta_inv, int head_dim, float theta) {
    for (int i = 0; i < head_dim / 2; i++)
        theta_inv[i] = 1.0f / powf(theta, (2.0f * (float)i) / (float)head_dim);
}

/* Adjacent-pair RoPE -- mistral/mistral_model.h:79-122.  angle is computed in
 * fp32 as theta_inv[i] * (float)pos (vDSP_vsmul); the rotation uses the NEON
 * fused forms vfmsq(even*c, odd, s) and vfmaq(odd*c, even, s). */
static void rope_heads(float *v, int n_h, int hd, const float *c, const float *s) {
    for (int h = 0; h < n_h; h++) {
        float *vh = v + h * hd;
        for (int i = 0; i < hd / 2; i++) {
            float e = vh[2 * i], o = vh[2 * i + 1];
            vh[2 * i] = fmaf(-o, s[i], e * c[i]);
            vh[2 * i + 1] = fmaf(e, s[i], o * c[i]);
        }
    }
}

void or_apply_rope(float *q, float *k, int pos, const float *theta_inv,
                   int n_heads, int n_kv_heads, int head_dim) {
    float c[256], s[256];
    float fpos = (float)pos;
    for (int i = 0; i < head_dim / 2; i++) {
        float a = theta_inv[i] * fpos;
        s[i] = sinf(a);
        c[i] = cosf(a);
    }
    if (q) rope_heads(q, n_heads, head_dim, c, s);
    if (k) rope_heads(k, n_kv_heads, head_dim, c, s);
}

/* SiLU(gate) * up -- mistral/mistral_model.h:174-199. */
void or_silu_mul(float *gate, const float *up, int n) {
    for (int i = 0; i < n; i++) {
        float e = expf(-gate[i]);
        float sig = 1.0f / (1.0f + e);
        gate[i] = (gate[i] * sig) * up[i];
    }
}

/* In-place softmax -- mistral/mistral_model.h:234-246 (vDSP max, subtract,
 * vvexpf, vDSP_sve, multiply by 1/sum). */
void or_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    for (int i = 0; i < n; i++) x[i] = x[i] - mx;
    for (int i = 0; i < n; i++) x[i] = expf(x[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += x[i];
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] = x[i] * inv;
}

/* q . k for one cached position, in the lane / accumulator order of the NEON
 * loop in mistral/mistral_model.h:395-437: four 4-lane fp32 accumulators,
 * 32 elements per step, combined as ((a0+a1)+(a2+a3)) then pairwise lanes. */
static float qk_dot(const float *q, const uint16_t *k, int hd) {
    float acc[4][4] = {{0}};
    for (int d = 0; d < hd; d += 32) {
        for (int m = 0; m < 8; m++) {
            int a = m & 3;
            for (int l = 0; l < 4; l++)
                acc[a][l] = fmaf(q[d + 4 * m + l], or_f16_to_f32(k[d + 4 * m + l]), acc[a][l]);
        }
    }
    float v[4];
    for (int l = 0; l < 4; l++) {
        float x01 = acc[0][l] + acc[1][l];
        float x23 = acc[2][l] + acc[3][l];
        v[l] = x01 + x23;
    }
    return (v[0] + v[1]) + (v[2] + v[3]);
}

/* GQA decode attention over the fp16 ring -- mistral/mistral_model.h:362-487. */
void or_attention(float *q, float *att, float *out, const uint16_t *kc,
                  const uint16_t *vc, int n_heads, int heads_per_kv, int hd,
                  int max_seq, int pos) {
    int seq_len = (pos + 1 < max_seq) ? pos + 1 : max_seq;
    int ring = (pos + 1 > max_seq);
    int ring_off = ring ? (pos + 1 - seq_len) : 0;
    float inv_sqrt_hd = 1.0f / sqrtf((float)hd);
    for (int i = 0; i < n_heads * hd; i++) q[i] = q[i] * inv_sqrt_hd;
    int n_kv = n_heads / heads_per_kv;
    int kv_dim = n_kv * hd;
    for (int h = 0; h < n_heads; h++) {
        float *qh = q + h * hd;
        float *ah = att + (size_t)h * max_seq;
        int kvh = h / heads_per_kv;
        for (int t = 0; t < seq_len; t++) {
            int ct = ring ? ((ring_off + t) % max_seq) : t;
            ah[t] = qk_dot(qh, kc + (size_t)ct * kv_dim + kvh * hd, hd);
        }
        or_softmax(ah, seq_len);
        float *oh = out + h * hd;
        memset(oh, 0, hd * sizeof(float));
        for (int t = 0; t < seq_len; t++) {
            float a = ah[t];
            if (a == 0.0f) continue;
            int ct = ring ? ((ring_off + t) % max_seq) : t;
            const uint16_t *vt = vc + (size_t)ct * kv_dim + kvh * hd;
            for (int d = 0; d < hd; d++) oh[d] = fmaf(a, or_f16_to_f32(vt[d]), oh[d]);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Model                                                                       */
/* ------------------------------------------------------------------------- */
int or_model_init(or_model *m, int max_seq) {
    const or_config *c = &m->cfg;
    int kv_dim = c->n_kv_heads * c->head_dim;
    m->theta_inv = (float *)malloc(sizeof(float) * (c->head_dim / 2));
    or_rope_theta(m->theta_inv, c->head_dim, c->rope_theta);
    m->att_cap = max_seq;
    m->xb = (float *)calloc(c->dim, 4);
    m->xb2 = (float *)calloc(c->dim, 4);
    m->q = (float *)calloc(c->dim, 4);
    m->k = (float *)calloc(kv_dim, 4);
    m->v = (float *)calloc(kv_dim, 4);
    m->att = (float *)calloc((size_t)c->n_heads * max_seq, 4);
    m->hb = (float *)calloc(c->hidden_dim, 4);
    m->hb2 = (float *)calloc(c->hidden_dim, 4);
    m->logits = (float *)calloc(c->vocab_size, 4);
    m->xb_q8 = (or_block_q8_0 *)calloc(c->dim / 32, sizeof(or_block_q8_0));
    m->hb_q8 = (or_block_q8_0 *)calloc(c->hidden_dim / 32, sizeof(or_block_q8_0));
    return (m->att && m->logits) ? 0 : -1;
}

void or_model_free(or_model *m) {
    free(m->theta_inv); free(m->xb); free(m->xb2); free(m->q); free(m->k); free(m->v);
    free(m->att); free(m->hb); free(m->hb2); free(m->logits); free(m->xb_q8); free(m->hb_q8);
    memset(&m->theta_inv, 0, sizeof(*m) - offsetof(or_model, theta_inv));
}

/* mistral/kv_cache.h:22-35 */
int or_kv_alloc(or_kv *kv, int n_layers, int n_kv_heads, int head_dim, int max_seq) {
    kv->n_layers = n_layers;
    kv->n_kv_heads = n_kv_heads;
    kv->head_dim = head_dim;
    kv->max_seq = max_seq;
    kv->kv_dim = n_kv_heads * head_dim;
    size_t n = (size_t)n_layers * max_seq * kv->kv_dim;
    kv->k = (uint16_t *)calloc(n, 2);
    kv->v = (uint16_t *)calloc(n, 2);
    kv->pos = 0;
    kv->len = 0;
    return (kv->k && kv->v) ? 0 : -1;
}

void or_kv_free(or_kv *kv) { free(kv->k); free(kv->v); kv->k = kv->v = NULL; }

/* ------------------------------------------------------------------------- */
/* K-quants -- mistral/dequant.h                                               */
/* ------------------------------------------------------------------------- */
/* dequant.h:292-306: value n of a super-block: low 4 bits from ql[n % 128] (low nibble for n < 128, high
 * nibble above), high 2 bits from qh[n % 64] at shift 2*(n / 128) + 4*((n % 128) >= 64); q = that - 32;
 * w = d * sc[n / 16] * q, evaluated left to right in fp32. */
static inline float q6k_value(const or_block_q6_K *b, int n) {
    const float d = or_f16_to_f32(b->d);
    const int il = n % 128, is = n / 16, ih = n / 128;
    const uint8_t lo = (n < 128) ? (b->ql[il] & 0xF) : (b->ql[il] >> 4);
    const uint8_t hi = (b->qh[il % 64] >> (2 * ih + (il >= 64 ? 4 : 0))) & 3;
    const int8_t q = (int8_t)((lo | (hi << 4)) - 32);
    return d * b->scales[is] * q;
}

void or_dequant_q6_K(const void *blocks, float *out, int n) {
    const or_block_q6_K *b = (const or_block_q6_K *)blocks;
    for (int i = 0; i < n; i++) out[i] = q6k_value(&b[i / 256], i % 256);
}

/* dequant.h:47-55 */
static inline void q4k_scale_min(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* dequant.h:63-113: per 64-value group j, scale / min pairs (2j, 2j+1) as fp16 products d*sc and dmin*m
 * (fp32 products rounded to fp16); value = fp16(fp16(q * dsc) - dm), q the low nibbles of 32 qs bytes for the
 * first 32 values and their high nibbles for the next 32. */
void or_dequant_q4_K_f16(const void *blocks, uint16_t *out, int n) {
    const or_block_q4_K *bk = (const or_block_q4_K *)blocks;
    for (int blk = 0; blk < n / 256; blk++) {
        const or_block_q4_K *b = &bk[blk];
        const float d = or_f16_to_f32(b->d), dmin = or_f16_to_f32(b->dmin);
        for (int j = 0; j < 4; j++) {
            uint8_t sc1, m1, sc2, m2;
            q4k_scale_min(2 * j, b->scales, &sc1, &m1);
            q4k_scale_min(2 * j + 1, b->scales, &sc2, &m2);
            const float vd1 = or_f16_to_f32(or_f32_to_f16(d * sc1)), vm1 = or_f16_to_f32(or_f32_to_f16(dmin * m1));
            const float vd2 = or_f16_to_f32(or_f32_to_f16(d * sc2)), vm2 = or_f16_to_f32(or_f32_to_f16(dmin * m2));
            for (int i = 0; i < 32; i++) {
                const uint8_t byte = b->qs[32 * j + i];
                const float lo = or_f16_to_f32(or_f32_to_f16((float)(byte & 0xF) * vd1));
                const float hi = or_f16_to_f32(or_f32_to_f16((float)(byte >> 4) * vd2));
                out[blk * 256 + 64 * j + i] = or_f32_to_f16(lo - vm1);
                out[blk * 256 + 64 * j + 32 + i] = or_f32_to_f16(hi - vm2);
            }
        }
    }
}

typedef struct {
    int type;
    const uint8_t *W;
    const float *x;
    float *y;
    int in_dim;
    size_t row_bytes;
} kq_job;

static void kq_rows(void *ctx, int r) {
    const kq_job *j = (const kq_job *)ctx;
    const uint8_t *row = j->W + (size_t)r * j->row_bytes;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int b = 0; b < j->in_dim / 256; b++) {
        float w[256];
        if (j->type == OR_TYPE_Q6_K) {
            const or_block_q6_K *blk = (const or_block_q6_K *)row + b;
            /* dequant.h:337-352: w = (float)q * (d * sc), exact in fp32 (q 6 bits, d * sc at most 18) */
            for (int n = 0; n < 256; n++) w[n] = q6k_value(blk, n);
        } else {
            uint16_t h[256];
            or_dequant_q4_K_f16((const or_block_q4_K *)row + b, h, 256);
            for (int n = 0; n < 256; n++) w[n] = or_f16_to_f32(h[n]);
        }
        const float *xb = j->x + (size_t)b * 256;
        for (int n = 0; n < 256; n++) acc[n & 3] = fmaf(w[n], xb[n], acc[n & 3]);
    }
    j->y[r] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

void or_matvec_kq_f32(int type, const void *W, const float *x, float *y, int rows, int in_dim) {
    kq_job j = {type, (const uint8_t *)W, x, y, in_dim,
                (size_t)(in_dim / 256) * (type == OR_TYPE_Q6_K ? sizeof(or_block_q6_K) : sizeof(or_block_q4_K))};
    parallel_chunks(rows, kq_rows, &j);
}

/* mistral/mistral_model.h:125-157 (Q4_0 and Q4_K branches). */
void or_embed_token(const or_model *m, int token, float *out) {
    int dim = m->cfg.dim;
    if (m->tok_embd_type == OR_TYPE_Q4_K) {
        uint16_t h[256];
        const or_block_q4_K *row = (const or_block_q4_K *)m->tok_embd + (size_t)token * (dim / 256);
        for (int b = 0; b < dim / 256; b++) {
            or_dequant_q4_K_f16(row + b, h, 256);
            for (int i = 0; i < 256; i++) out[b * 256 + i] = or_f16_to_f32(h[i]);
        }
        return;
    }
    const or_block_q4_0 *row = (const or_block_q4_0 *)m->tok_embd + (size_t)token * (dim / 32);
    or_dequant_q4_0(row, out, dim);
}

/* Decode layer -- mistral/mistral_model.h:818-899. */
void or_layer_decode(or_model *m, or_kv *kv, float *x, int layer, int pos) {
    const or_config *c = &m->cfg;
    const or_layer *lw = &m->layers[layer];
    int dim = c->dim, kv_dim = c->n_kv_heads * c->head_dim, hidden = c->hidden_dim;
    int hd = c->head_dim, hpkv = c->n_heads / c->n_kv_heads;

    or_rmsnorm(m->xb, x, lw->rms_att, dim, c->rms_eps);                 /* 1 */
    or_quantize_q8_0(m->xb, m->xb_q8, dim, OR_QUANT_IEEE);               /* 2 */
    or_matvec_q4_0_q8_0(lw->wq, m->xb_q8, m->q, dim, dim);               /* 3 */
    or_matvec_q4_0_q8_0(lw->wk, m->xb_q8, m->k, kv_dim, dim);
    or_matvec_q4_0_q8_0(lw->wv, m->xb_q8, m->v, kv_dim, dim);
    or_apply_rope(m->q, m->k, pos, m->theta_inv, c->n_heads, c->n_kv_heads, hd);  /* 4 */
    int slot = pos % kv->max_seq;                                        /* 5 */
    uint16_t *kd = kv->k + ((size_t)layer * kv->max_seq + slot) * kv_dim;
    uint16_t *vd = kv->v + ((size_t)layer * kv->max_seq + slot) * kv_dim;
    for (int i = 0; i < kv_dim; i++) { kd[i] = or_f32_to_f16(m->k[i]); vd[i] = or_f32_to_f16(m->v[i]); }
    if (kv->len < kv->max_seq && pos + 1 > kv->len) kv->len = pos + 1;
    or_attention(m->q, m->att, m->xb2,                                   /* 6 */
                 kv->k + (size_t)layer * kv->max_seq * kv_dim,
                 kv->v + (size_t)layer * kv->max_seq * kv_dim,
                 c->n_heads, hpkv, hd, kv->max_seq, pos);
    or_quantize_q8_0(m->xb2, m->xb_q8, dim, OR_QUANT_IEEE);              /* 7 */
    or_matvec_q4_0_q8_0(lw->wo, m->xb_q8, m->xb, dim, dim);
    for (int i = 0; i < dim; i++) x[i] = x[i] + m->xb[i];               /* 8 */
    or_rmsnorm(m->xb, x, lw->rms_ffn, dim, c->rms_eps);                  /* 9 */
    or_quantize_q8_0(m->xb, m->xb_q8, dim, OR_QUANT_IEEE);               /* 10 */
    or_matvec_q4_0_q8_0(lw->w1, m->xb_q8, m->hb, hidden, dim);           /* 11 */
    or_matvec_q4_0_q8_0(lw->w3, m->xb_q8, m->hb2, hidden, dim);
    or_silu_mul(m->hb, m->hb2, hidden);
    or_quantize_q8_0(m->hb, m->hb_q8, hidden, OR_QUANT_IEEE);
    or_matvec_q4_0_q8_0(lw->w2, m->hb_q8, m->xb, dim, hidden);
    for (int i = 0; i < dim; i++) x[i] = x[i] + m->xb[i];               /* 12 */
}

/* mistral/mistral_model.h:1110-1122 */
void or_logits(or_model *m, const float *x) {
    or_rmsnorm(m->xb, x, m->rms_final, m->cfg.dim, m->cfg.rms_eps);
    if (m->lm_head_type == OR_TYPE_Q6_K || m->lm_head_type == OR_TYPE_Q4_K) {
        /* non-Q4_0 LM head: the fp32 path on the normalised state (mistral_model.h:1118-1121) */
        or_matvec_kq_f32(m->lm_head_type, m->lm_head, m->xb, m->logits, m->cfg.vocab_size, m->cfg.dim);
        return;
    }
    or_quantize_q8_0(m->xb, m->xb_q8, m->cfg.dim, OR_QUANT_IEEE);
    or_matvec_q4_0_q8_0(m->lm_head, m->xb_q8, m->logits, m->cfg.vocab_size, m->cfg.dim);
}

/* ------------------------------------------------------------------------- */
/* Philox4x32-10 (Salmon et al., SC'11) -- seeded replacement for arc4random. */
/* ------------------------------------------------------------------------- */
static inline void mulhilo32(uint32_t a, uint32_t b, uint32_t *hi, uint32_t *lo) {
    uint64_t p = (uint64_t)a * b;
    *hi = (uint32_t)(p >> 32);
    *lo = (uint32_t)p;
}

uint32_t or_philox_u32(uint64_t seed, uint64_t counter) {
    uint32_t c0 = (uint32_t)counter, c1 = (uint32_t)(counter >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
    for (int r = 0; r < 10; r++) {
        uint32_t hi0, lo0, hi1, lo1;
        mulhilo32(0xD2511F53u, c0, &hi0, &lo0);
        mulhilo32(0xCD9E8D57u, c2, &hi1, &lo1);
        uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

uint32_t or_rng_next(or_rng *r) { return or_philox_u32(r->seed, r->counter++); }

/* (float)arc4random() / (float)UINT32_MAX -- speculative.h:61, mistral_model.h:1228 */
float or_rng_uniform(or_rng *r) { return (float)or_rng_next(r) / (float)UINT32_MAX; }

/* ------------------------------------------------------------------------- */
/* Sampling -- mistral/mistral_model.h:1136-1240                               */
/* ------------------------------------------------------------------------- */
int or_sample_argmax(const float *logits, int n) {
    int best = 0;
    float bv = logits[0];
    for (int i = 1; i < n; i++)
        if (logits[i] > bv) { bv = logits[i]; best = i; }
    return best;
}

static inline void swap_kv(float *v, int *ix, int a, int b) {
    float tv = v[a]; v[a] = v[b]; v[b] = tv;
    int ti = ix[a]; ix[a] = ix[b]; ix[b] = ti;
}

int or_sample_token(float *logits, int n, const or_sample_params *p, or_rng *rng) {
    /* repetition penalty, once per occurrence in the window (:1147-1158) */
    if (p->rep_penalty != 1.0f && p->prev_tokens && p->n_prev > 0) {
        for (int i = 0; i < p->n_prev; i++) {
            int t = p->prev_tokens[i];
            if (t < 0 || t >= n) continue;
            if (logits[t] > 0) logits[t] /= p->rep_penalty;
            else logits[t] *= p->rep_penalty;
        }
    }
    if (p->temp <= 0) return or_sample_argmax(logits, n);

    int top_k = p->top_k > 0 ? p->top_k : 40;
    if (top_k > n) top_k = n;
    int *ix = (int *)malloc(sizeof(int) * top_k);
    float *v = (float *)malloc(sizeof(float) * top_k);
    float *pr = (float *)malloc(sizeof(float) * top_k);
    /* ascending partial selection (:1165-1191): fill, sort once full, then
     * replace the minimum and bubble it up */
    int k = 0;
    for (int i = 0; i < n; i++) {
        if (k < top_k) {
            ix[k] = i; v[k] = logits[i]; k++;
            if (k == top_k)
                for (int a = 0; a < top_k; a++)
                    for (int b = a + 1; b < top_k; b++)
                        if (v[a] > v[b]) swap_kv(v, ix, a, b);
        } else if (logits[i] > v[0]) {
            v[0] = logits[i]; ix[0] = i;
            for (int a = 0; a < top_k - 1; a++) {
                if (v[a] > v[a + 1]) swap_kv(v, ix, a, a + 1);
                else break;
            }
        }
    }
    /* descending sort for top-p (:1194-1199) */
    for (int a = 0; a < top_k - 1; a++)
        for (int b = a + 1; b < top_k; b++)
            if (v[a] < v[b]) swap_kv(v, ix, a, b);
    /* tempered softmax over top-k (:1202-1208) */
    float mx = v[0], sum = 0.0f;
    for (int i = 0; i < top_k; i++) { pr[i] = expf((v[i] - mx) / p->temp); sum += pr[i]; }
    for (int i = 0; i < top_k; i++) pr[i] /= sum;
    /* nucleus cut + renormalise (:1211-1224) */
    int eff = top_k;
    if (p->top_p > 0 && p->top_p < 1.0f) {
        float cum = 0.0f;
        for (int i = 0; i < top_k; i++) {
            cum += pr[i];
            if (cum >= p->top_p) { eff = i + 1; break; }
        }
        sum = 0.0f;
        for (int i = 0; i < eff; i++) sum += pr[i];
        for (int i = 0; i < eff; i++) pr[i] /= sum;
    }
    /* linear CDF draw (:1227-1234) */
    float r = or_rng_uniform(rng);
    float cdf = 0.0f;
    int res = ix[0];
    for (int i = 0; i < eff; i++) {
        cdf += pr[i];
        if (r < cdf) { res = ix[i]; break; }
    }
    free(ix); free(v); free(pr);
    return res;
}

/* ------------------------------------------------------------------------- */
/* Speculative decoding -- mistral/speculative.h                               */
/* ------------------------------------------------------------------------- */
/* speculative.h:37-57 */
void or_spec_softmax(const float *logits, float *probs, int n, float temperature) {
    float mx = logits[0];
    for (int i = 1; i < n; i++) if (logits[i] > mx) mx = logits[i];
    float inv_t = (temperature > 0) ? 1.0f / temperature : 0.0f;
    for (int i = 0; i < n; i++) probs[i] = (logits[i] - mx) * inv_t;
    for (int i = 0; i < n; i++) probs[i] = expf(probs[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += probs[i];
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) probs[i] = probs[i] * inv;
}

/* speculative.h:60-68 */
int or_spec_sample_probs(const float *probs, int n, or_rng *rng) {
    float r = or_rng_uniform(rng);
    float cdf = 0.0f;
    for (int i = 0; i < n; i++) {
        cdf += probs[i];
        if (r < cdf) return i;
    }
    return n - 1;
}

/* speculative.h:121-198 */
int or_spec_accept(const float *draft_probs, const float *target_logits,
                   const int *draft_tokens, int n_draft, int vocab, float temperature,
                   int *accepted, or_rng *rng) {
    if (temperature <= 0.0f) {
        for (int i = 0; i < n_draft; i++) {
            int t = or_sample_argmax(target_logits + (size_t)i * vocab, vocab);
            accepted[i] = t;
            if (t != draft_tokens[i]) return i + 1;
        }
        /* bonus from index n_draft-1 (the caller overrides it, :312-317) */
        accepted[n_draft] = or_sample_argmax(target_logits + (size_t)(n_draft - 1) * vocab, vocab);
        return n_draft + 1;
    }
    float *p = (float *)malloc(sizeof(float) * vocab);
    float *adj = (float *)malloc(sizeof(float) * vocab);
    for (int i = 0; i < n_draft; i++) {
        or_spec_softmax(target_logits + (size_t)i * vocab, p, vocab, temperature);
        int tok = draft_tokens[i];
        float p_tok = p[tok], q_tok = draft_probs[i];
        float ap = (q_tok > 0) ? fminf(1.0f, p_tok / q_tok) : 0.0f;
        float r = or_rng_uniform(rng);
        if (r < ap) {
            accepted[i] = tok;
        } else {
            float sum_adj = 0.0f;
            for (int v = 0; v < vocab; v++) {
                float qv = (v == tok) ? q_tok : 0.0f;
                adj[v] = fmaxf(0.0f, p[v] - qv);
                sum_adj += adj[v];
            }
            if (sum_adj > 0) {
                float inv = 1.0f / sum_adj;
                for (int v = 0; v < vocab; v++) adj[v] *= inv;
            } else {
                memcpy(adj, p, sizeof(float) * vocab);
            }
            accepted[i] = or_spec_sample_probs(adj, vocab, rng);
            free(p); free(adj);
            return i + 1;
        }
    }
    or_spec_softmax(target_logits + (size_t)(n_draft - 1) * vocab, p, vocab, temperature);
    accepted[n_draft] = or_spec_sample_probs(p, vocab, rng);
    free(p); free(adj);
    return n_draft + 1;
}

/* N-gram drafter -- speculative.h:387-464 */
int or_ngram_init(or_ngram *d, const int *prompt, int n_prompt, int ngram_n, int max_draft) {
    d->ngram_n = (ngram_n > 0) ? ngram_n : 3;
    d->max_draft = (max_draft > 0) ? max_draft : 4;
    if (d->max_draft > OR_SPEC_MAX_DRAFT) d->max_draft = OR_SPEC_MAX_DRAFT;
    d->history_cap = n_prompt + 4096;
    d->history = (int *)malloc(sizeof(int) * d->history_cap);
    if (!d->history) return -1;
    memcpy(d->history, prompt, sizeof(int) * n_prompt);
    d->history_len = n_prompt;
    return 0;
}

void or_ngram_push(or_ngram *d, int token) {
    if (d->history_len >= d->history_cap) {
        d->history_cap *= 2;
        d->history = (int *)realloc(d->history, sizeof(int) * d->history_cap);
    }
    d->history[d->history_len++] = token;
}

void or_ngram_free(or_ngram *d) { free(d->history); d->history = NULL; }

int or_ngram_scan(const int *history, int hlen, int ngram_n, int max_draft,
                  int current_token, int *draft_tokens, int *match_pos_out) {
    int n = ngram_n;
    if (match_pos_out) *match_pos_out = -1;
    if (hlen < n) return 0;
    int plen = n > 16 ? 16 : n;
    int pattern[16];
    for (int i = 0; i < plen - 1; i++) pattern[i] = history[hlen - plen + 1 + i];
    pattern[plen - 1] = current_token;
    int match = -1;
    for (int i = 0; i <= hlen - plen - 1; i++) {   /* earliest match, tail skipped */
        int ok = 1;
        for (int j = 0; j < plen; j++)
            if (history[i + j] != pattern[j]) { ok = 0; break; }
        if (ok) { match = i + plen; break; }
    }
    if (match < 0) return 0;
    if (match_pos_out) *match_pos_out = match;
    int nd = 0;
    for (int i = match; i < hlen && nd < max_draft; i++, nd++) draft_tokens[nd] = history[i];
    return nd;
}

int or_ngram_draft(const or_ngram *d, int current_token, int *draft_tokens, float *draft_probs) {
    int nd = or_ngram_scan(d->history, d->history_len, d->ngram_n, d->max_draft,
                           current_token, draft_tokens, NULL);
    for (int i = 0; i < nd; i++) draft_probs[i] = 0.9f;
    return nd;
}

/* ------------------------------------------------------------------------- */
/* Whole-token forward helpers                                                 */
/* ------------------------------------------------------------------------- */
static float *g_x = NULL;
static int g_x_cap = 0;
static float *xbuf(int dim) {
    if (g_x_cap < dim) { free(g_x); g_x = (float *)malloc(sizeof(float) * dim); g_x_cap = dim; }
    return g_x;
}

/* embed -> n_layers decode layers -> logits (mistral_infer.m:694-699) */
static void forward_token_kv(or_model *m, or_kv *kv, int token, int pos, int n_layers) {
    float *x = xbuf(m->cfg.dim);
    or_embed_token(m, token, x);
    for (int l = 0; l < n_layers; l++) or_layer_decode(m, kv, x, l, pos);
    or_logits(m, x);
}

static or_kv g_fwd_kv;   /* KV used by or_forward_token (tests drive it directly) */
void or_forward_token(or_model *m, or_kv *kv, int token, int pos, int n_layers) {
    forward_token_kv(m, kv ? kv : &g_fwd_kv, token, pos, n_layers);
}

void or_prefill(or_model *m, or_kv *kv, const int *tokens, int n, int n_layers, float *x_out) {
    float *x = xbuf(m->cfg.dim);
    for (int t = 0; t < n; t++) {
        or_embed_token(m, tokens[t], x);
        for (int l = 0; l < n_layers; l++) or_layer_decode(m, kv, x, l, t);
    }
    if (x_out) memcpy(x_out, x, sizeof(float) * m->cfg.dim);
}

/* Prompt prefill + first-token sample with repetition penalty over the prompt
 * window (mistral_infer.m:594-621). Returns the first token. */
static int start_generation(or_model *m, or_kv *kv, const int *prompt, int n_prompt,
                            const or_gen_opts *o, int *hist, int *n_hist, or_rng *rng) {
    int dim = m->cfg.dim, vocab = m->cfg.vocab_size;
    float *x = (float *)malloc(sizeof(float) * dim);
    or_prefill(m, kv, prompt, n_prompt, m->cfg.n_layers, x);
    or_logits(m, x);
    free(x);
    memcpy(hist, prompt, sizeof(int) * n_prompt);
    *n_hist = n_prompt;
    float *lb = (float *)malloc(sizeof(float) * vocab);
    memcpy(lb, m->logits, sizeof(float) * vocab);
    int hs = *n_hist > o->rep_window ? *n_hist - o->rep_window : 0;
    or_sample_params sp = { o->temp, o->top_k, o->top_p, o->rep_penalty, hist + hs, *n_hist - hs };
    int t = or_sample_token(lb, vocab, &sp, rng);
    free(lb);
    hist[(*n_hist)++] = t;
    return t;
}

static int is_stop(const or_gen_opts *o, int tok) { return !o->ignore_eos && tok == o->eos_id; }

/* Greedy / normal decode loop -- mistral_infer.m:690-716. */
int or_generate_greedy(or_model *m, const int *prompt, int n_prompt,
                       const or_gen_opts *o, int *out, or_gen_stats *st) {
    int vocab = m->cfg.vocab_size;
    or_kv kv;
    if (or_kv_alloc(&kv, m->cfg.n_layers, m->cfg.n_kv_heads, m->cfg.head_dim, o->max_seq)) return -1;
    or_rng rng = { o->seed, 0 };
    int *hist = (int *)malloc(sizeof(int) * (n_prompt + o->max_tokens + 16));
    int n_hist = 0;
    int next = start_generation(m, &kv, prompt, n_prompt, o, hist, &n_hist, &rng);
    int n_out = 0;
    out[n_out++] = next;
    float *lb = (float *)malloc(sizeof(float) * vocab);
    for (int t = 0; t < o->max_tokens; t++) {
        if (is_stop(o, next)) break;
        int pos = n_prompt + t;
        forward_token_kv(m, &kv, next, pos, m->cfg.n_layers);
        memcpy(lb, m->logits, sizeof(float) * vocab);
        int hs = n_hist > o->rep_window ? n_hist - o->rep_window : 0;
        or_sample_params sp = { o->temp, o->top_k, o->top_p, o->rep_penalty, hist + hs, n_hist - hs };
        next = or_sample_token(lb, vocab, &sp, &rng);
        hist[n_hist++] = next;
        out[n_out++] = next;
    }
    free(lb); free(hist); or_kv_free(&kv);
    if (st) { memset(st, 0, sizeof(*st)); st->n_generated = n_out; }
    return n_out;
}

/* Bonus token when every draft was accepted (speculative.h:312-317,
 * mistral_infer.m:332-337).  OR_BONUS_REFERENCE keeps the reference: sample
 * from spec_softmax(logits[n_draft], temp), which at temp 0 is uniform.
 * OR_BONUS_ARGMAX uses argmax at temp <= 0. */
static int bonus_token(const or_gen_opts *o, const float *logits, int vocab, or_rng *rng) {
    if (o->temp <= 0.0f && o->bonus_mode == OR_BONUS_ARGMAX) return or_sample_argmax(logits, vocab);
    float *bp = (float *)malloc(sizeof(float) * vocab);
    or_spec_softmax(logits, bp, vocab, o->temp);
    int t = or_spec_sample_probs(bp, vocab, rng);
    free(bp);
    return t;
}

/* Sequential verify -- speculative.h:81-105 */
static void verify_seq(or_model *m, or_kv *kv, const int *tokens, int n, int start_pos,
                       float *logits_out) {
    int vocab = m->cfg.vocab_size;
    for (int i = 0; i < n; i++) {
        forward_token_kv(m, kv, tokens[i], start_pos + i, m->cfg.n_layers);
        memcpy(logits_out + (size_t)i * vocab, m->logits, sizeof(float) * vocab);
    }
}

/* N-gram speculative loop -- mistral_infer.m:252-391, verify restated as the
 * CPU W4A8 forward (the Metal verify is W4A32; parity targets the CPU path). */
int or_generate_ngram(or_model *m, const int *prompt, int n_prompt,
                      const or_gen_opts *o, int *out, or_gen_stats *st) {
    int vocab = m->cfg.vocab_size;
    or_kv kv;
    if (or_kv_alloc(&kv, m->cfg.n_layers, m->cfg.n_kv_heads, m->cfg.head_dim, o->max_seq)) return -1;
    or_rng rng = { o->seed, 0 };
    int cap = n_prompt + o->max_tokens + 2 * OR_SPEC_MAX_DRAFT + 16;
    int *hist = (int *)malloc(sizeof(int) * cap);
    int n_hist = 0;
    int first = start_generation(m, &kv, prompt, n_prompt, o, hist, &n_hist, &rng);
    int n_out = 0;
    out[n_out++] = first;

    or_ngram dr;
    or_ngram_init(&dr, hist, n_hist, o->ngram_n, o->spec_k);
    or_gen_stats s; memset(&s, 0, sizeof(s));
    int K = dr.max_draft;
    float *all = (float *)malloc(sizeof(float) * (size_t)(K + 1) * vocab);
    float *lb = (float *)malloc(sizeof(float) * vocab);
    int cur = first, pos = n_prompt, gen = 0, limit = o->max_tokens - 1;
    int dtok[OR_SPEC_MAX_DRAFT], acc[OR_SPEC_MAX_DRAFT + 1];
    float dprob[OR_SPEC_MAX_DRAFT];
    while (gen < limit) {
        if (is_stop(o, cur)) break;
        /* history includes the current token (reference wiring) or not */
        int hlen = o->history_has_current ? dr.history_len : dr.history_len - 1;
        int nd = or_ngram_scan(dr.history, hlen, dr.ngram_n, dr.max_draft, cur, dtok, NULL);
        for (int i = 0; i < nd; i++) dprob[i] = 0.9f;
        if (nd <= 0) {
            forward_token_kv(m, &kv, cur, pos, m->cfg.n_layers);
            memcpy(lb, m->logits, sizeof(float) * vocab);
            int hs = n_hist > o->rep_window ? n_hist - o->rep_window : 0;
            or_sample_params sp = { o->temp, o->top_k, o->top_p, o->rep_penalty, hist + hs, n_hist - hs };
            cur = or_sample_token(lb, vocab, &sp, &rng);
            or_ngram_push(&dr, cur);
            hist[n_hist++] = cur;
            out[n_out++] = cur;
            pos++; gen++; s.total_iterations++;
            continue;
        }
        int vt[OR_SPEC_MAX_DRAFT + 1];
        vt[0] = cur;
        memcpy(vt + 1, dtok, sizeof(int) * nd);
        verify_seq(m, &kv, vt, nd + 1, pos, all);
        int na = or_spec_accept(dprob, all, dtok, nd, vocab, o->temp, acc, &rng);
        if (na == nd + 1) acc[nd] = bonus_token(o, all + (size_t)nd * vocab, vocab, &rng);
        int stop = 0;
        for (int i = 0; i < na; i++) {
            or_ngram_push(&dr, acc[i]);
            hist[n_hist++] = acc[i];
            out[n_out++] = acc[i];
            if (is_stop(o, acc[i])) { gen += i + 1; stop = 1; break; }
        }
        if (stop) break;
        s.total_draft += nd; s.total_accepted += na; s.total_iterations++;
        pos += na;
        cur = acc[na - 1];
        gen += na;
    }
    free(all); free(lb); free(hist); or_ngram_free(&dr); or_kv_free(&kv);
    s.n_generated = n_out;
    if (st) *st = s;
    return n_out;
}

/* Self-speculative loop -- mistral_infer.m:660-689 + speculative.h:217-379
 * with the truncated-depth drafter of speculative.h:479-538. */
int or_generate_self_spec(or_model *m, const int *prompt, int n_prompt,
                          const or_gen_opts *o, int *out, or_gen_stats *st) {
    int vocab = m->cfg.vocab_size, nl = m->cfg.n_layers;
    int L = o->draft_layers < 1 ? 1 : o->draft_layers;
    if (L >= nl) L = nl - 1;
    int K = o->spec_k < 1 ? 1 : (o->spec_k > OR_SPEC_MAX_DRAFT ? OR_SPEC_MAX_DRAFT : o->spec_k);
    or_kv kv, dkv;
    if (or_kv_alloc(&kv, nl, m->cfg.n_kv_heads, m->cfg.head_dim, o->max_seq)) return -1;
    if (or_kv_alloc(&dkv, L, m->cfg.n_kv_heads, m->cfg.head_dim, o->max_seq)) return -1;
    or_rng rng = { o->seed, 0 };
    int *hist = (int *)malloc(sizeof(int) * (n_prompt + o->max_tokens + 2 * OR_SPEC_MAX_DRAFT + 16));
    int n_hist = 0;
    int first = start_generation(m, &kv, prompt, n_prompt, o, hist, &n_hist, &rng);
    int n_out = 0;
    out[n_out++] = first;
    /* draft prefill through the first L layers (mistral_infer.m:675-681) */
    or_prefill(m, &dkv, prompt, n_prompt, L, NULL);
    dkv.len = n_prompt;

    or_gen_stats s; memset(&s, 0, sizeof(s));
    float *all = (float *)malloc(sizeof(float) * (size_t)(K + 1) * vocab);
    int cur = first, pos = n_prompt, gen = 0, limit = o->max_tokens - 1;
    int dtok[OR_SPEC_MAX_DRAFT], acc[OR_SPEC_MAX_DRAFT + 1];
    float dprob[OR_SPEC_MAX_DRAFT];
    while (gen < limit) {
        if (is_stop(o, cur)) break;
        /* self_spec_draft_fn (speculative.h:511-538) */
        if (dkv.len > pos) dkv.len = pos;
        int tok = cur;
        for (int k = 0; k < K; k++) {
            forward_token_kv(m, &dkv, tok, pos + k, L);
            int nx = or_sample_argmax(m->logits, vocab);
            dtok[k] = nx;
            dprob[k] = 1.0f;
            tok = nx;
        }
        int nd = K;
        int vt[OR_SPEC_MAX_DRAFT + 1];
        vt[0] = cur;
        memcpy(vt + 1, dtok, sizeof(int) * nd);
        verify_seq(m, &kv, vt, nd + 1, pos, all);
        int na = or_spec_accept(dprob, all, dtok, nd, vocab, o->temp, acc, &rng);
        if (na == nd + 1) acc[nd] = bonus_token(o, all + (size_t)nd * vocab, vocab, &rng);
        int stop = 0;
        for (int i = 0; i < na; i++) {
            out[n_out++] = acc[i];
            if (is_stop(o, acc[i])) { gen += i + 1; stop = 1; break; }
        }
        if (stop) break;
        s.total_draft += nd; s.total_accepted += na; s.total_iterations++;
        pos += na;
        cur = acc[na - 1];
        gen += na;
    }
    free(all); free(hist); or_kv_free(&kv); or_kv_free(&dkv);
    s.n_generated = n_out;
    if (st) *st = s;
    return n_out;
}
