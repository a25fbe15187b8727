/* Test program: the drop-in headers (include/compat) compile as C, link against libspecdec_b200.so and run
 * the reference-signature entry points with the reference's argument lists.  Prints one line per check
 * (tests/test_gpu_boundary.py parses them); exit code 0 = all ran.  Without a GPU it only checks that the
 * calls fail cleanly. */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "compat/dequant.h"
#include "compat/gguf_loader.h"
#include "compat/kv_cache.h"
#include "compat/mistral_model.h"
#include "compat/metal_matvec.h"
#include "compat/speculative.h"
#include "compat/tokenizer.h"

static int argmax_row(const float *x, int n) {
    int b = 0;
    for (int i = 1; i < n; i++)
        if (x[i] > x[b]) b = i;
    return b;
}

/* Greedy decode of n tokens after the prompt (positions [0, start) already in the ring), the reference's
 * non-speculative loop shape: one forward, argmax, print. */
static void greedy_pieces(MistralModel *m, KVCache *kv, Tokenizer *tok, int first, int start, int n) {
    float *lg = malloc(sizeof(float) * m->cfg.vocab_size);
    int cur = first;
    for (int i = 0; i < n; i++) {
        spec_verify(m, kv, &cur, 1, start + i, lg);
        cur = sample_argmax(lg, m->cfg.vocab_size);
        printf("%s", tokenizer_decode_token(tok, cur));
        if (cur == tok->eos_id) break;
    }
    free(lg);
}

int main(int argc, char **argv) {
    if (sd_device_count() == 0) {
        sd_ctx *c = NULL;
        int rc = sd_ctx_create_file("/nonexistent.gguf", NULL, &c);
        printf("no-device rc=%d\n", rc);
        return rc < 0 ? 0 : 1;
    }
    const int n = 4096, rows = 1024;
    float *x = malloc(sizeof(float) * n);
    for (int i = 0; i < n; i++) x[i] = sinf(0.37f * i) * (1 + i % 7);
    block_q8_0 *xq = malloc(sizeof(block_q8_0) * (n / 32));
    quantize_f32_to_q8_0(x, xq, n);
    block_q4_0 *W = malloc(sizeof(block_q4_0) * rows * (n / 32));
    for (int i = 0; i < rows * (n / 32); i++) {
        W[i].d = 0x2000 + (i % 97);  /* small positive fp16 */
        for (int j = 0; j < 16; j++) W[i].qs[j] = (unsigned char)(i * 31 + j * 7);
    }
    float *y = malloc(sizeof(float) * rows);
    q4_0_q8_0_matvec_sdot_parallel(W, xq, y, rows, n);
    printf("q8 d0=%.9g q0=%d y0=%.9g y%d=%.9g\n", xq[0].d, xq[0].qs[0], y[0], rows - 1, y[rows - 1]);
    int hist[] = {1, 2, 3, 4, 9, 9, 1, 2, 3, 4, 5, 6};
    NGramDraft *d = ngram_draft_init(hist, 12, 3, 4);
    SpeculativeState s;
    spec_state_init(&s);
    int nd = ngram_draft_fn(d, NULL, NULL, 3, 0, 0.0f, &s);
    printf("ngram n=%d first=%d\n", nd, nd > 0 ? s.draft_tokens[0] : -1);
    ngram_draft_free(d);
    if (argc < 2) return 0;

    /* gguf_loader.h / tokenizer.h */
    GGUFFile *g = gguf_open(argv[1]);
    if (!g) return 3;
    Tokenizer *tok = tokenizer_init(g);
    if (!tok) return 3;
    int ids[64];
    char *chat = tokenizer_apply_chat("hello world");
    int nt = tokenizer_encode(tok, chat, ids, 64, 1);
    char *dec = tokenizer_decode(tok, ids, nt);
    printf("tokenizer vocab=%d bos=%d eos=%d n=%d chat=[%s] decoded=[%s]\n", tok->vocab_size, tok->bos_id, tok->eos_id,
           nt, chat, dec);
    free(chat);
    free(dec);

    /* mistral_model.h + metal_matvec.h on one context */
    MistralModel *m = mistral_load_context(argv[1], 512);
    if (!m) return 4;
    const MistralConfig *cfg = &m->cfg;
    const int V = cfg->vocab_size;
    KVCache kv = kv_alloc(cfg->n_layers, cfg->n_kv_heads, cfg->head_dim, 512);
    MetalContext *mc = metal_context_init(m->gguf->mmap_base, m->gguf->mmap_len, cfg->dim, cfg->n_kv_heads * cfg->head_dim,
                                          cfg->hidden_dim, V, cfg->n_heads, cfg->n_layers, 512);
    if (!mc) return 4;
    metal_wire_kv_cache(mc, &kv);
    printf("metal shared=%d batch5=%d batch9=%d batch17=%d\n", mc == m->ctx, metal_alloc_batch_buffers(mc, 5, 0, 0, 0, 0, 512),
           metal_alloc_batch_buffers(mc, 9, 0, 0, 0, 0, 512), metal_alloc_batch_buffers(mc, 17, 0, 0, 0, 0, 512));

    /* prompt of repeated segments (the n-gram drafter finds matches), prefilled through spec_verify */
    int prompt[24];
    for (int i = 0; i < 24; i++) prompt[i] = 5 + (i % 8) * 3;
    float *lg = malloc(sizeof(float) * (size_t)24 * V);
    int rc = spec_verify(m, &kv, prompt, 24, 0, lg);
    const int first = argmax_row(lg + (size_t)23 * V, V);
    printf("prefill rc=%d kvlen=%d first=%d\n", rc, kv.len, first);

    /* embed_token / mistral_layer_decode_parallel / mistral_logits vs the batched forward of the same token */
    float *xs = malloc(sizeof(float) * cfg->dim);
    embed_token(m, first, xs);
    for (int l = 0; l < cfg->n_layers; l++) mistral_layer_decode_parallel(m, &kv, xs, l, 24);
    mistral_logits(m, xs);
    float *ref = malloc(sizeof(float) * V);
    spec_verify(m, &kv, &first, 1, 24, ref);
    double md = 0, mx = 0;
    for (int v = 0; v < V; v++) {
        md = fmax(md, fabs((double)m->logits[v] - ref[v]));
        mx = fmax(mx, fabs((double)ref[v]));
    }
    printf("layer_path rel=%.3g argmax=%d/%d\n", md / mx, sample_argmax(m->logits, V), argmax_row(ref, V));

    /* sampling: sample_token (temperature, top-k, top-p, repetition penalty), sample_temperature, spec_softmax,
     * spec_sample_probs */
    spec_rng_seed(7);
    SampleParams sp = {0.7f, 40, 0.9f, 1.1f, prompt, 24};
    float *tmp = malloc(sizeof(float) * V);
    memcpy(tmp, ref, sizeof(float) * V);
    int st = sample_token(tmp, V, &sp);
    int stt = sample_temperature(ref, V, 0.7f);
    float *pr = malloc(sizeof(float) * V);
    spec_softmax(ref, pr, V, 0.7f);
    double psum = 0;
    for (int v = 0; v < V; v++) psum += pr[v];
    int sp_i = spec_sample_probs(pr, V);
    printf("sample token=%d temperature=%d softmax_sum=%.6f probs_draw=%d in_range=%d\n", st, stt, psum, sp_i,
           st >= 0 && st < V && stt >= 0 && stt < V && sp_i >= 0 && sp_i < V);

    /* spec_accept on a verify of [first, four drafts = each row's argmax]: everything accepted + bonus */
    int vt[5] = {first, 0, 0, 0, 0};
    for (int i = 1; i < 5; i++) {
        spec_verify(m, &kv, vt, i, 24, lg);
        vt[i] = argmax_row(lg + (size_t)(i - 1) * V, V);
    }
    rc = spec_verify(m, &kv, vt, 5, 24, lg);
    int acc[SPEC_MAX_DRAFT + 1];
    int na = spec_accept(NULL, lg, vt + 1, 4, V, 0.0f, acc);
    printf("verify rc=%d accepted=%d bonus_ok=%d\n", rc, na, na == 5 && acc[4] == argmax_row(lg + (size_t)3 * V, V));

    /* spec_decode_loop at temp 0: greedy, the n-gram drafter on the device loop, the same drafter host-driven
     * (history longer than the prefilled prompt), the self-speculative drafter; all print the same text */
    const int N = 24;
    printf("greedy=[");
    greedy_pieces(m, &kv, tok, first, 24, N);
    printf("]\n");
    SpeculativeState ss;
    spec_state_init(&ss);
    NGramDraft *ng = ngram_draft_init(prompt, 24, 3, 4);
    printf("ngram_device=[");
    fflush(stdout);
    spec_decode_loop(m, &kv, tok, &ss, ngram_draft_fn, ng, first, 24, N, 0.0f);
    printf("] iters=%lld\n", (long long)ss.total_iterations);
    ngram_draft_push(ng, first);  /* history now longer than the ring's prompt: the host-driven loop */
    spec_state_init(&ss);
    printf("ngram_host=[");
    fflush(stdout);
    spec_decode_loop(m, &kv, tok, &ss, ngram_draft_fn, ng, first, 24, N, 0.0f);
    printf("] iters=%lld\n", (long long)ss.total_iterations);
    ngram_draft_free(ng);
    SelfSpecDraft *sd = self_spec_draft_init(m, 1, 4, 512);
    spec_state_init(&ss);
    printf("self_host=[");
    fflush(stdout);
    spec_decode_loop(m, &kv, tok, &ss, self_spec_draft_fn, sd, first, 24, N, 0.0f);
    printf("] iters=%lld draft=%lld\n", (long long)ss.total_iterations, (long long)ss.total_draft);
    self_spec_draft_free(sd);

    metal_context_free(mc);
    kv_free(&kv);
    mistral_free(m);
    tokenizer_free(tok);
    gguf_close(g);
    free(lg); free(xs); free(ref); free(tmp); free(pr);
    return 0;
}
