/* Test program: the drop-in headers (include/compat) compile as C, link against libspecdec_b200.so and
 * run the reference-signature entry points.  Prints one line per check; exit code 0 = all ran.
 * Without a GPU it only checks that the calls fail cleanly. */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "compat/dequant.h"
#include "compat/metal_matvec.h"
#include "compat/speculative.h"

int main(int argc, char **argv) {
    (void)argv;
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
    if (argc > 1) {
        /* metal_matvec.h context on a model file given on the command line */
        FILE *f = fopen(argv[1], "rb");
        if (!f) return 2;
        fseek(f, 0, SEEK_END);
        long len = ftell(f);
        fseek(f, 0, SEEK_SET);
        void *buf = malloc(len);
        if (fread(buf, 1, len, f) != (size_t)len) return 2;
        fclose(f);
        sd_model_info in;
        sd_ctx *probe = NULL;
        if (sd_ctx_create(buf, len, NULL, &probe) != SD_OK) return 3;
        sd_ctx_info(probe, &in);
        sd_ctx_free(probe);
        MetalContext *mc = metal_context_init(buf, len, in.dim, in.n_kv_heads * in.head_dim, in.hidden_dim, in.vocab_size,
                                              in.n_heads, in.n_layers, 512);
        if (!mc) return 4;
        printf("batch5=%d batch9=%d batch17=%d\n", metal_alloc_batch_buffers(mc, 5, 0, 0, 0, 0, 512),
               metal_alloc_batch_buffers(mc, 9, 0, 0, 0, 0, 512), metal_alloc_batch_buffers(mc, 17, 0, 0, 0, 0, 512));
        int toks[5] = {5, 6, 7, 8, 9};
        float *lg = malloc(sizeof(float) * 5 * in.vocab_size);
        int rc = spec_verify(mc, NULL, toks, 5, 0, lg);
        spec_bind_context(mc);
        int draft[4], acc[5];
        for (int i = 0; i < 4; i++) {
            int best = 0;
            for (int v = 1; v < in.vocab_size; v++)
                if (lg[(size_t)i * in.vocab_size + v] > lg[(size_t)i * in.vocab_size + best]) best = v;
            draft[i] = best;
        }
        int na = spec_accept(NULL, lg, draft, 4, in.vocab_size, 0.0f, acc);
        printf("verify rc=%d accepted=%d\n", rc, na);
        metal_context_free(mc);
    }
    return 0;
}
