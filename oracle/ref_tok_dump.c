/*
 * ref_tok_dump.c -- TEST INFRASTRUCTURE.  Links the reference's own tokenizer (mistral/tokenizer.h with its
 * GGUF parser mistral/gguf_loader.h, included from the reference tree at build time, never copied) and runs
 * it on a model file: every stdin line is a hex-encoded UTF-8 text; the output line is
 *   <ids of tokenizer_encode(text, add_bos=1)> | <hex of tokenizer_decode(ids)>
 * (ids space-separated).  tests/golden/make_tokenizer_golden.py turns this into the committed fixture that
 * pins the library's tokenizer.
 */
#include <stdio.h>
#include "tokenizer.h"

static int hexval(int c) { return c <= '9' ? c - '0' : (c | 32) - 'a' + 10; }

int main(int argc, char **argv) {
    if (argc < 2) { fprintf(stderr, "usage: %s model.gguf < hex-lines\n", argv[0]); return 2; }
    GGUFFile *f = gguf_open(argv[1]);
    if (!f) return 1;
    Tokenizer *t = tokenizer_init(f);
    static char line[1 << 16], text[1 << 15];
    static int ids[1 << 16];
    while (fgets(line, sizeof line, stdin)) {
        size_t n = strcspn(line, "\r\n");
        size_t m = 0;
        for (size_t i = 0; i + 1 < n + 1 && i + 1 < sizeof line && m + 1 < sizeof text; i += 2) {
            if (i + 1 >= n) break;
            text[m++] = (char)(hexval(line[i]) * 16 + hexval(line[i + 1]));
        }
        text[m] = '\0';
        int k = tokenizer_encode(t, text, ids, (int)(sizeof ids / sizeof ids[0]), 1);
        for (int i = 0; i < k; i++) printf(i ? " %d" : "%d", ids[i]);
        char *d = tokenizer_decode(t, ids, k);
        printf(" |");
        for (const unsigned char *p = (const unsigned char *)d; *p; p++) printf("%02x", *p);
        printf("\n");
        free(d);
    }
    tokenizer_free(t);
    gguf_close(f);
    return 0;
}
