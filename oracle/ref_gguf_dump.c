/*
 * ref_gguf_dump.c -- TEST INFRASTRUCTURE.  Links the reference's own GGUF v3
 * parser (mistral/gguf_loader.h, included from the reference tree at build
 * time, never copied) and prints what it extracts from a file as JSON:
 * MistralConfig (gguf_loader.h:51-63, filled at :195-259), bos/eos ids, vocab
 * size, and the tensor table (name, type, dims, data offset relative to the
 * 32-byte aligned data section, :262-281).  tests/test_gguf.py compares this
 * with the synthetic-model writer and the product's own loader.
 */
#include <stdio.h>
#include "gguf_loader.h"

int main(int argc, char **argv) {
    if (argc < 2) { fprintf(stderr, "usage: %s model.gguf\n", argv[0]); return 2; }
    GGUFFile *f = gguf_open(argv[1]);
    if (!f) return 1;
    MistralConfig *c = &f->cfg;
    printf("{\"version\": %u, \"dim\": %d, \"hidden_dim\": %d, \"n_layers\": %d, "
           "\"n_heads\": %d, \"n_kv_heads\": %d, \"head_dim\": %d, \"vocab_size\": %d, "
           "\"max_seq_len\": %d, \"rope_theta\": %.9g, \"rms_eps\": %.9g, "
           "\"sliding_window\": %d, \"bos_id\": %d, \"eos_id\": %d, \"unk_id\": %d, "
           "\"data_start\": %zu, \"tensors\": [",
           f->version, c->dim, c->hidden_dim, c->n_layers, c->n_heads, c->n_kv_heads,
           c->head_dim, c->vocab_size, c->max_seq_len, c->rope_theta, c->rms_eps,
           c->sliding_window, f->bos_id, f->eos_id, f->unk_id,
           (size_t)(f->data_start - (uint8_t *)f->mmap_base));
    for (uint32_t i = 0; i < f->n_tensors; i++) {
        GGUFTensor *t = &f->tensors[i];
        printf("%s{\"name\": \"%s\", \"type\": %u, \"ne\": [%llu, %llu], \"offset\": %llu, \"bytes\": %zu}",
               i ? ", " : "", t->name, t->type, (unsigned long long)t->ne[0],
               (unsigned long long)t->ne[1], (unsigned long long)t->offset, gguf_tensor_bytes(t));
    }
    printf("], \"token0\": \"%s\", \"token_last\": \"%s\"}\n",
           f->vocab_size > 0 ? f->vocab_tokens[0] : "",
           f->vocab_size > 0 ? f->vocab_tokens[f->vocab_size - 1] : "");
    gguf_close(f);
    return 0;
}
