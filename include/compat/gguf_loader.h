/*
 * compat/gguf_loader.h -- drop-in for the reference's mistral/gguf_loader.h entry points that the decode path
 * uses, backed by libspecdec_b200.so.
 *
 *   MistralConfig, GGUFFile     mistral/gguf_loader.h:51-84   (same field names; tensors are not listed: the
 *                                                               engine reads them from the image itself)
 *   gguf_open                   mistral/gguf_loader.h:151-313 -> mmap (MAP_PRIVATE, as :159) + sd_gguf_describe
 *                                                               + the vocabulary through sd_tokenizer_*
 *   gguf_close                  mistral/gguf_loader.h:376-390
 */
#ifndef SPECDEC_COMPAT_GGUF_LOADER_H
#define SPECDEC_COMPAT_GGUF_LOADER_H
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include "../specdec_b200.h"

typedef struct {
    int dim;
    int hidden_dim;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int vocab_size;
    int max_seq_len;
    float rope_theta;
    float rms_eps;
    int sliding_window;
} MistralConfig;

typedef struct {
    int fd;
    void *mmap_base;
    size_t mmap_len;
    uint8_t *data_start;   /* the tensor data section */
    uint32_t version;
    uint32_t n_tensors;
    MistralConfig cfg;
    int vocab_size;
    char **vocab_tokens;   /* [vocab_size] owned copies */
    float *vocab_scores;   /* [vocab_size] */
    int *vocab_types;      /* [vocab_size] */
    int bos_id, eos_id, unk_id;
} GGUFFile;

static inline void gguf_close(GGUFFile *f) {
    if (!f) return;
    if (f->vocab_tokens)
        for (int i = 0; i < f->vocab_size; i++) free(f->vocab_tokens[i]);
    free(f->vocab_tokens);
    free(f->vocab_scores);
    free(f->vocab_types);
    if (f->mmap_base && f->mmap_base != MAP_FAILED) munmap(f->mmap_base, f->mmap_len);
    if (f->fd >= 0) close(f->fd);
    free(f);
}

static inline GGUFFile *gguf_open(const char *path) {
    GGUFFile *f = (GGUFFile *)calloc(1, sizeof(GGUFFile));
    if (!f) return NULL;
    f->fd = open(path, O_RDONLY);
    if (f->fd < 0) {
        fprintf(stderr, "gguf_open: cannot open %s\n", path);
        free(f);
        return NULL;
    }
    struct stat st;
    if (fstat(f->fd, &st) != 0) {
        gguf_close(f);
        return NULL;
    }
    f->mmap_len = (size_t)st.st_size;
    f->mmap_base = mmap(NULL, f->mmap_len, PROT_READ, MAP_PRIVATE, f->fd, 0);
    if (f->mmap_base == MAP_FAILED) {
        f->mmap_base = NULL;
        gguf_close(f);
        return NULL;
    }
    sd_gguf_desc d;
    if (sd_gguf_describe(f->mmap_base, f->mmap_len, &d) != SD_OK) {
        fprintf(stderr, "gguf_open: %s\n", sd_last_error());
        gguf_close(f);
        return NULL;
    }
    f->version = d.version;
    f->n_tensors = d.n_tensors;
    f->data_start = (uint8_t *)f->mmap_base + d.data_offset;
    f->cfg.dim = d.dim;
    f->cfg.hidden_dim = d.hidden_dim;
    f->cfg.n_layers = d.n_layers;
    f->cfg.n_heads = d.n_heads;
    f->cfg.n_kv_heads = d.n_kv_heads;
    f->cfg.head_dim = d.head_dim;
    f->cfg.vocab_size = d.vocab_size;
    f->cfg.max_seq_len = d.context_length;
    f->cfg.rope_theta = d.rope_theta;
    f->cfg.rms_eps = d.rms_eps;
    f->cfg.sliding_window = 0;
    f->bos_id = d.bos_id;
    f->eos_id = d.eos_id;
    f->unk_id = 0;
    sd_tokenizer *t = NULL;
    if (sd_tokenizer_create(f->mmap_base, f->mmap_len, &t) == SD_OK) {
        sd_tokenizer_info(t, &f->vocab_size, NULL, NULL);
        f->vocab_tokens = (char **)calloc((size_t)f->vocab_size, sizeof(char *));
        f->vocab_scores = (float *)calloc((size_t)f->vocab_size, sizeof(float));
        f->vocab_types = (int *)calloc((size_t)f->vocab_size, sizeof(int));
        for (int i = 0; i < f->vocab_size; i++) {
            const char *p = "";
            sd_tokenizer_entry(t, i, &p, &f->vocab_scores[i], &f->vocab_types[i]);
            f->vocab_tokens[i] = strdup(p);
        }
        sd_tokenizer_free(t);
    }
    return f;
}

#endif
