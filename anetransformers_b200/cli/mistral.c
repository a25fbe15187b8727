/*
 * mistral -- command-line driver with the reference's flags (mistral/mistral_infer.m:394-450) on the B200
 * engine.  Decode modes follow mistral_infer.m:
 *   default            greedy / sampled decode          (mistral_infer.m:690-716)
 *   --speculative      self-speculative decode          (mistral_infer.m:660-689)
 *   --speculative --metal | --draft ngram
 *                      n-gram (prompt-lookup) speculative decode (mistral_infer.m:638-659)
 * --prompt TEXT is tokenized with the model's vocabulary (sd_tokenizer_*, mistral/tokenizer.h semantics, BOS
 * first), after the instruct template "[INST] TEXT [/INST]" with --chat (mistral_infer.m:538-550).
 * Added flags: --prompt-ids (comma-separated token ids instead of text), --ignore-eos, --draft ngram|self,
 * --ngram-n, --seed, --device.  Generated tokens go to stdout as tokenizer_decode_token pieces
 * (mistral_infer.m:630, U+2581 shown as a space); stats to stderr in the reference's layout.
 */
#define _GNU_SOURCE
#include <getopt.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "specdec_b200.h"

static void usage(const char *argv0) {
    fprintf(stderr, "Usage: %s --model <gguf> (--prompt TEXT [--chat] | --prompt-ids 1,2,3) [--tokens N] [--temp T]\n",
            argv0);
    fprintf(stderr, "       [--top-p P] [--top-k K] [--rep-penalty R] [--rep-window W]\n");
    fprintf(stderr, "       [--context N] [--speculative] [--spec-k K] [--spec-layers N] [--metal]\n");
    fprintf(stderr, "       [--draft ngram|self] [--ngram-n N] [--ignore-eos] [--seed S] [--device D]\n");
    fprintf(stderr, "  --speculative    speculative decode (self-speculative; n-gram with --metal or --draft ngram)\n");
    fprintf(stderr, "  --spec-k K       drafts per iteration (default 4, max 15)\n");
    fprintf(stderr, "  --spec-layers N  self-speculative draft depth (default 8)\n");
}

/* A generated token as the reference prints it: the tokenizer's piece with U+2581 shown as a space. */
static void print_token(const sd_tokenizer *tok, int id) {
    const char *s = sd_tokenizer_piece(tok, id);
    for (const char *c = s; *c; c++) {
        if ((unsigned char)c[0] == 0xE2 && (unsigned char)c[1] == 0x96 && (unsigned char)c[2] == 0x81) {
            putchar(' ');
            c += 2;
        } else {
            putchar(*c);
        }
    }
    fflush(stdout);
}

int main(int argc, char **argv) {
    const char *model_path = NULL, *prompt_ids = NULL, *prompt_text = NULL, *draft = NULL;
    int max_tokens = 128, top_k = 40, rep_window = 64, context_len = 0, use_spec = 0, spec_k = 4, spec_layers = 8;
    int use_metal = 0, ngram_n = 3, ignore_eos = 0, device = 0, chat_mode = 0;
    float temperature = 0.7f, top_p = 0.9f, rep_penalty = 1.1f;
    unsigned long long seed = 0;
    static struct option opts[] = {
        {"model", required_argument, 0, 'm'},       {"prompt", required_argument, 0, 'p'},
        {"tokens", required_argument, 0, 'n'},      {"temp", required_argument, 0, 't'},
        {"top-p", required_argument, 0, 'P'},       {"top-k", required_argument, 0, 'K'},
        {"rep-penalty", required_argument, 0, 'r'}, {"rep-window", required_argument, 0, 'w'},
        {"chat", no_argument, 0, 'c'},              {"context", required_argument, 0, 'C'},
        {"speculative", no_argument, 0, 'S'},       {"spec-k", required_argument, 0, 'k'},
        {"spec-layers", required_argument, 0, 'L'}, {"metal", no_argument, 0, 'G'},
        {"ane", no_argument, 0, 'A'},               {"prompt-ids", required_argument, 0, 'I'},
        {"ignore-eos", no_argument, 0, 'E'},        {"draft", required_argument, 0, 'D'},
        {"ngram-n", required_argument, 0, 'N'},     {"seed", required_argument, 0, 's'},
        {"device", required_argument, 0, 'd'},      {0, 0, 0, 0}};
    int o;
    while ((o = getopt_long(argc, argv, "m:p:n:t:P:K:r:w:cC:Sk:L:GAI:ED:N:s:d:", opts, NULL)) != -1) {
        switch (o) {
            case 'm': model_path = optarg; break;
            case 'p': prompt_text = optarg; break;
            case 'n': max_tokens = atoi(optarg); break;
            case 't': temperature = (float)atof(optarg); break;
            case 'P': top_p = (float)atof(optarg); break;
            case 'K': top_k = atoi(optarg); break;
            case 'r': rep_penalty = (float)atof(optarg); break;
            case 'w': rep_window = atoi(optarg); break;
            case 'c': chat_mode = 1; break;
            case 'C': context_len = atoi(optarg); break;
            case 'S': use_spec = 1; break;
            case 'k': spec_k = atoi(optarg); break;
            case 'L': spec_layers = atoi(optarg); break;
            case 'G': use_metal = 1; break;
            case 'A': break;
            case 'I': prompt_ids = optarg; break;
            case 'E': ignore_eos = 1; break;
            case 'D': draft = optarg; use_spec = 1; break;
            case 'N': ngram_n = atoi(optarg); break;
            case 's': seed = strtoull(optarg, NULL, 10); break;
            case 'd': device = atoi(optarg); break;
            default: usage(argv[0]); return 1;
        }
    }
    if (!model_path) {
        usage(argv[0]);
        return 1;
    }
    if (!prompt_ids && !prompt_text) {
        usage(argv[0]);
        return 1;
    }
    int fd = open(model_path, O_RDONLY);
    if (fd < 0) {
        perror("open");
        return 1;
    }
    struct stat st;
    fstat(fd, &st);
    void *base = mmap(NULL, st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (base == MAP_FAILED) {
        perror("mmap");
        return 1;
    }
    sd_tokenizer *tok = NULL;
    if (sd_tokenizer_create(base, st.st_size, &tok) != SD_OK) {
        fprintf(stderr, "Failed to init tokenizer: %s\n", sd_last_error());
        return 1;
    }
    int vocab_n = 0;
    sd_tokenizer_info(tok, &vocab_n, NULL, NULL);
    fprintf(stderr, "Tokenizer: %d tokens\n", vocab_n);
    int cap = 16, n_prompt = 0;
    int32_t *prompt = NULL;
    if (prompt_ids) {
        prompt = (int32_t *)malloc(sizeof(int32_t) * cap);
        for (const char *c = prompt_ids; *c;) {
            char *end;
            long v = strtol(c, &end, 10);
            if (end == c) break;
            if (n_prompt == cap) prompt = (int32_t *)realloc(prompt, sizeof(int32_t) * (cap *= 2));
            prompt[n_prompt++] = (int32_t)v;
            c = *end == ',' ? end + 1 : end;
        }
    } else {
        char *chat = chat_mode ? sd_tokenizer_apply_chat(prompt_text) : NULL;
        const char *text = chat ? chat : prompt_text;
        cap = 3 * (int)strlen(text) + 8;  /* a character can fall back to 3 byte tokens */
        prompt = (int32_t *)malloc(sizeof(int32_t) * cap);
        n_prompt = sd_tokenizer_encode(tok, text, prompt, cap, 1);
        sd_free(chat);
    }
    fprintf(stderr, "Prompt: %d tokens\n", n_prompt);
    if (n_prompt <= 0) {
        fprintf(stderr, "Empty prompt after tokenization\n");
        return 1;
    }
    sd_ctx_opts co;
    sd_ctx_opts_default(&co);
    co.device = device;
    co.max_seq = context_len > 0 ? context_len : 65536;
    if (co.max_seq > 131072) co.max_seq = 131072;
    sd_ctx *ctx = NULL;
    fprintf(stderr, "Loading model: %s\n", model_path);
    if (sd_ctx_create(base, st.st_size, &co, &ctx) != SD_OK) {
        fprintf(stderr, "Failed to load model: %s\n", sd_last_error());
        return 1;
    }
    munmap(base, st.st_size);
    sd_model_info in;
    sd_ctx_info(ctx, &in);
    fprintf(stderr, "dim=%d hidden=%d layers=%d heads=%d kv_heads=%d vocab=%d context=%d (B200, W4A8)\n", in.dim,
            in.hidden_dim, in.n_layers, in.n_heads, in.n_kv_heads, in.vocab_size, in.max_seq);
    sd_gen_params p;
    sd_gen_params_default(&p);
    p.max_tokens = max_tokens;
    p.temp = temperature;
    p.top_p = top_p;
    p.top_k = top_k;
    p.rep_penalty = rep_penalty;
    p.rep_window = rep_window;
    p.ignore_eos = ignore_eos;
    p.spec_k = spec_k;
    p.ngram_n = ngram_n;
    p.draft_layers = spec_layers;
    p.seed = seed;
    p.mode = SD_GEN_GREEDY;
    if (use_spec) p.mode = (use_metal || (draft && strcmp(draft, "ngram") == 0)) ? SD_GEN_NGRAM : SD_GEN_SELF_SPEC;
    int out_cap = max_tokens + 32;
    int32_t *out = (int32_t *)malloc(sizeof(int32_t) * out_cap);
    sd_gen_stats gs;
    int n = sd_generate(ctx, &p, prompt, n_prompt, out, out_cap, &gs);
    if (n < 0) {
        fprintf(stderr, "generation failed: %s\n", sd_last_error());
        sd_ctx_free(ctx);
        return 1;
    }
    for (int i = 0; i < n; i++) print_token(tok, out[i]);
    printf("\n");
    fprintf(stderr, "\n--- Stats ---\n");
    fprintf(stderr, "Prompt tokens:    %d\n", n_prompt);
    fprintf(stderr, "Generated tokens: %d\n", n);
    fprintf(stderr, "Prefill:          %.1f ms (%.2f tok/s)\n", gs.ms_prefill, n_prompt / (gs.ms_prefill / 1000.0));
    if (n > 1 && gs.ms_decode > 0)
        fprintf(stderr, "Decode:           %.1f ms (%.2f tok/s)\n", gs.ms_decode, (n - 1) / (gs.ms_decode / 1000.0));
    if (p.mode != SD_GEN_GREEDY && gs.total_iterations > 0) {
        fprintf(stderr, "Draft iterations: %lld\n", (long long)gs.total_iterations);
        fprintf(stderr, "Acceptance rate:  %.1f%%\n",
                gs.total_draft > 0 ? 100.0 * (gs.total_accepted - gs.total_iterations) / gs.total_draft : 0.0);
    }
    sd_ctx_free(ctx);
    sd_tokenizer_free(tok);
    free(out);
    free(prompt);
    return 0;
}
