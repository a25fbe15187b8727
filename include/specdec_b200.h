/*
 * specdec_b200.h -- C ABI of libspecdec_b200.so, the B200 (sm_100a) implementation of the
 * speculative-decode hot path of m0at/ANEtransformers (Mistral-architecture Q4_0 models).
 *
 * Plain C: opaque handles, plain pointers and sizes, int status codes.  No CUDA, torch or C++
 * types appear in any signature (a CUDA stream is passed as void*; NULL = the legacy default
 * stream).  "_dev" entry points take device pointers and are stream-ordered; the others take host
 * pointers and return when their results are in host memory.
 *
 * Each declaration names the reference interface it replaces (path:line in the reference repo).
 * The reference has no ABI of its own -- every hot-path symbol is a `static` function in a header
 * compiled as one translation unit (mistral/Makefile:11-14) -- so the drop-in for those headers is
 * include/compat/{dequant.h,speculative.h,metal_matvec.h}, whose inline bodies call the functions
 * below.
 */
#ifndef SPECDEC_B200_H
#define SPECDEC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SD_ABI_VERSION 1
/* Most tokens one verify forward carries (current token + up to 15 drafts). */
#define SD_MAX_VERIFY 16

#if defined(__GNUC__)
#define SD_API __attribute__((visibility("default")))
#else
#define SD_API
#endif

/* Status codes.  The reference reports failure as NULL / -1 plus a stderr line
 * (e.g. metal_alloc_batch_buffers, mistral/metal_matvec.h:253-293); this ABI keeps 0 = success and
 * negative = failure, with a message from sd_last_error(). */
enum {
    SD_OK = 0,
    SD_ERR_INVALID = -1,      /* bad argument / unsupported shape */
    SD_ERR_OOM = -2,          /* device or host allocation failed */
    SD_ERR_CUDA = -3,         /* CUDA runtime error */
    SD_ERR_TIMEOUT = -4,      /* a bounded device wait ran out (device error word set) */
    SD_ERR_FORMAT = -5,       /* malformed GGUF / unsupported tensor type */
    SD_ERR_UNSUPPORTED = -6,  /* feature not available in this build or configuration */
    SD_ERR_NO_DEVICE = -7     /* no CUDA device */
};

/* Last error message of the calling thread ("" if none). */
SD_API const char *sd_last_error(void);
SD_API int sd_abi_version(void);
/* Number of visible CUDA devices (0 without a GPU; never fails). */
SD_API int sd_device_count(void);

/* Reference block layouts: mistral/dequant.h:17-21 (18-byte Q4_0, fp16 scale bits) and
 * mistral/dequant.h:537-541 (36-byte Q8_0 with an fp32 scale). */
typedef struct { uint16_t d; uint8_t qs[16]; } sd_block_q4_0;
typedef struct { float d; int8_t qs[32]; } sd_block_q8_0;

/* ======================================================================================
 * Single-op layer: Q8_0 quantizer and W4A8 matvec
 * ====================================================================================== */

/* Device-resident Q4_0 matrix, repacked from the reference's AoS blocks into the 16-row tile
 * layout the matvec streams.  rows % 16 == 0 is not required (padded); cols % 1024 == 0. */
typedef struct sd_qmat sd_qmat;

/* q4_0_host: [rows][cols/32] sd_block_q4_0 in host memory (e.g. an mmap'd GGUF tensor). */
SD_API int sd_qmat_create(const void *q4_0_host, int rows, int cols, int device, sd_qmat **out);
SD_API void sd_qmat_free(sd_qmat *m);
SD_API int sd_qmat_shape(const sd_qmat *m, int *rows, int *cols, size_t *device_bytes);

/* Q8_0 activations for S rows of n values in device memory, as three planes:
 *   qs [S][n] int8 codes, d [S][n/32] fp32 scales, sum [S][n/32] int32 (sum of the 32 codes). */
typedef struct { int8_t *qs; float *d; int32_t *sum; } sd_q8_dev;

/* Replaces quantize_f32_to_q8_0 (mistral/dequant.h:545-599) for S rows; bit-exact codes and scales.
 * x: device [S][n] fp32, n % 32 == 0. */
SD_API int sd_quantize_q8_0_dev(const float *x, sd_q8_dev out, int S, int n, void *stream);
/* Planes <-> reference AoS blocks (device buffers of S*n/32 sd_block_q8_0). */
SD_API int sd_q8_to_blocks_dev(sd_q8_dev in, sd_block_q8_0 *out, int S, int n, void *stream);
SD_API int sd_blocks_to_q8_dev(const sd_block_q8_0 *in, sd_q8_dev out, int S, int n, void *stream);

/* Replaces q4_0_q8_0_matvec_sdot_parallel (mistral/dequant.h:1022-1137) for S <= 8 activation
 * rows sharing one weight read (the S=K+1 verify shape of mistral/mistral_infer.m:134-164).
 * y: device [S][rows] fp32. */
SD_API int sd_matvec_q4_0_q8_0_dev(const sd_qmat *W, sd_q8_dev x, float *y, int S, void *stream);

/* Exact int32 block dot products of activation row 0: isum[r][b] = sum_j (q_j - 8) * x8_j, the
 * per-block SDOT result of mistral/dequant.h:1078-1083.  isum: device [rows][cols/32]. */
SD_API int sd_block_sums_dev(const sd_qmat *W, sd_q8_dev x, int32_t *isum, void *stream);

/* sd_matvec_q4_0_q8_0_dev for callers that cannot have device memory allocated on their behalf:
 * a process that gives all free HBM to its own pool at start-up, or a latency loop that cannot take
 * the device-wide synchronisation of a cudaFree.  It has no counterpart in the reference.
 * Where the matvec splits K (long rows at larger S), the partial outputs go to a fixed array of
 * SD_NOALLOC_SCRATCH_BYTES that the library keeps on every GPU that loads it, until exit; a shape
 * whose partials do not fit is rejected with SD_ERR_INVALID.  The first call on a device looks up
 * that array's address (and may load the library's device code): make it before any stream capture.
 * All calls on one device share the array, so calls that overlap on the GPU (different streams, or
 * different threads) race and give wrong results; serialise them.  Results equal those of
 * sd_matvec_q4_0_q8_0_dev bit for bit.  Both entry points must be called with W's device current
 * (SD_ERR_INVALID otherwise).  A bounded device wait that runs out records its code in the device's error
 * word (a file-scope device variable, no allocation), which sd_device_error reads. */
#define SD_NOALLOC_SCRATCH_BYTES (1u << 20)
SD_API int sd_matvec_q4_0_q8_0_noalloc_dev(const sd_qmat *W, sd_q8_dev x, float *y, int S, void *stream);

/* Read and clear the error word of `device` that the single-op device entry points above (matvec, block
 * sums, no-alloc matvec) share: 0 if no bounded device wait ran out since the last read, else the positive
 * device error code; negative on a CUDA failure.  Synchronises the device.  No reference counterpart (the
 * reference's CPU calls cannot time out). */
SD_API int sd_device_error(int device);

/* Host-pointer drop-ins with the reference signatures (mistral/dequant.h:545 and :1022).  They run
 * on the current device; the matvec uploads and repacks W on first use and caches it keyed by the
 * host address and shape (weights are immutable mmap'd tensors in the reference).  Errors are
 * reported on stderr and through sd_last_error(); y is left unchanged on failure. */
SD_API void sd_host_quantize_f32_to_q8_0(const float *x, sd_block_q8_0 *out, int n);
SD_API void sd_host_q4_0_q8_0_matvec(const void *W, const sd_block_q8_0 *x, float *y, int out_dim, int in_dim);
/* Replaces the reference's fp32 matvec of K-quant matrices (q4_matvec for Q6_K / Q4_K,
 * mistral/mistral_model.h:211-242: q6_K_matvec_f32_neon, mistral/dequant.h:349-520; Q4_K: the fp16 dequant of
 * dequant_q4_K_block_neon, :63-113, then an fp32 sgemv): y = W x for W [out_dim][in_dim/256] GGUF super-blocks
 * of `type` (14 = Q6_K, 12 = Q4_K) and fp32 x, in_dim % 256 == 0.  Runs on the current device; W is uploaded
 * once per (address, type, shape) and cached as above. */
SD_API void sd_host_kq_matvec(int type, const void *W, const float *x, float *y, int out_dim, int in_dim);
/* Drop the host-drop-in weight cache (frees its device copies). */
SD_API void sd_host_cache_clear(void);

/* ======================================================================================
 * Model context: weights in HBM, fp16 KV ring, verify / decode forward, generation loops
 * ====================================================================================== */

typedef struct sd_ctx sd_ctx;

typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab_size;
    int max_seq;          /* KV ring slots (--context, mistral/mistral_infer.m:518-523) */
    float rope_theta, rms_eps;
    int bos_id, eos_id;
    int tp_rank, tp_size;
    size_t weight_bytes;  /* device bytes of repacked weights held by this rank */
    size_t kv_bytes;      /* device bytes of this rank's KV ring */
    int forward_kernel;   /* 1 if forwards run as one persistent kernel, 0 if one kernel per op */
} sd_model_info;

typedef struct {
    int device;           /* CUDA device ordinal */
    int max_seq;          /* 0 = 65536, capped at 131072 (mistral/mistral_infer.m:518-523) */
    int max_batch;        /* tokens per forward, 1..8 (0 = 8) */
    int tp_rank, tp_size; /* tensor parallelism (tp_size 1 = single GPU) */
    void *nccl_comm;      /* ncclComm_t for tp_size > 1, created by the caller */
    int use_graphs;       /* capture per-S forwards in CUDA graphs (default 1) */
    int use_pdl;          /* programmatic dependent launch between kernels (default 1) */
    int forward_kernel;   /* 1 = each forward is one persistent kernel (default; tensor-parallel contexts
                             once their peers are connected), 0 = one kernel per op; both give
                             bit-identical logits */
    int prefill_gemm;     /* 1 (default): sd_prefill / sd_generate run prompts of at least 256 tokens through the
                             batched engine's tensor-core GEMMs (64 slices of 8 tokens per forward, all writing this
                             context's K/V ring) instead of 8-token matvec forwards; single-GPU contexts with a
                             Q4_0 embedding and LM head.  Logits agree with the matvec path within the batched
                             path's tolerance (its attention uses single fp16 Q and P).  0 = always matvecs. */
} sd_ctx_opts;

SD_API void sd_ctx_opts_default(sd_ctx_opts *o);

/* Tensor parallelism within one node (one process per GPU): Wq/Wk/Wv/W1/W3 split by output rows,
 * Wo/W2 by input columns, and a sum all-reduce of the S x dim partial outputs after o-proj and
 * down-proj.  The reference runs on one device and has no counterpart; these only create the NCCL
 * communicator that sd_ctx_opts.nccl_comm takes.  NCCL (libnccl.so.2) is loaded at run time.
 * One rank calls sd_nccl_unique_id and sends the SD_NCCL_ID_BYTES bytes to the others; every rank then
 * calls sd_nccl_comm_create with its rank and device. */
#define SD_NCCL_ID_BYTES 128
SD_API int sd_nccl_unique_id(void *id_out);
SD_API int sd_nccl_comm_create(const void *id, int nranks, int rank, int device, void **comm_out);
SD_API void sd_nccl_comm_destroy(void *comm);
/* The same reduction without NCCL: each rank's o-proj / down-proj partial outputs stay in its own HBM
 * and the following RMSNorm kernel of every rank reads all ranks' partials over NVLink (peer memory,
 * CUDA IPC), adding them in rank order, after a flag handshake with bounded waits.  Every rank exports
 * its SD_TP_HANDLE_BYTES handle, the handles are exchanged by the caller, and every rank connects
 * with all of them in rank order; from then on no NCCL call is made.  No reference counterpart. */
#define SD_TP_HANDLE_BYTES 64
SD_API int sd_ctx_tp_handle(sd_ctx *ctx, void *handle_out);
SD_API int sd_ctx_tp_connect(sd_ctx *ctx, const void *handles, int n_ranks);

/* What mistral/gguf_loader.h's gguf_open (:151-313) extracts from a GGUF v3 image: version, tensor count, the
 * model configuration (MistralConfig, :51-63, read at :195-259), BOS / EOS ids and the offset of the 32-byte
 * aligned tensor data section (:280-281). */
typedef struct {
    uint32_t version, n_tensors;
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab_size, context_length;
    float rope_theta, rms_eps;
    int bos_id, eos_id;
    size_t data_offset;
} sd_gguf_desc;
SD_API int sd_gguf_describe(const void *gguf_base, size_t gguf_len, sd_gguf_desc *out);

/* Replaces metal_context_init (mistral/metal_matvec.h:134-225) + mistral_load
 * (mistral/mistral_model.h:262-357): parses the GGUF v3 image at gguf_base (the mmap'd file, as
 * metal_context_init receives it), uploads every tensor and repacks the Q4_0 matrices in HBM,
 * computes the RoPE inverse frequencies (mistral/mistral_model.h:69-74) and allocates the fp16 KV
 * ring [n_layers][max_seq][kv_dim] (mistral/kv_cache.h:22-35) and per-forward buffers
 * (metal_alloc_batch_buffers, mistral/metal_matvec.h:253-293). */
SD_API int sd_ctx_create(const void *gguf_base, size_t gguf_len, const sd_ctx_opts *opts, sd_ctx **out);
SD_API int sd_ctx_create_file(const char *gguf_path, const sd_ctx_opts *opts, sd_ctx **out);
/* Replaces metal_context_free (mistral/metal_matvec.h:540-565). */
SD_API void sd_ctx_free(sd_ctx *ctx);
SD_API int sd_ctx_info(const sd_ctx *ctx, sd_model_info *out);
/* Read and clear the context's device error word (non-zero after a bounded wait ran out). */
SD_API int sd_ctx_device_error(sd_ctx *ctx);
/* Stream the context launches on (cudaStream_t as void*). */
SD_API void *sd_ctx_stream(sd_ctx *ctx);

/* Forward S tokens at positions pos..pos+S-1 through all layers (writing their K/V into the ring)
 * and the LM head.  Replaces metal_forward (S=1, mistral/mistral_infer.m:31-92),
 * metal_forward_batch (S=K+1, :103-179) with the CPU logits of metal_spec_verify (:224-248), and
 * spec_verify (mistral/speculative.h:81-105).  logits: host [S][vocab] or NULL; argmax: host [S]
 * (first index on ties, mistral/mistral_model.h:1136-1143) or NULL.  S <= SD_MAX_VERIFY; a batch wider
 * than max_batch runs as consecutive forwards, with logits identical to one wide forward. */
SD_API int sd_forward(sd_ctx *ctx, const int32_t *tokens, int S, int pos, float *logits, int32_t *argmax);
/* Same with device buffers, stream-ordered, no host synchronisation. */
SD_API int sd_forward_dev(sd_ctx *ctx, const int32_t *tokens_dev, int S, int pos, float *logits_dev,
                   int32_t *argmax_dev, void *stream);
/* Prefill n prompt tokens at positions start_pos.. in chunks of max_batch (fills the KV ring). */
SD_API int sd_prefill(sd_ctx *ctx, const int32_t *tokens, int n, int start_pos);
/* First n_layers layers only (self-speculative drafter depth); same contract as sd_forward. */
SD_API int sd_forward_layers(sd_ctx *ctx, int n_layers, const int32_t *tokens, int S, int pos, float *logits,
                      int32_t *argmax);
/* Single-op model layer for whole-model parity and host-driven loops (single-GPU contexts; the kernel-per-op
 * path, not graph-captured).  Host pointers; each returns when its result is in host memory.
 *   sd_embed_token   replaces embed_token (mistral/mistral_model.h:125-157): out [dim] = row `token` of the
 *                    Q4_0 embedding, dequantised.
 *   sd_layer_decode  replaces mistral_layer_decode_parallel (mistral/mistral_model.h:818-899): x [dim] in/out
 *                    through layer `layer` at position pos, writing that layer's K/V into the ring slot
 *                    pos % max_seq (attention covers positions max(0, pos+1-max_seq) .. pos).
 *   sd_logits        replaces mistral_logits (mistral/mistral_model.h:1110-1122): final RMSNorm, Q8_0 and the
 *                    Q4_0 LM head of S <= max_batch hidden states x [S][dim] -> logits [S][vocab]. */
SD_API int sd_embed_token(sd_ctx *ctx, int token, float *out);
SD_API int sd_layer_decode(sd_ctx *ctx, float *x, int layer, int pos);
SD_API int sd_logits(sd_ctx *ctx, const float *x, int S, float *logits);

/* Copy n ring slots [pos0, pos0+n) of one layer's K and V (fp16 bits) to host buffers
 * [n][kv_dim_local].  The ring itself lives in HBM (mistral/kv_cache.h layout). */
SD_API int sd_kv_read(sd_ctx *ctx, int layer, int pos0, int n, uint16_t *k, uint16_t *v);

/* ======================================================================================
 * Speculative primitives on the device
 * ====================================================================================== */

/* Replaces ngram_draft_fn (mistral/speculative.h:425-464): earliest exact match of
 * history[hlen-n+1..hlen-1] ++ [current] among history[i..i+n-1], i in [0, hlen-n-1]; drafts
 * history[match+n ..] up to max_draft.  Runs as a device scan.  Returns the draft count (>= 0) or
 * a negative status; *match_pos gets the match start + n (or -1). */
SD_API int sd_ngram_draft(const int32_t *history, int hlen, int ngram_n, int max_draft, int current,
                   int32_t *draft_out, int *match_pos);

/* Replaces spec_accept (mistral/speculative.h:121-198) on the device.  logits: host
 * [n_draft+1][vocab] (row n_draft is the bonus row the callers use, speculative.h:312-317).
 * temp <= 0: greedy; else the Leviathan et al. rule with the seeded Philox stream (seed, *counter),
 * advanced in *counter.  bonus_mode: 0 = argmax bonus at temp 0 (fixed), 1 = the reference's
 * uniform draw.  accepted: host [n_draft+1].  Returns n_accepted in [1, n_draft+1] or < 0. */
SD_API int sd_spec_accept(sd_ctx *ctx, const float *draft_probs, const float *logits, const int32_t *draft,
                   int n_draft, float temp, int bonus_mode, uint64_t seed, uint64_t *counter,
                   int32_t *accepted);

/* Replaces sample_token (mistral/mistral_model.h:1145-1240) on the device of ctx: repetition penalty over
 * prev_tokens[0..n_prev) (applied to logits in place, as the reference does), then at temp <= 0 the argmax
 * (first index on ties), else top-k (top_k <= 64; 0 = 40), tempered softmax, top-p cut and renormalisation,
 * and a linear-CDF draw of one uniform from the Philox stream (seed, *counter) (arc4random in the reference),
 * advancing *counter.  logits: host [n], n <= vocab; n_prev <= 4096.  Returns the token or < 0. */
SD_API int sd_sample_token(sd_ctx *ctx, float *logits, int n, float temp, int top_k, float top_p, float rep_penalty,
                           const int32_t *prev_tokens, int n_prev, uint64_t seed, uint64_t *counter);
/* Replace spec_softmax (mistral/speculative.h:37-57: probs = softmax((logits - max) / temp), host arrays [n])
 * and spec_sample_probs (mistral/speculative.h:60-68: first i with r < cumsum(probs[0..i]), n-1 if none, r one
 * uniform of the Philox stream (seed, *counter), advanced by one).  n <= vocab.  sd_spec_sample_probs returns the
 * index or < 0. */
SD_API int sd_spec_softmax(sd_ctx *ctx, const float *logits, float *probs, int n, float temp);
SD_API int sd_spec_sample_probs(sd_ctx *ctx, const float *probs, int n, uint64_t seed, uint64_t *counter);

/* ======================================================================================
 * Generation loops (mistral/mistral_infer.m:579-716, speculative.h:217-379)
 * ====================================================================================== */
enum { SD_GEN_GREEDY = 0, SD_GEN_NGRAM = 1, SD_GEN_SELF_SPEC = 2 };
enum { SD_BONUS_ARGMAX = 0, SD_BONUS_REFERENCE = 1 };

typedef struct {
    int mode;                 /* SD_GEN_* */
    int max_tokens;           /* --tokens */
    float temp, top_p;        /* --temp, --top-p */
    int top_k;                /* --top-k */
    float rep_penalty;        /* --rep-penalty */
    int rep_window;           /* --rep-window */
    int ignore_eos;
    int spec_k;               /* drafts per iteration, <= SD_MAX_VERIFY - 1 */
    int ngram_n;              /* n-gram order */
    int draft_layers;         /* self-speculative drafter depth */
    int history_has_current;  /* 1 = reference n-gram wiring (history ends with the current token) */
    int bonus_mode;           /* SD_BONUS_* */
    uint64_t seed;            /* Philox seed replacing arc4random */
    int reuse_draft_kv;       /* sd_decode, self-speculative: the drafter's K/V of history[0 .. n_hist-2] is already
                                 in place (an earlier sd_decode of the same history), skip its prefill */
} sd_gen_params;

typedef struct {
    int n_generated;
    int64_t total_draft, total_accepted, total_iterations;
    double ms_prefill, ms_decode;
} sd_gen_stats;

SD_API void sd_gen_params_default(sd_gen_params *p);

/* Prefill the prompt, sample the first token, then decode.  out_tokens receives the generated
 * tokens (first token included); returns their count (<= out_cap) or a negative status. */
SD_API int sd_generate(sd_ctx *ctx, const sd_gen_params *p, const int32_t *prompt, int n_prompt,
                int32_t *out_tokens, int out_cap, sd_gen_stats *stats);

/* Decode only (the prompt already prefilled into positions [0, n_prompt)): starts from
 * first_token at position n_prompt with the drafter history = history[0..n_hist). */
SD_API int sd_decode(sd_ctx *ctx, const sd_gen_params *p, const int32_t *history, int n_hist, int first_token,
              int32_t *out_tokens, int out_cap, sd_gen_stats *stats);

/* ======================================================================================
 * Tokenizer (host code): the SentencePiece-style BPE of the GGUF vocabulary, token for token the reference's
 * (mistral/tokenizer.h), including its merge order among equal scores.
 * ====================================================================================== */
typedef struct sd_tokenizer sd_tokenizer;

/* Replaces tokenizer_init (mistral/tokenizer.h:121-153): tokenizer.ggml.tokens / scores / token_type and the
 * BOS / EOS ids of the GGUF image (absent scores read as 0, absent types as NORMAL). */
SD_API int sd_tokenizer_create(const void *gguf_base, size_t gguf_len, sd_tokenizer **out);
/* Replaces tokenizer_free (mistral/tokenizer.h:431-442). */
SD_API void sd_tokenizer_free(sd_tokenizer *t);
SD_API int sd_tokenizer_info(const sd_tokenizer *t, int *vocab_size, int *bos_id, int *eos_id);
/* Raw vocabulary entry `id`: its piece (valid while t lives), score and SentencePiece type (1 normal,
 * 2 unknown, 3 control, 4 unused, 6 byte). */
SD_API int sd_tokenizer_entry(const sd_tokenizer *t, int id, const char **piece, float *score, int *type);
/* Replaces tokenizer_encode (mistral/tokenizer.h:200-346): ids of text into out (at most max_tokens, BOS first
 * when add_bos); returns the count or < 0. */
SD_API int sd_tokenizer_encode(const sd_tokenizer *t, const char *text, int32_t *out, int max_tokens, int add_bos);
/* Replaces tokenizer_decode_token (mistral/tokenizer.h:348-373): the text of one token ("" for BOS, EOS and ids
 * out of range; a byte token <0xNN> gives that byte, in a per-thread buffer overwritten by the next call). */
SD_API const char *sd_tokenizer_piece(const sd_tokenizer *t, int token);
/* Replaces tokenizer_decode (mistral/tokenizer.h:375-412): U+2581 becomes a space and one leading space is
 * dropped.  Returns a malloc'd string (release with sd_free) or NULL. */
SD_API char *sd_tokenizer_decode(const sd_tokenizer *t, const int32_t *tokens, int n);
/* Replaces tokenizer_apply_chat (mistral/tokenizer.h:416-429): "[INST] " + msg + " [/INST]", malloc'd. */
SD_API char *sd_tokenizer_apply_chat(const char *user_msg);
/* Release a string returned by this library. */
SD_API void sd_free(void *p);

/* ======================================================================================
 * Batched serving: many independent streams on one GPU sharing a context's weights.  Every stream
 * has its own KV ring and generation state; one forward processes T tokens of every stream with the
 * wide-token W4A8 GEMM (M = n_streams * T rows of int8 MMA work per weight tile read).  Per stream
 * the semantics are those of sd_generate / sd_decode (the reference runs one stream per process), with
 * one difference at temp > 0: stream s draws its uniforms from the Philox stream of seed p->seed + s
 * (the stream sd_generate / sd_decode would use with seed + s), so streams of one batch never share draws.
 * Single-GPU contexts only (tp_size 1).
 * ====================================================================================== */
#define SD_BATCH_MAX_WIDTH 8
typedef struct sd_batch sd_batch;

typedef struct {
    int64_t n_generated;                                   /* over all streams */
    int64_t total_draft, total_accepted, total_iterations; /* decode loop, summed over streams */
    int64_t verify_forwards;                               /* batched forwards of the decode loop */
    double ms_prefill, ms_decode;
} sd_batch_stats;

/* n_streams >= 1; max_seq ring positions per stream; max_width tokens per stream per forward
 * (1..SD_BATCH_MAX_WIDTH; the verify width spec_k + 1 and the prefill chunk; the GEMMs' K splits are planned
 * for it).  The batch reads the context's weights: free every batch before its context.  A batch, like a
 * context, is used by one host thread at a time. */
SD_API int sd_batch_create(sd_ctx *ctx, int n_streams, int max_seq, int max_width, sd_batch **out);
SD_API void sd_batch_free(sd_batch *b);
/* The CUDA stream (cudaStream_t) every sd_batch_* call of this batch is ordered on. */
SD_API void *sd_batch_stream(sd_batch *b);
/* Which tensor-core GEMM the batch's forwards use (no reference counterpart: the reference has one
 * Metal GEMM, q4_0_gemm at mistral/q4_0_metal.metal:264-383).  AUTO (the default): tcgen05 MMA with TMEM
 * accumulators for forwards of at least 64 tokens (n_streams * T), the mma.sync GEMM below that; MMA: always
 * mma.sync; TC: always tcgen05.  Both give bit-identical results.  Drops the batch's captured graphs. */
#define SD_BATCH_GEMM_AUTO 0
#define SD_BATCH_GEMM_MMA 1
#define SD_BATCH_GEMM_TC 2
SD_API int sd_batch_set_gemm(sd_batch *b, int mode);
/* One forward of T <= max_width tokens per stream: tokens [n_streams][T] at positions pos[s] .. pos[s]+T-1
 * (K/V written to each stream's ring); logits: host [n_streams][T][vocab] or NULL. */
SD_API int sd_batch_forward(sd_batch *b, const int32_t *tokens, int T, const int32_t *pos, float *logits);
/* K/V of positions [0, n) of every stream from tokens [n_streams][n] (chunks of max_width tokens). */
SD_API int sd_batch_prefill(sd_batch *b, const int32_t *tokens, int n);
/* Decode of every stream after a prefill of history[s][0 .. n_hist-1): starts from first[s] at position
 * n_hist - 1 (sd_decode per stream).  out: [n_streams][out_cap]; n_out: [n_streams] tokens written. */
SD_API int sd_batch_decode(sd_batch *b, const sd_gen_params *p, const int32_t *history, int n_hist, const int32_t *first,
                           int32_t *out, int out_cap, int32_t *n_out, sd_batch_stats *stats);
/* Prefill + first token + decode of every stream (sd_generate per stream): prompts [n_streams][n_prompt]. */
SD_API int sd_batch_generate(sd_batch *b, const sd_gen_params *p, const int32_t *prompts, int n_prompt, int32_t *out,
                             int out_cap, int32_t *n_out, sd_batch_stats *stats);

#ifdef __cplusplus
}
#endif
#endif /* SPECDEC_B200_H */
