// sd_host.h -- host-side helpers shared by the C ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include "sd_internal.h"

namespace sd {
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
void clear_error();
int device_sm_count(int dev);
int device_max_smem(int dev);
int* device_error_word(int dev);
int check_device_error(int* word, cudaStream_t st);
int check_current_device(int dev, const char* what);
int repack_matrix(const uint8_t* aos_dev, int rows, int cols, RowMap map, uint8_t* dst, cudaStream_t st);
// Plan + launch a matvec.  a.kparts <= 0 lets the planner choose; a.kparts == 1 forces one slice.
// For EPI_STORE with a K split the partial outputs go to a.out + p*a.part_stride (the caller sums).
int gemv_prepare_device(int dev);
int gemv_plan(GemvArgs& a, int dev, int* grid, size_t* smem);
int gemv_plan_fixed(GemvArgs& a, int dev, int* grid, size_t* smem);
int run_gemv(int epi, const GemvArgs& a, int dev, cudaStream_t st, bool pdl);
// Sum-all-reduce of n fp32 values in place over an NCCL communicator (sd_nccl.cu).
int nccl_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st);

// A context's device-resident model, as the batched engine (sd_batch.cu) reads it.
constexpr int kMaxLayers = 128;
struct ModelView {
    int dev, tp_size;
    int dim, hidden, n_layers, n_heads, n_kv, hd, vocab, eos;
    float eps;
    int q_rows, kv_rows, qkv_rows;
    const uint8_t *qkv[kMaxLayers], *wo[kMaxLayers], *w13[kMaxLayers], *w2[kMaxLayers];  // tile16x4
    const float *rms_att[kMaxLayers], *rms_ffn[kMaxLayers];
    const uint8_t* embd;  // Q4_0 AoS [vocab][dim/32] (embd_type 2) or Q4_K rows (12)
    int embd_type;
    const uint8_t* lm;    // tile16x4 [vocab][dim] (lm_type 2) or a K-quant layout (sd_kquant.h)
    int lm_type;
    const float* rms_final;
    const float* theta_inv;
    int* err;             // the context's device error word
};
}  // namespace sd

struct sd_ctx;
struct sd_batch;
int sd_ctx_model_view(sd_ctx* c, sd::ModelView* out);  // defined in sd_engine.cu

namespace sd {
// A batch of n_slices x width tokens per forward whose streams all address the context's own K/V ring
// (kc / vc: [layer][max_seq][kv_rows] fp16) and run on the context's stream: single-stream prompt prefill
// through the wide GEMMs (sd_batch.cu).  Released with sd_batch_free.
int batch_create_prefill(sd_ctx* ctx, int n_slices, int width, void* kc, void* vc, int max_seq, cudaStream_t st,
                         sd_batch** out);
// Write the K/V of prompt tokens [0, n) at positions start_pos .. into that ring (no logits).
int batch_prefill_ring(sd_batch* b, const int32_t* tokens, int n, int start_pos);
}  // namespace sd
