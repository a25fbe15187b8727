// sd_fwd.h -- arguments of the persistent forward kernel (sd_fwd.cu).
#pragma once
#include "sd_attn.h"

namespace sd {

// One matvec phase of the persistent forward; the same plan serves every layer.
// Work item = (K slice, unit); items are ordered slice-major and each CTA takes a contiguous range.
struct MvPhase {
    int n_units;  // units of rpu row-groups (a unit is never split between CTAs)
    int rpu;      // row-groups per unit: kRPW, or 2*kRPW for gate|up (SiLU needs both halves of a unit)
    int nq;       // 128-column quads per row
    int kparts;   // K slices; slice partials are summed by the slice that finishes last
    int chunk;    // tiles per row-group per ring stage (nq / kparts when that is below 16)
};

struct FwdLayer {
    const uint8_t *qkv, *wo, *w13, *w2;  // tile16x4 matrices
    const float *rms_att, *rms_ffn;
};

struct FwdArgs {
    const FwdLayer* layers;  // device array [n_layers]
    int n_layers;
    const uint8_t* embd;     // token embedding rows as in the GGUF: Q4_0 (embd_type 2) or Q4_K (12)
    int embd_type;
    const float* rms_out;    // final norm weight
    const uint8_t* lm;       // output matrix; null = no LM head
    int dim, hidden, q_rows, kv_rows, vocab, head_dim, n_heads, n_kvh;
    int S, max_seq;
    float eps, q_scale;
    const float* theta_inv;
    __half *k_cache, *v_cache;  // [n_layers][max_seq][kv_rows]
    size_t kv_layer;            // max_seq * kv_rows
    MvPhase qkv, wo, w13, w2, lmp;
    int nstage;                 // weight ring stages
    float* x;                   // [S][dim] residual stream
    float* ssq;                 // [S][dim/16] sums of squares of x per 16-row group
    ActImage un_img;            // Q8_0 of x * (next RMSNorm weight), block scales before the norm scale
    ActImage attn_img;          // Q8_0 head outputs (o-proj input)
    ActImage h_img;             // Q8_0 SiLU(gate)*up (down-projection input)
    float* q;                   // [S][q_rows]
    Q8Planes attn;              // [S][q_rows] quantised head outputs (planes; unused when attn_img is set)
    Q8Planes h;                 // [S][hidden] quantised SiLU(gate)*up (planes; unused when h_img is set)
    float* yparts;              // [kparts][S][dim] K-slice partials
    size_t ypart_stride;
    unsigned* sync;             // [0] grid barrier counter; from word 32: argmax keys [kMaxS] u64; zero at launch
    float2* part_ml;            // attention partials
    float* part_acc;
    int attn_chunk, max_chunks;
    float* logits;              // [S][vocab]
    const int* tokens;          // token ids (null: ctrl->tokens)
    const DevCtrl* ctrl;        // pos / n_valid / done (null: pos = 0, all S valid)
    int* err;
    TpXchg tp;                  // tensor parallel over peer memory (tp.n = 0: single GPU)
};

constexpr int kFwdAttnGroups = 2;  // 128-thread attention groups per CTA

size_t fwd_smem_bytes(int nstage);
int fwd_pick_stages(int max_smem);
size_t fwd_sync_words(int dim);
cudaError_t fwd_init_attrs(int max_smem);
cudaError_t fwd_blocks_per_sm(size_t smem, int* n);
cudaError_t launch_forward(const FwdArgs& a, int grid, size_t smem, cudaStream_t st);

}  // namespace sd
