// sd_attn.h -- arguments of the GQA attention kernels (sd_attn.cu).
#pragma once
#include "sd_internal.h"

namespace sd {

struct AttnArgs {
    const float* q;        // [S][q_ld] RoPE'd, pre-scaled by 1/sqrt(head_dim)
    int q_ld;
    const __half* k;       // layer base of the ring: [max_seq][kv_ld]
    const __half* v;
    int kv_ld;
    int n_heads, n_kvh;    // local (this rank's) query / kv heads
    int S, pos;            // pos used when ctrl is null
    int max_seq;
    int chunk;             // positions per split-K chunk (multiple of 32)
    int max_chunks;        // ceil(max_seq / chunk): stride of the partial buffers
    float2* part_ml;       // [S][n_heads][max_chunks] (running max, sum)
    float* part_acc;       // [S][n_heads][max_chunks][128]
    Q8Planes out;          // [S][n_heads*128] quantised head outputs (o-proj input)
    ActImage img;          // if img.b is set: the head outputs go here instead, in the matvec fragment layout
    float* out_f32;        // optional fp32 copy of the head outputs
    const DevCtrl* ctrl;
    // batched path: head outputs of token s go to token tok0 + s of this wide image (if wimg.p is set)
    WImg wimg;
    int tok0;
};

cudaError_t launch_attention(const AttnArgs& a, int grid_partial, cudaStream_t st, bool pdl);

}  // namespace sd
