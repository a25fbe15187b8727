// sd_attn.cu -- 4:1 GQA attention over the fp16 sequence-major KV ring for S <= 8 query tokens.
//
// Replaces gqa_attention_neon (mistral/mistral_model.h:362-487, S=1 decode) and the batched causal
// verify kernel of the Metal path (q4_0_metal.metal:945-1084).  Token s of a forward sits at
// position p = pos + s and attends the ring slots of positions [max(0, p+1-max_seq), p]
// (slot = position % max_seq), i.e. the reference's CPU semantics per token; attention length comes
// from the position, so rejected draft positions are never attended (KV rollback = position reset).
//
// Split-K ("flash decoding"): the position axis is cut into fixed chunks of C absolute positions;
// work item = (kv head, chunk) and processes every query row (4 heads x S tokens) of that kv head,
// so each K/V row is read once per forward.  Partial (max, sum, acc[128]) per (token, head, chunk)
// are merged by k_attn_combine in chunk order, which also quantises the head output to Q8_0 for
// the o-proj matvec.  Chunk boundaries depend only on absolute positions, so a token's result is
// bit-identical whatever S it is computed with.
#include "sd_dev.cuh"

namespace sd {

__global__ void __launch_bounds__(kAttnThreads) k_attn_partial(const AttnArgs a) {
    __shared__ __align__(16) uint8_t smem[attn_smem_bytes()];
    if (a.ctrl && a.ctrl->done) return;
    pdl_trigger();
    pdl_wait();
    const int nv = a.ctrl ? min(a.ctrl->n_valid, a.S) : a.S;
    if (nv <= 0) return;
    const int pos = a.ctrl ? a.ctrl->pos : a.pos;
    const int hi_max = pos + nv - 1;
    const int lo_min = max(0, pos + 1 - a.max_seq);
    const int c_first = lo_min / a.chunk, c_last = hi_max / a.chunk;
    const int n_items = (c_last - c_first + 1) * a.n_kvh;
    const AttnSmem sm = attn_smem_at(smem);
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int nx = item + gridDim.x;  // this CTA's next item, prefetched into L2 during this one
        attn_item(a, nv, pos, lo_min, hi_max, item % a.n_kvh, c_first + item / a.n_kvh, nx % a.n_kvh,
                  nx < n_items ? c_first + nx / a.n_kvh : -1, sm, threadIdx.x, [] { __syncthreads(); });
    }
}

// Merge chunk partials and quantise each head's 128 outputs to 4 Q8_0 blocks: one CTA of
// combine_warps(max_seq) warps per (token, head).
__global__ void __launch_bounds__(kCombineWarpsMax * 32) k_attn_combine(const AttnArgs a) {
    __shared__ __align__(16) float obuf[kCombineWarpsMax * kHD];
    if (a.ctrl && a.ctrl->done) return;
    pdl_trigger();
    pdl_wait();
    const int nv = a.ctrl ? min(a.ctrl->n_valid, a.S) : a.S;
    const int pos = a.ctrl ? a.ctrl->pos : a.pos;
    const int row = blockIdx.x;
    if (row >= nv * a.n_heads) return;
    attn_combine_row(a, blockDim.x >> 5, pos, row / a.n_heads, row % a.n_heads, threadIdx.x >> 5, threadIdx.x & 31,
                     obuf, [] { __syncthreads(); });
}

static void fill_cfg(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* at, dim3 grid, dim3 block, cudaStream_t st, bool pdl) {
    cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
}

cudaError_t launch_attention(const AttnArgs& a, int grid_partial, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[1];
    fill_cfg(cfg, at, dim3(grid_partial), dim3(kAttnThreads), st, pdl);
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn_partial, a);
    if (e != cudaSuccess) return e;
    fill_cfg(cfg, at, dim3(a.S * a.n_heads), dim3(combine_warps(a.max_seq) * 32), st, pdl);
    return cudaLaunchKernelEx(&cfg, k_attn_combine, a);
}

}  // namespace sd
