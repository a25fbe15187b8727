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
#include "sd_common.cuh"
#include "sd_attn.h"

namespace sd {

constexpr int kHD = 128;        // head_dim
constexpr int kGQA = 4;         // query heads per kv head
constexpr int kSub = 32;        // positions per sub-block (one per lane)
constexpr int kAttnThreads = 128;

__global__ void __launch_bounds__(kAttnThreads) k_attn_partial(const AttnArgs a) {
    __shared__ float qs[kMaxS * kGQA][kHD];              // 16 KB: query rows r = s*4 + hq
    __shared__ __half kt[kHD][kSub + 2];                 // K sub-block transposed [d][j] (padded)
    __shared__ __align__(16) __half vt[kSub][kHD];       // V sub-block [j][d]
    if (a.ctrl && a.ctrl->done) return;
    pdl_trigger();
    pdl_wait();
    const int nv = a.ctrl ? min(a.ctrl->n_valid, a.S) : a.S;
    if (nv <= 0) return;
    const int pos = a.ctrl ? a.ctrl->pos : a.pos;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hi_max = pos + nv - 1;
    const int lo_min = max(0, pos + 1 - a.max_seq);
    const int c_first = lo_min / a.chunk, c_last = hi_max / a.chunk;
    const int n_items = (c_last - c_first + 1) * a.n_kvh;
    const int hq = warp;                                 // warp w computes query head 4*kvh + w, all tokens

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int kvh = item % a.n_kvh;
        const int c = c_first + item / a.n_kvh;
        const int p0 = max(c * a.chunk, lo_min);
        const int p1 = min((c + 1) * a.chunk, hi_max + 1);  // exclusive
        __syncthreads();
        for (int i = tid; i < kMaxS * kGQA * (kHD / 4); i += kAttnThreads) {
            const int r = i / (kHD / 4), d4 = (i % (kHD / 4)) * 4;
            const int s = r / kGQA, h = r % kGQA;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (s < nv)
                v = *reinterpret_cast<const float4*>(a.q + (size_t)s * a.q_ld + (size_t)(kvh * kGQA + h) * kHD + d4);
            *reinterpret_cast<float4*>(&qs[r][d4]) = v;
        }
        // per-token running state for this warp's head; lane owns dims 4*lane..4*lane+3
        float m[kMaxS], l[kMaxS], acc[kMaxS][4];
#pragma unroll
        for (int s = 0; s < kMaxS; ++s) {
            m[s] = -INFINITY;
            l[s] = 0.f;
            acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0.f;
        }
        for (int sb = p0; sb < p1; sb += kSub) {
            __syncthreads();
            for (int i = tid; i < kSub * (kHD / 8); i += kAttnThreads) {
                const int j = i / (kHD / 8), d8 = (i % (kHD / 8)) * 8;
                const int p = sb + j;
                uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
                if (p < p1) {
                    const size_t off = (size_t)(p % a.max_seq) * a.kv_ld + (size_t)kvh * kHD + d8;
                    kv4 = *reinterpret_cast<const uint4*>(a.k + off);
                    vv4 = *reinterpret_cast<const uint4*>(a.v + off);
                }
                const __half* kh = reinterpret_cast<const __half*>(&kv4);
#pragma unroll
                for (int e = 0; e < 8; ++e) kt[d8 + e][j] = kh[e];
                *reinterpret_cast<uint4*>(&vt[j][d8]) = vv4;
            }
            __syncthreads();
            // scores of (token s, position sb + lane)
            float sc[kMaxS];
#pragma unroll
            for (int s = 0; s < kMaxS; ++s) sc[s] = 0.f;
            for (int d = 0; d < kHD; d += 4) {
                const float k0 = __half2float(kt[d][lane]), k1 = __half2float(kt[d + 1][lane]);
                const float k2 = __half2float(kt[d + 2][lane]), k3 = __half2float(kt[d + 3][lane]);
#pragma unroll
                for (int s = 0; s < kMaxS; ++s) {
                    if (s < nv) {
                        const float4 qv = *reinterpret_cast<const float4*>(&qs[s * kGQA + hq][d]);
                        sc[s] = fmaf(qv.x, k0, sc[s]);
                        sc[s] = fmaf(qv.y, k1, sc[s]);
                        sc[s] = fmaf(qv.z, k2, sc[s]);
                        sc[s] = fmaf(qv.w, k3, sc[s]);
                    }
                }
            }
            const int p = sb + lane;
            float pr[kMaxS];
#pragma unroll
            for (int s = 0; s < kMaxS; ++s) {
                pr[s] = 0.f;
                if (s >= nv) continue;
                const int hi = pos + s, lo = max(0, hi + 1 - a.max_seq);
                const bool ok = p < p1 && p >= lo && p <= hi;
                const float v = ok ? sc[s] : -INFINITY;
                const float mx = warp_max(v);
                const float mn = fmaxf(m[s], mx);
                // a token with nothing valid yet keeps m = -inf and contributes nothing
                const float e = (mn == -INFINITY || !ok) ? 0.f : expf(v - mn);
                const float corr = (mn == -INFINITY || m[s] == -INFINITY) ? 0.f : expf(m[s] - mn);
                const float es = warp_sum(e);
                l[s] = l[s] * corr + es;
                acc[s][0] *= corr;
                acc[s][1] *= corr;
                acc[s][2] *= corr;
                acc[s][3] *= corr;
                m[s] = mn;
                pr[s] = e;
            }
            // acc[s][d] += sum_j pr[s](lane j) * V[j][d]
            for (int j = 0; j < kSub; ++j) {
                const uint2 vraw = *reinterpret_cast<const uint2*>(&vt[j][lane * 4]);
                const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.x));
                const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.y));
#pragma unroll
                for (int s = 0; s < kMaxS; ++s) {
                    if (s < nv) {
                        const float w = __shfl_sync(0xffffffffu, pr[s], j);
                        acc[s][0] = fmaf(w, f01.x, acc[s][0]);
                        acc[s][1] = fmaf(w, f01.y, acc[s][1]);
                        acc[s][2] = fmaf(w, f23.x, acc[s][2]);
                        acc[s][3] = fmaf(w, f23.y, acc[s][3]);
                    }
                }
            }
        }
        const int h = kvh * kGQA + hq;
#pragma unroll
        for (int s = 0; s < kMaxS; ++s) {
            if (s >= nv) continue;
            const size_t pi = ((size_t)s * a.n_heads + h) * a.max_chunks + c;
            if (lane == 0) a.part_ml[pi] = make_float2(m[s], l[s]);
            *reinterpret_cast<float4*>(a.part_acc + pi * kHD + lane * 4) =
                make_float4(acc[s][0], acc[s][1], acc[s][2], acc[s][3]);
        }
    }
}

// Merge chunk partials (fixed chunk order per lane group); quantise each head's 128 outputs to 4
// Q8_0 blocks.  One warp per (token, head): the (max, sum) statistics are read lane-parallel over
// chunks; the 128-wide accumulators with 8 independent loads in flight per lane.
__global__ void k_attn_combine(const AttnArgs a) {
    if (a.ctrl && a.ctrl->done) return;
    pdl_trigger();
    pdl_wait();
    const int nv = a.ctrl ? min(a.ctrl->n_valid, a.S) : a.S;
    const int pos = a.ctrl ? a.ctrl->pos : a.pos;
    const int lane = threadIdx.x & 31;
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (wid >= nv * a.n_heads) return;
    const int s = wid / a.n_heads, h = wid % a.n_heads;
    const int hi = pos + s, lo = max(0, hi + 1 - a.max_seq);
    const int c0 = lo / a.chunk, c1 = hi / a.chunk;
    const size_t base = ((size_t)s * a.n_heads + h) * a.max_chunks;
    float M = -INFINITY;
    for (int c = c0 + lane; c <= c1; c += 32) M = fmaxf(M, a.part_ml[base + c].x);
    M = warp_max(M);
    float L = 0.f;
    for (int c = c0 + lane; c <= c1; c += 32) {
        const float2 ml = a.part_ml[base + c];
        L += (ml.x == -INFINITY) ? 0.f : ml.y * expf(ml.x - M);
    }
    L = warp_sum(L);
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    constexpr int U = 8;
    for (int cb = c0; cb <= c1; cb += U) {
        float4 ac[U];
        float f[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = cb + u;
            if (c <= c1) {
                const float mx = a.part_ml[base + c].x;
                f[u] = (mx == -INFINITY) ? 0.f : expf(mx - M);
                ac[u] = *reinterpret_cast<const float4*>(a.part_acc + (base + c) * kHD + lane * 4);
            } else {
                f[u] = 0.f;
                ac[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            o[0] = fmaf(ac[u].x, f[u], o[0]);
            o[1] = fmaf(ac[u].y, f[u], o[1]);
            o[2] = fmaf(ac[u].z, f[u], o[2]);
            o[3] = fmaf(ac[u].w, f[u], o[3]);
        }
    }
    const float inv = 1.0f / L;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] *= inv;
    if (a.out_f32) {
        float* op = a.out_f32 + (size_t)s * a.n_heads * kHD + (size_t)h * kHD + lane * 4;
        *reinterpret_cast<float4*>(op) = make_float4(o[0], o[1], o[2], o[3]);
    }
    // Q8_0 blocks: dims [32*bk, 32*bk+32) are lanes 8*bk..8*bk+7 (4 values each)
    float am = fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3])));
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    const float d = __fdiv_rn(am, 127.0f);
    int q[4] = {0, 0, 0, 0};
    if (am != 0.0f) {
        const float id = __fdiv_rn(1.0f, d);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = __float2int_rn(__fmul_rn(o[e], id));
            q[e] = r > 127 ? 127 : (r < -128 ? -128 : r);
        }
    }
    int qsum = q[0] + q[1] + q[2] + q[3];
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, off);
    const size_t row_off = (size_t)s * a.n_heads * kHD + (size_t)h * kHD;
    const uint32_t packed = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                            ((uint32_t)(q[3] & 0xFF) << 24);
    *reinterpret_cast<uint32_t*>(a.out.qs + row_off + lane * 4) = packed;
    if ((lane & 7) == 0) {
        const size_t bi = row_off / 32 + (lane >> 3);
        a.out.d[bi] = d;
        a.out.sum[bi] = qsum;
    }
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
    const int warps = a.S * a.n_heads;
    fill_cfg(cfg, at, dim3((warps * 32 + 255) / 256), dim3(256), st, pdl);
    return cudaLaunchKernelEx(&cfg, k_attn_combine, a);
}

}  // namespace sd
