// sd_batch.cu -- batched serving: n independent streams on one GPU, each with its own KV ring and
// generation state, sharing one context's weights.
//
// The reference serves one stream per process (mistral/mistral_infer.m:252-391 per stream); here one
// forward carries T tokens of every stream (T = spec_k + 1 for the verify, up to 8 for prefill chunks),
// M = n_streams * T tokens in all, so every weight tile read from HBM feeds M tokens of int8 MMA work:
//   embed + RMSNorm + Q8_0            k_bnorm<0>              (one CTA per token, wide-image output)
//   per layer:
//     QKV GEMM                        k_wgemm<WG_STORE>       (K-split partials)
//     RoPE + KV write                 k_brope_kv              (each stream's own ring, position pos_s + j)
//     GQA attention + Q8_0            k_battn_partial, k_battn_combine (items per stream x kv head x chunk)
//     o-proj GEMM                     k_wgemm<WG_STORE>
//     residual + RMSNorm + Q8_0       k_bnorm<1>
//     gate|up GEMM + SiLU + Q8_0      k_wgemm<WG_SILU>
//     down GEMM                       k_wgemm<WG_STORE>
//     residual + next RMSNorm + Q8_0  k_bnorm<1>
//   LM head                           k_wgemm<WG_STORE>, k_argmax
// Per token the arithmetic is the single-stream forward's (sd_engine.cu): the same quantizer, per-block
// W4A8 products, RoPE, attention item and combine, in orders that do not depend on the other streams, so
// a stream's tokens do not depend on what the other streams hold.  Per stream, drafting, acceptance and
// emission are the single-stream kernels (sd_spec.cu), one CTA per stream.  Tokens of a stream beyond its
// valid count (fewer drafts than T - 1, or a finished stream) are computed with stale activations and
// dropped: they write no K/V and no output.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <vector>

#include "sd_dev.cuh"
#include "sd_host.h"
#include "sd_spec.h"
#include "specdec_b200.h"

using namespace sd;

static_assert(sd::kMaxS == SD_BATCH_MAX_WIDTH, "batch width differs between the ABI and the kernels");

namespace sd {
namespace {

// ---------------------------------------------------------------------------------------------
// Per-token kernels.  Token m of a forward is token j = m % T of stream b = m / T.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ bool token_valid(const DevCtrl* ctrl, int m, int T, int* b_out, int* j_out) {
    const int b = m / T, j = m - b * T;
    *b_out = b;
    *j_out = j;
    const DevCtrl& c = ctrl[b];
    return !c.done && j < c.n_valid;
}

constexpr int kBNormThreads = 1024;

struct BNormArgs {
    float* x;             // [M][dim] residual stream
    const float* y;       // [yparts][M][dim] (MODE 1), slices summed in order
    size_t ystride;
    int yparts;
    const uint8_t* embd;  // Q4_0 AoS [vocab][dim/32] (MODE 0)
    const float* w;       // RMSNorm weight
    WImg out;             // Q8_0 of the normalised row
    int dim, T;
    float eps;
    const DevCtrl* ctrl;  // [n_streams]
};

// Residual add / embed + RMSNorm + Q8_0 of one token (the arithmetic of k_norm_quant, sd_quant.cu).
template <int MODE>
__global__ void __launch_bounds__(kBNormThreads) k_bnorm(const BNormArgs a) {
    __shared__ __align__(16) float vs[4096];
    __shared__ float gss[256];
    __shared__ float scale;
    int b, j;
    const int m = blockIdx.x;
    if (!token_valid(a.ctrl, m, a.T, &b, &j)) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = a.dim >> 5, bpw = nb >> 5;
    float* x = a.x + (size_t)m * a.dim;
    float v[4], wv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v[k] = wv[k] = 0.f;
        if (k < bpw) {
            const int e = (warp + 32 * k) * 32 + lane;
            wv[k] = a.w[e];
            if constexpr (MODE == 0) {
                const int token = a.ctrl[b].tokens[j];
                v[k] = q4_0_value(a.embd + ((size_t)token * nb + (warp + 32 * k)) * 18, lane);
            } else {
                v[k] = x[e];
            }
        }
    }
    if constexpr (MODE == 1) {
        float yv[4] = {0.f, 0.f, 0.f, 0.f};
        for (int p = 0; p < a.yparts; ++p) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (k < bpw) yv[k] += a.y[(size_t)p * a.ystride + (size_t)m * a.dim + (warp + 32 * k) * 32 + lane];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = v[k] + yv[k];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
        if (k < bpw) {
            const int e = (warp + 32 * k) * 32 + lane;
            vs[e] = v[k];
            x[e] = v[k];
        }
    __syncthreads();
    const int ngroups = a.dim >> 4;
    if ((int)threadIdx.x < ngroups) gss[threadIdx.x] = group16_sumsq(&vs[threadIdx.x * 16]);
    __syncthreads();
    if (warp == 0) {
        const float tot = row_sumsq(gss, ngroups, lane);
        if (lane == 0) scale = rms_scale(tot, a.dim, a.eps);
    }
    __syncthreads();
    const float s = scale;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if (k >= bpw) continue;
        const int blk = warp + 32 * k;
        // Q8_0 of u = x*w with the block scale times s (the codes do not depend on s > 0)
        const float u = v[k] * wv[k];
        float du;
        int sum;
        const int q = q8_quant_lane(u, &du, &sum);
        uint32_t word = (uint32_t)(q & 0xFF) << (8 * (lane & 3));
        word |= __shfl_xor_sync(0xffffffffu, word, 1);
        word |= __shfl_xor_sync(0xffffffffu, word, 2);
        if ((lane & 3) == 0) wimg_put_word(a.out, m, blk, lane >> 2, word);
        if (lane == 0) wimg_put_meta(a.out, m, blk, du * s, sum);
    }
}

struct BRopeArgs {
    const float* qkv;     // [kparts][M][qkv_rows] GEMM partials
    size_t pstride;
    int kparts;
    float* q;             // [M][q_rows]: RoPE'd, times q_scale
    __half *k, *v;        // this layer's ring of stream 0: [max_seq][kv_rows]; stream b at + b * kv_stream
    size_t kv_stream;
    int q_rows, kv_rows, max_seq, head_dim, T;
    const float* theta_inv;
    float q_scale;
    const DevCtrl* ctrl;
};

// RoPE of q and k (mistral/mistral_model.h:79-122, the matvec epilogue's arithmetic) and the fp16 K/V write
// at slot (pos + j) % max_seq of the token's stream.
__global__ void __launch_bounds__(256) k_brope_kv(const BRopeArgs a) {
    int b, j;
    const int m = blockIdx.x;
    if (!token_valid(a.ctrl, m, a.T, &b, &j)) return;
    const int tpos = a.ctrl[b].pos + j;
    const int rows = a.q_rows + 2 * a.kv_rows;
    const float* src = a.qkv + (size_t)m * rows;
    const size_t ring = (size_t)b * a.kv_stream + (size_t)(tpos % a.max_seq) * a.kv_rows;
    for (int pr = threadIdx.x; pr < rows / 2; pr += blockDim.x) {
        const int gr = 2 * pr;
        float ve = 0.f, vo = 0.f;
        for (int p = 0; p < a.kparts; ++p) {
            const float2 t2 = *reinterpret_cast<const float2*>(src + (size_t)p * a.pstride + gr);
            ve += t2.x;
            vo += t2.y;
        }
        if (gr < a.q_rows + a.kv_rows) {
            const int i = (gr % a.head_dim) >> 1;
            const float ang = a.theta_inv[i] * (float)tpos;
            float sn, cs;
            sincosf(ang, &sn, &cs);
            const float e2 = fmaf(-vo, sn, ve * cs);
            const float o2 = fmaf(ve, sn, vo * cs);
            if (gr < a.q_rows) {
                *reinterpret_cast<float2*>(a.q + (size_t)m * a.q_rows + gr) = make_float2(e2 * a.q_scale, o2 * a.q_scale);
            } else {
                *reinterpret_cast<__half2*>(a.k + ring + (gr - a.q_rows)) = __halves2half2(__float2half_rn(e2), __float2half_rn(o2));
            }
        } else {
            *reinterpret_cast<__half2*>(a.v + ring + (gr - a.q_rows - a.kv_rows)) =
                __halves2half2(__float2half_rn(ve), __float2half_rn(vo));
        }
    }
}

struct BAttnArgs {
    AttnArgs a;        // stream 0's view (q, ring, partial buffers); a.S = T, a.wimg = o-proj input image
    size_t kv_stream;  // halves between consecutive streams' rings
    int T;
    int n_streams;
    const DevCtrl* ctrl;
};

__device__ __forceinline__ AttnArgs stream_view(const BAttnArgs& ba, int b) {
    AttnArgs v = ba.a;
    v.q = ba.a.q + (size_t)b * ba.T * ba.a.q_ld;
    v.k = ba.a.k + (size_t)b * ba.kv_stream;
    v.v = ba.a.v + (size_t)b * ba.kv_stream;
    const size_t rows = (size_t)b * ba.T * ba.a.n_heads * ba.a.max_chunks;
    v.part_ml = ba.a.part_ml + rows;
    v.part_acc = ba.a.part_acc + rows * kHD;
    v.tok0 = b * ba.T;
    v.ctrl = nullptr;
    return v;
}

// ---------------------------------------------------------------------------------------------
// Batched attention item: every query row (4 heads x nv tokens) of one stream's kv head kvh over chunk c.
// The online softmax is that of attn_item (sd_dev.cuh), with three changes for throughput over the many
// streams' rings (together ~1 GB of K/V per layer at 64 x 4096 positions):
//  - K/V sub-blocks of 32 positions stream into a kBStages-slot shared-memory ring by cp.async (no register
//    round trip; two pairs of sub-blocks in flight while one pair is computed, one barrier per pair);
//  - Q and the probabilities P enter the fp16 MMAs as single fp16 values (relative error ~5e-4 on the head
//    outputs, which are then quantised to Q8_0 with steps of 1/254);
//  - the two warps of an n-tile split each sub-block's positions (16 each) and keep separate running states
//    over all 128 output dims, merged at the end of the item, so no score tile is computed twice.
// ---------------------------------------------------------------------------------------------
constexpr int kBPair = 2;    // sub-blocks per barrier
constexpr int kBStages = 6;  // ring slots: three pairs (one computed, two in flight)
constexpr size_t kBStageHalves = (size_t)2 * kSub * kQStride;  // K then V of one sub-block
constexpr size_t battn_smem_bytes() { return ((size_t)kQRows * kQStride + kBStages * kBStageHalves) * 2; }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_pair() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Sub-block at positions [sb, sb + 32) of kv head column col0 into ring slot `slot` (zero past p1).
__device__ __forceinline__ void battn_issue(const AttnArgs& a, __half* ring, int slot, int sb, int p1, int col0, int tid) {
    __half* kk = ring + (size_t)slot * kBStageHalves;
    __half* vv = kk + kSub * kQStride;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int i = tid + u * kAttnThreads;
        const int j = i >> 4, d8 = (i & 15) * 8;
        const int p = sb + j;
        const bool ok = p < p1;
        const size_t off = ok ? (size_t)ring_slot(p, a.max_seq) * a.kv_ld + col0 + d8 : 0;
        cp_async16(smem_u32(kk + j * kQStride + d8), a.k + off, ok ? 16u : 0u);
        cp_async16(smem_u32(vv + j * kQStride + d8), a.v + off, ok ? 16u : 0u);
    }
}

__device__ void battn_item(const AttnArgs& a, int nv, int pos, int lo_min, int hi_max, int kvh, int c, __half* qh,
                           __half* ring, float* xch, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nt = warp & 3, ph = warp >> 2;  // n-tile; which 16 positions of each sub-block (m-tile ph)
    const bool active = 2 * nt < nv;
    const int p0 = max(c * a.chunk, lo_min);
    const int p1 = min((c + 1) * a.chunk, hi_max + 1);
    const int lo_max = max(0, pos + nv - a.max_seq);
    const int col0 = kvh * kHD;
    const int nsb = (p1 - p0 + kSub - 1) / kSub;
    const int npair = (nsb + kBPair - 1) / kBPair;
    __syncthreads();  // the previous item is done with Q, the ring and the exchange buffer
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
#pragma unroll
        for (int h = 0; h < kBPair; ++h) {
            const int ib = jp * kBPair + h;
            if (ib < nsb) battn_issue(a, ring, ib, p0 + ib * kSub, p1, col0, tid);
        }
        cp_async_commit();
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = tid + u * kAttnThreads;
        const int r = i >> 5, d4 = (i & 31) * 4;
        const int s = r >> 2, h = r & 3;
        float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s < nv) qv = *reinterpret_cast<const float4*>(a.q + (size_t)s * a.q_ld + (size_t)(kvh * kGQA + h) * kHD + d4);
        *reinterpret_cast<uint2*>(qh + r * kQStride + d4) =
            make_uint2(h2u(__floats2half2_rn(qv.x, qv.y)), h2u(__floats2half2_rn(qv.z, qv.w)));
    }
    const int lr = lane & 7, lq = lane >> 3;
    const uint32_t q_a = smem_u32(qh + (nt * 8 + lr) * kQStride + (lq & 1) * 8);
    // K (A of S^T) for m-tile ph; V (A of O^T via .trans) for the same 16 positions, all 128 dims
    const uint32_t k_off = (uint32_t)(((ph * 16 + lr + (lq & 1) * 8) * kQStride + (lq >> 1) * 8) * 2);
    const uint32_t v_off = (uint32_t)(((kSub + ph * 16 + lr + (lq >> 1) * 8) * kQStride + (lq & 1) * 8) * 2);
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    for (int jp = 0; jp < npair; ++jp) {
        cp_async_wait_pair();
        __syncthreads();  // pair jp landed for every thread; the slots of pair jp - 1 are free
#pragma unroll
        for (int h = 0; h < kBPair; ++h) {
            const int ib = (jp + 2) * kBPair + h;
            if (ib < nsb) battn_issue(a, ring, ib % kBStages, p0 + ib * kSub, p1, col0, tid);
        }
        cp_async_commit();
        if (!active) continue;
#pragma unroll 1
        for (int h = 0; h < kBPair; ++h) {
            const int ib = jp * kBPair + h;
            if (ib >= nsb) break;
            const int sb = p0 + ib * kSub;
            const uint32_t slot = smem_u32(ring + (size_t)(ib % kBStages) * kBStageHalves);
            const uint32_t k_a = slot + k_off, v_a = slot + v_off;
            // ---- S^T: positions sb + 16 ph + (g, g+8) x rows 8 nt + (2t, 2t+1) ----
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < kHD / 16; ++ks) {
                uint32_t b0, b1, k0, k1, k2, k3;
                ldsm_x2(q_a + ks * 32, b0, b1);
                ldsm_x4(k_a + ks * 32, k0, k1, k2, k3);
                mma_f16(sc, k0, k1, k2, k3, b0, b1);
            }
            const int pb = sb + ph * 16;
            if (pb + 16 > p1 || pb + 15 > pos || pb < lo_max) {
                const int s = 2 * nt + (t >> 1);
                const int hi = pos + s, lo = max(0, hi + 1 - a.max_seq);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int p = pb + g + (e >> 1) * 8;
                    if (!(s < nv && p < p1 && p >= lo && p <= hi)) sc[e] = -INFINITY;
                }
            }
            float x0 = fmaxf(sc[0], sc[2]), x1 = fmaxf(sc[1], sc[3]);
#pragma unroll
            for (int o2 = 4; o2 < 32; o2 <<= 1) {
                x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, o2));
                x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, o2));
            }
            const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
            const float c0 = (m0 == -INFINITY) ? 0.f : exp_fast(m0 - n0);
            const float c1 = (m1 == -INFINITY) ? 0.f : exp_fast(m1 - n1);
            sc[0] = sc[0] == -INFINITY ? 0.f : exp_fast(sc[0] - n0);
            sc[1] = sc[1] == -INFINITY ? 0.f : exp_fast(sc[1] - n1);
            sc[2] = sc[2] == -INFINITY ? 0.f : exp_fast(sc[2] - n0);
            sc[3] = sc[3] == -INFINITY ? 0.f : exp_fast(sc[3] - n1);
            m0 = n0;
            m1 = n1;
            l0 = l0 * c0 + (sc[0] + sc[2]);
            l1 = l1 * c1 + (sc[1] + sc[3]);
            if (c0 != 1.0f || c1 != 1.0f) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    o[i][0] *= c0;
                    o[i][1] *= c1;
                    o[i][2] *= c0;
                    o[i][3] *= c1;
                }
            }
            // ---- O^T (dims 16 i + (g, g+8) x rows 2t, 2t+1) += V^T P^T over the 16 positions ----
            const uint32_t ph0 = movm_t(h2u(__floats2half2_rn(sc[0], sc[1])));
            const uint32_t ph1 = movm_t(h2u(__floats2half2_rn(sc[2], sc[3])));
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t v0, v1, v2, v3;
                ldsm_x4_t(v_a + i * 32, v0, v1, v2, v3);
                mma_f16(o[i], v0, v1, v2, v3, ph0, ph1);
            }
        }
    }
    // ---- merge the two position halves of each n-tile (warp nt + 4 hands its state to warp nt) ----
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o2);
    }
    float* xw = xch + (size_t)nt * (36 * 32);  // [36][32]: o[8][4], m0, m1, l0, l1 per lane
    __syncthreads();  // the exchange buffer overlays the ring: every warp is done with the last sub-blocks
    if (ph == 1 && active) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) xw[(i * 4 + e) * 32 + lane] = o[i][e];
        xw[32 * 32 + lane] = m0;
        xw[33 * 32 + lane] = m1;
        xw[34 * 32 + lane] = l0;
        xw[35 * 32 + lane] = l1;
    }
    __syncthreads();
    if (ph != 0 || !active) return;
    {
        const float bm0 = xw[32 * 32 + lane], bm1 = xw[33 * 32 + lane];
        const float bl0 = xw[34 * 32 + lane], bl1 = xw[35 * 32 + lane];
        const float M0 = fmaxf(m0, bm0), M1 = fmaxf(m1, bm1);
        const float fa0 = (m0 == -INFINITY) ? 0.f : exp_fast(m0 - M0), fb0 = (bm0 == -INFINITY) ? 0.f : exp_fast(bm0 - M0);
        const float fa1 = (m1 == -INFINITY) ? 0.f : exp_fast(m1 - M1), fb1 = (bm1 == -INFINITY) ? 0.f : exp_fast(bm1 - M1);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[i][0] = o[i][0] * fa0 + xw[(i * 4 + 0) * 32 + lane] * fb0;
            o[i][1] = o[i][1] * fa1 + xw[(i * 4 + 1) * 32 + lane] * fb1;
            o[i][2] = o[i][2] * fa0 + xw[(i * 4 + 2) * 32 + lane] * fb0;
            o[i][3] = o[i][3] * fa1 + xw[(i * 4 + 3) * 32 + lane] * fb1;
        }
        l0 = l0 * fa0 + bl0 * fb0;
        l1 = l1 * fa1 + bl1 * fb1;
        m0 = M0;
        m1 = M1;
    }
    const int r0 = nt * 8 + 2 * t;
    const int s = 2 * nt + (t >> 1);
    if (s < nv) {
        const size_t pi = ((size_t)s * a.n_heads + kvh * kGQA + (r0 & 3)) * a.max_chunks + c;
        float* acc0 = a.part_acc + pi * kHD;
        float* acc1 = acc0 + (size_t)a.max_chunks * kHD;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int d = 16 * i + g;
            acc0[d] = o[i][0];
            acc1[d] = o[i][1];
            acc0[d + 8] = o[i][2];
            acc1[d + 8] = o[i][3];
        }
        if (g == 0) {
            a.part_ml[pi] = make_float2(m0, l0);
            a.part_ml[pi + a.max_chunks] = make_float2(m1, l1);
        }
    }
}

// Work items (stream, kv head, chunk): every stream owns max_chunks * n_kvh item slots (the slots past its
// ring's chunks, and those of finished streams, are skipped), and one resident wave of CTAs (two per SM)
// walks the whole list with a grid stride, so no CTA runs in a second, nearly empty wave.
__global__ void __launch_bounds__(kAttnThreads, 2) k_battn_partial(const BAttnArgs ba) {
    extern __shared__ __align__(16) uint8_t dsm[];
    __half* qh = reinterpret_cast<__half*>(dsm);
    __half* ring = qh + kQRows * kQStride;
    float* xch = reinterpret_cast<float*>(ring);  // merge buffer of the two position halves, after the ring is drained
    const int per_stream = ba.a.max_chunks * ba.a.n_kvh;
    const int n_slots = ba.n_streams * per_stream;
    for (int item = blockIdx.x; item < n_slots; item += gridDim.x) {
        const int b = item / per_stream, local = item - b * per_stream;
        const DevCtrl& c = ba.ctrl[b];
        const int nv = c.done ? 0 : min(c.n_valid, ba.T);
        if (nv <= 0) continue;
        const AttnArgs a = stream_view(ba, b);
        const int pos = c.pos;
        const int hi_max = pos + nv - 1;
        const int lo_min = max(0, pos + 1 - a.max_seq);
        const int c_first = lo_min / a.chunk, c_last = hi_max / a.chunk;
        if (local >= (c_last - c_first + 1) * a.n_kvh) continue;
        battn_item(a, nv, pos, lo_min, hi_max, local % a.n_kvh, c_first + local / a.n_kvh, qh, ring, xch, threadIdx.x);
    }
    cp_async_wait_all();
}

// Merge of the chunk partials of one (token, head) row and its Q8_0 quantisation into the o-proj image: one
// warp per row, eight rows per CTA.  Lane l holds the (max, sum) pair of chunk c0 + l; every chunk's max and sum
// and the first eight chunks' 128-dim partials (lane = 4 dims) are loaded in one round trip.  The chunks are
// merged in chunk order (M = max of the maxima, L = sum of sum * exp(max - M) in lane order then butterfly,
// o = sum of partial * exp(max - M) in chunk order, o / L), the arithmetic of the single-stream combine with all
// chunks in one warp, so a row's result depends only on its own partials.
constexpr int kBCombWarps = 8;

__global__ void __launch_bounds__(kBCombWarps * 32) k_battn_combine(const BAttnArgs ba) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kBCombWarps + warp;
    if (row >= ba.n_streams * ba.T * ba.a.n_heads) return;
    const int m = row / ba.a.n_heads, h = row - m * ba.a.n_heads;
    int b, s;
    if (!token_valid(ba.ctrl, m, ba.T, &b, &s)) return;
    const AttnArgs a = stream_view(ba, b);
    const int hi = ba.ctrl[b].pos + s, lo = max(0, hi + 1 - a.max_seq);
    const int c0 = lo / a.chunk, c1 = hi / a.chunk;
    const size_t base = ((size_t)s * a.n_heads + h) * a.max_chunks;
    constexpr int U = 8;
    float4 ac[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
        ac[u] = c0 + u <= c1 ? *reinterpret_cast<const float4*>(a.part_acc + (base + c0 + u) * kHD + lane * 4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    const float2 ml0 = c0 + lane <= c1 ? a.part_ml[base + c0 + lane] : make_float2(-INFINITY, 0.f);
    float M = ml0.x;
    for (int c = c0 + 32 + lane; c <= c1; c += 32) M = fmaxf(M, a.part_ml[base + c].x);
    M = warp_max(M);
    float L = (ml0.x == -INFINITY) ? 0.f : ml0.y * expf(ml0.x - M);
    for (int c = c0 + 32 + lane; c <= c1; c += 32) {
        const float2 ml = a.part_ml[base + c];
        L += (ml.x == -INFINITY) ? 0.f : ml.y * expf(ml.x - M);
    }
    L = warp_sum(L);
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int cc = c0; cc <= c1; cc += U) {
        if (cc > c0) {
#pragma unroll
            for (int u = 0; u < U; ++u)
                ac[u] = cc + u <= c1 ? *reinterpret_cast<const float4*>(a.part_acc + (base + cc + u) * kHD + lane * 4)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = cc + u;
            if (c > c1) break;
            const float mx = c - c0 < 32 ? __shfl_sync(0xffffffffu, ml0.x, c - c0) : a.part_ml[base + c].x;
            const float f = (mx == -INFINITY) ? 0.f : expf(mx - M);
            o[0] = fmaf(ac[u].x, f, o[0]);
            o[1] = fmaf(ac[u].y, f, o[1]);
            o[2] = fmaf(ac[u].z, f, o[2]);
            o[3] = fmaf(ac[u].w, f, o[3]);
        }
    }
    const float inv = 1.0f / L;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] *= inv;
    // Q8_0 blocks: dims [32*bk, 32*bk+32) are lanes 8*bk..8*bk+7 (4 values each), as attn_combine_row
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
    const uint32_t packed = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                            ((uint32_t)(q[3] & 0xFF) << 24);
    const int blk = h * (kHD / 32) + (lane >> 3);
    wimg_put_word(a.wimg, a.tok0 + s, blk, lane & 7, packed);
    if ((lane & 7) == 0) wimg_put_meta(a.wimg, a.tok0 + s, blk, d, qsum);
}

// Control blocks of a forward of T tokens per stream: tokens[b * stride + col0 + j], position pos[b] (or col0).
__global__ void k_bset_ctrl(DevCtrl* ctrl, int n, const int* tokens, int stride, int col0, int T, const int* pos) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    DevCtrl& c = ctrl[b];
    for (int j = 0; j < T; ++j) c.tokens[j] = tokens[(size_t)b * stride + col0 + j];
    c.pos = pos ? pos[b] : col0;
    c.n_valid = T;
    c.done = 0;
}

// Generation state of stream b from host-chosen fields: history row b of hist_src (stride), current
// token cur[b] (or 0), position pos (same for all streams).
__global__ void k_binit_gen(GenState* gs, int n, GenState tmpl, int* out, int* hist, int cap, const int* hist_src,
                            int hstride, int n_hist, const int* cur, unsigned long long seed) {
    const int b = blockIdx.x;
    if (b >= n) return;
    for (int i = threadIdx.x; i < n_hist; i += blockDim.x) hist[(size_t)b * cap + i] = hist_src[(size_t)b * hstride + i];
    if (threadIdx.x == 0) {
        GenState g = tmpl;
        g.out = out + (size_t)b * cap;
        g.hist = hist + (size_t)b * cap;
        g.cur = cur ? cur[b] : 0;
        g.seed = seed + (unsigned long long)b;
        gs[b] = g;
    }
}

// ---------------------------------------------------------------------------------------------
// GEMM planning: the unit shape (token tile, K split) with the least estimated time.
// ---------------------------------------------------------------------------------------------
struct WgPlan {
    WGemmArgs a{};
    int grid = 0;
    size_t smem = 0;
    bool tc = false;  // tcgen05 GEMM (sd_tcgemm.cu) instead of k_wgemm
};

// Cost model in ns: a quad (128 columns) of a unit costs (0.8 + n8 tiles per warp) x 800 ns (the A-fragment
// work of a quad is worth most of one n8 tile; 800 ns is the measured QKV unit time at M = 320 over its quads);
// a unit adds about one quad of fill / epilogue; K-split partial slices are written and read back at ~6.5 TB/s.
void wg_plan(WgPlan& p, int epi, int rows, int K, int M, int kp_lo, int kp_max, int sms, int max_smem) {
    const int n_rt = wide_row_tiles(rows);
    const int nq = K / 128;
    const int NT = (M + 7) / 8;
    double best = 1e300;
    int bt = kWgTokGroups, bk = kp_lo;
    for (int tt = kWgTokGroups; tt <= kWgMaxTT; tt += kWgTokGroups) {
        if (tt > kWgTokGroups && tt - kWgTokGroups >= NT) break;  // wider tiles than the tokens add nothing
        const int n_tt = (NT + tt - 1) / tt;
        const int per = (std::min(tt, NT) + kWgTokGroups - 1) / kWgTokGroups;
        for (int kp = kp_lo; kp <= kp_max; ++kp) {
            if (kp > kp_lo && nq / kp < 2) break;
            const long long units = (long long)n_rt * kp * n_tt;
            const long long waves = (units + sms - 1) / sms;
            double t = (double)waves * ((double)nq / kp + 1.0) * (0.8 + per) * 800.0;
            if (kp > 1) t += (double)kp * M * rows * 8.0 / 6500.0;
            if (t < best * 0.999) {
                best = t;
                bt = tt;
                bk = kp;
            }
        }
    }
    WGemmArgs& a = p.a;
    a = WGemmArgs{};
    a.n_rt = n_rt;
    a.nq = nq;
    a.NT = NT;
    a.M = M;
    a.tt_n8 = bt;
    a.n_tt = (NT + bt - 1) / bt;
    a.kparts = epi == WG_SILU ? 1 : bk;
    a.stage_bytes = kWgWStage + bt * kWSeg;
    a.nstage = std::min(kWgMaxStages, (int)((max_smem - 2 * kWgMaxStages * 8) / a.stage_bytes));
    const long long units = (long long)n_rt * a.kparts * a.n_tt;
    p.grid = (int)std::min<long long>(units, sms);
    p.smem = wgemm_smem_bytes(bt, a.nstage);
}

// The tcgen05 form of a k_wgemm plan: the same K split (so both GEMMs give the same bits), token tiles of at
// most 128 tokens in an even number of n8 tiles (the MMA's N is a multiple of 16), as many ring stages as fit.
void tc_plan(WgPlan& p, int epi, int sms, int max_smem) {
    WGemmArgs& a = p.a;
    const int n_tt = (a.NT + kTcMaxTT - 1) / kTcMaxTT;
    int tt = (a.NT + n_tt - 1) / n_tt;
    tt += tt & 1;
    a.tt_n8 = tt;
    a.n_tt = (a.NT + tt - 1) / tt;
    a.stage_bytes = kWgWStage + tt * kWSeg + kTcAStage;
    a.nstage = std::min(kTcMaxStages, (int)(((size_t)max_smem - tcgemm_smem_bytes(tt, 0, epi)) / a.stage_bytes));
    const long long units = (long long)a.n_rt * a.kparts * a.n_tt;
    p.grid = (int)std::min<long long>(units, sms);
    p.smem = tcgemm_smem_bytes(tt, a.nstage, epi);
    p.tc = true;
}

struct BPlans {
    bool ready = false;
    bool tc = false;  // this width's forwards use the tcgen05 GEMM and the tensor-core image arrangement
    WgPlan qkv, wo, w13, w2, lm;
};

}  // namespace
}  // namespace sd

struct sd_batch {
    sd_ctx* ctx = nullptr;
    ModelView m{};
    // the context's matrices repacked into the wide GEMM layout (sd_batch.h)
    std::vector<uint8_t*> wqkv, wwo, ww13, ww2;
    uint8_t* wlm = nullptr;
    int dev = 0, sms = 0, max_smem = 0;
    cudaStream_t st = nullptr;
    int B = 0, W = 0, max_seq = 0, M_max = 0;
    int chunk = 512, max_chunks = 0, kp_max = 8;  // attention: positions per item (partials per 512 positions)
    __half *kc = nullptr, *vc = nullptr;  // [n_layers][B][max_seq][kv_rows]
    size_t kv_stream = 0, kv_layer = 0;
    float *x = nullptr, *y = nullptr, *qkv = nullptr, *q = nullptr;
    uint8_t *img_x = nullptr, *img_attn = nullptr, *img_h = nullptr;
    float2* part_ml = nullptr;
    float* part_acc = nullptr;
    float* logits = nullptr;  // [M_max][vocab]
    int* argmax = nullptr;    // [M_max]
    float* probs = nullptr;   // [B][vocab]
    DevCtrl* ctrl = nullptr;  // [B]
    int* tok = nullptr;       // token staging (prefill / forward inputs)
    size_t tok_cap = 0;
    int* pos_dev = nullptr;   // [B]
    GenState* gs = nullptr;   // [B]
    GenState* gs_h = nullptr; // pinned [B]
    int *g_out = nullptr, *g_hist = nullptr;
    int g_cap = 0;
    int* ndone = nullptr;     // [2]: streams done, most tokens a live stream still has to generate
    int* ndone_h = nullptr;   // pinned copy
    int gemm_mode = SD_BATCH_GEMM_AUTO;
    bool shared_ring = false;  // kc / vc and st belong to the context (GEMM prefill of a single stream)
    BPlans plans[SD_BATCH_MAX_WIDTH + 1];
    cudaGraphExec_t fwd_graph[SD_BATCH_MAX_WIDTH + 1][2] = {};
    cudaGraphExec_t iter_graph = nullptr;
    int iter_T = -1;
    GenParamsDev iter_p{};
};

namespace {

int ck(cudaError_t e, const char* what) { return e == cudaSuccess ? SD_OK : cuda_fail(e, what); }

#define CK(expr, what)                 \
    do {                               \
        int _rc = ck((expr), (what));  \
        if (_rc) return _rc;           \
    } while (0)

template <class T>
int dalloc(T** p, size_t n) {
    cudaError_t e = cudaMalloc((void**)p, n * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    return SD_OK;
}

double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Plans for T tokens per stream.  The K split of each matrix is the one chosen for the batch width (the widest
// forward, normally the verify width K+1) and is kept for every T, so a token's sums (slice partials added in
// slice order) do not depend on T: a verify of T = K+1 and a one-token decode give a stream bit-identical
// logits.  Only the token tiling follows T.
BPlans& plans_for(sd_batch* b, int T) {
    BPlans& P = b->plans[T];
    if (P.ready) return P;
    const ModelView& m = b->m;
    const int M = b->B * T, Mw = b->B * b->W;
    auto plan = [&](WgPlan& out, int epi, int rows, int K, int kp_max) {
        WgPlan wide;
        wg_plan(wide, epi, rows, K, Mw, 1, kp_max, b->sms, b->max_smem);
        wg_plan(out, epi, rows, K, M, wide.a.kparts, wide.a.kparts, b->sms, b->max_smem);
    };
    plan(P.qkv, WG_STORE, m.qkv_rows, m.dim, b->kp_max);
    plan(P.wo, WG_STORE, m.dim, m.q_rows, b->kp_max);
    plan(P.w13, WG_SILU, 2 * m.hidden, m.dim, 1);
    plan(P.w2, WG_STORE, m.dim, m.hidden, b->kp_max);
    plan(P.lm, WG_STORE, m.vocab, m.dim, 1);
    P.tc = b->gemm_mode == SD_BATCH_GEMM_TC || (b->gemm_mode == SD_BATCH_GEMM_AUTO && M >= kTcMinTokens);
    if (P.tc) {
        tc_plan(P.qkv, WG_STORE, b->sms, b->max_smem);
        tc_plan(P.wo, WG_STORE, b->sms, b->max_smem);
        tc_plan(P.w13, WG_SILU, b->sms, b->max_smem);
        tc_plan(P.w2, WG_STORE, b->sms, b->max_smem);
        tc_plan(P.lm, WG_STORE, b->sms, b->max_smem);
    }
    P.ready = true;
    return P;
}

int run_wgemm(sd_batch* b, int epi, WgPlan p, const uint8_t* w, const uint8_t* act) {
    p.a.w = w;
    p.a.act = act;
    p.a.err = b->m.err;
    if (p.tc)
        CK(launch_tcgemm(epi, p.a, p.grid, p.smem, b->st), "tcgen05 gemm");
    else
        CK(launch_wgemm(epi, p.a, p.grid, p.smem, b->st), "wide gemm");
    return SD_OK;
}

// One forward of T tokens per stream (positions and token ids from the control blocks).
int enqueue_bforward(sd_batch* b, int T, bool logits) {
    const ModelView& m = b->m;
    const int M = b->B * T, NT = (M + 7) / 8;
    BPlans& P = plans_for(b, T);
    BNormArgs na{};
    na.x = b->x;
    na.y = b->y;
    na.ystride = (size_t)b->M_max * m.dim;
    na.embd = m.embd;
    const int tcimg = P.tc ? 1 : 0;
    na.out = WImg{b->img_x, NT, tcimg};
    na.dim = m.dim;
    na.T = T;
    na.eps = m.eps;
    na.ctrl = b->ctrl;
    na.w = m.rms_att[0];
    k_bnorm<0><<<M, kBNormThreads, 0, b->st>>>(na);
    CK(cudaGetLastError(), "embed");
    for (int l = 0; l < m.n_layers; ++l) {
        int rc;
        // QKV
        WgPlan pq = P.qkv;
        pq.a.out = b->qkv;
        pq.a.ld = m.qkv_rows;
        pq.a.out_rows = m.qkv_rows;
        pq.a.part_stride = (size_t)b->M_max * m.qkv_rows;
        if ((rc = run_wgemm(b, WG_STORE, pq, b->wqkv[l], b->img_x))) return rc;
        BRopeArgs ra{};
        ra.qkv = b->qkv;
        ra.pstride = pq.a.part_stride;
        ra.kparts = pq.a.kparts;
        ra.q = b->q;
        ra.k = b->kc + (size_t)l * b->kv_layer;
        ra.v = b->vc + (size_t)l * b->kv_layer;
        ra.kv_stream = b->kv_stream;
        ra.q_rows = m.q_rows;
        ra.kv_rows = m.kv_rows;
        ra.max_seq = b->max_seq;
        ra.head_dim = m.hd;
        ra.T = T;
        ra.theta_inv = m.theta_inv;
        ra.q_scale = 1.0f / sqrtf((float)m.hd);
        ra.ctrl = b->ctrl;
        k_brope_kv<<<M, 256, 0, b->st>>>(ra);
        CK(cudaGetLastError(), "rope");
        // attention
        BAttnArgs ba{};
        ba.a.q = b->q;
        ba.a.q_ld = m.q_rows;
        ba.a.k = ra.k;
        ba.a.v = ra.v;
        ba.a.kv_ld = m.kv_rows;
        ba.a.n_heads = m.n_heads;
        ba.a.n_kvh = m.n_kv;
        ba.a.S = T;
        ba.a.max_seq = b->max_seq;
        ba.a.chunk = b->chunk;
        ba.a.max_chunks = b->max_chunks;
        ba.a.part_ml = b->part_ml;
        ba.a.part_acc = b->part_acc;
        ba.a.wimg = WImg{b->img_attn, NT, tcimg};
        ba.kv_stream = b->kv_stream;
        ba.T = T;
        ba.ctrl = b->ctrl;
        ba.n_streams = b->B;
        k_battn_partial<<<std::min(2 * b->sms, b->B * b->max_chunks * m.n_kv), kAttnThreads, battn_smem_bytes(), b->st>>>(ba);
        CK(cudaGetLastError(), "attention");
        k_battn_combine<<<(M * m.n_heads + kBCombWarps - 1) / kBCombWarps, kBCombWarps * 32, 0, b->st>>>(ba);
        CK(cudaGetLastError(), "combine");
        // o-proj, residual + norm
        WgPlan po = P.wo;
        po.a.out = b->y;
        po.a.ld = m.dim;
        po.a.out_rows = m.dim;
        po.a.part_stride = (size_t)b->M_max * m.dim;
        if ((rc = run_wgemm(b, WG_STORE, po, b->wwo[l], b->img_attn))) return rc;
        na.w = m.rms_ffn[l];
        na.yparts = po.a.kparts;
        k_bnorm<1><<<M, kBNormThreads, 0, b->st>>>(na);
        CK(cudaGetLastError(), "norm");
        // gate|up + SiLU + Q8_0
        WgPlan pg = P.w13;
        pg.a.h = WImg{b->img_h, NT, tcimg};
        pg.a.hidden = m.hidden;
        if ((rc = run_wgemm(b, WG_SILU, pg, b->ww13[l], b->img_x))) return rc;
        // down, residual + next norm
        WgPlan pd = P.w2;
        pd.a.out = b->y;
        pd.a.ld = m.dim;
        pd.a.out_rows = m.dim;
        pd.a.part_stride = (size_t)b->M_max * m.dim;
        if ((rc = run_wgemm(b, WG_STORE, pd, b->ww2[l], b->img_h))) return rc;
        na.w = (l + 1 < m.n_layers) ? m.rms_att[l + 1] : m.rms_final;
        na.yparts = pd.a.kparts;
        k_bnorm<1><<<M, kBNormThreads, 0, b->st>>>(na);
        CK(cudaGetLastError(), "norm");
    }
    if (!logits) return SD_OK;
    WgPlan pl = P.lm;
    pl.a.out = b->logits;
    pl.a.ld = m.vocab;
    pl.a.out_rows = m.vocab;
    int rc = run_wgemm(b, WG_STORE, pl, b->wlm, b->img_x);
    if (rc) return rc;
    CK(launch_argmax(b->logits, m.vocab, M, b->argmax, nullptr, b->st, false), "argmax");
    return SD_OK;
}

int run_bforward(sd_batch* b, int T, bool logits) {
    cudaGraphExec_t& slot = b->fwd_graph[T][logits ? 1 : 0];
    if (!slot) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal), "capture");
        const int rc = enqueue_bforward(b, T, logits);
        const cudaError_t e = cudaStreamEndCapture(b->st, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        CK(e, "capture end");
        const cudaError_t ie = cudaGraphInstantiate(&slot, g, 0);
        cudaGraphDestroy(g);
        CK(ie, "graph instantiate");
    }
    CK(cudaGraphLaunch(slot, b->st), "graph launch");
    return SD_OK;
}

int check_host_tokens(sd_batch* b, const int32_t* t, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (t[i] < 0 || t[i] >= b->m.vocab) return fail(SD_ERR_INVALID, "token %d out of range [0, %d)", t[i], b->m.vocab);
    return SD_OK;
}

int ensure_tok(sd_batch* b, size_t n) {
    if (b->tok_cap >= n) return SD_OK;
    cudaFree(b->tok);
    b->tok = nullptr;
    b->tok_cap = 0;
    int rc = dalloc(&b->tok, n);
    if (!rc) b->tok_cap = n;
    return rc;
}

int ensure_gen(sd_batch* b, int cap) {
    if (b->g_cap >= cap) return SD_OK;
    cudaFree(b->g_out);
    cudaFree(b->g_hist);
    b->g_out = b->g_hist = nullptr;
    b->g_cap = 0;
    int rc = dalloc(&b->g_out, (size_t)b->B * cap);
    if (!rc) rc = dalloc(&b->g_hist, (size_t)b->B * cap);
    if (!rc) b->g_cap = cap;
    return rc;
}

int finish(sd_batch* b) {
    CK(cudaStreamSynchronize(b->st), "stream sync");
    return check_device_error(b->m.err, b->st);
}

// Prefill of positions [0, n) of every stream from the device tokens b->tok ([B][stride], columns [0, n));
// the last chunk's logits are computed when last_logits is set.
int prefill_dev(sd_batch* b, int n, int stride, bool last_logits) {
    for (int i = 0; i < n; i += b->W) {
        const int T = std::min(b->W, n - i);
        k_bset_ctrl<<<(b->B + 127) / 128, 128, 0, b->st>>>(b->ctrl, b->B, b->tok, stride, i, T, nullptr);
        CK(cudaGetLastError(), "ctrl");
        int rc = run_bforward(b, T, last_logits && i + T >= n);
        if (rc) return rc;
    }
    return SD_OK;
}

GenParamsDev gen_params_dev(sd_batch* b, const sd_gen_params* gp, int* K_out) {
    GenParamsDev p{};
    p.mode = gp->mode == SD_GEN_NGRAM ? SD_MODE_NGRAM : SD_MODE_GREEDY;
    p.temp = gp->temp;
    p.top_k = gp->top_k;
    p.top_p = gp->top_p;
    p.rep_penalty = gp->rep_penalty;
    p.rep_window = gp->rep_window;
    p.ignore_eos = gp->ignore_eos;
    p.eos_id = b->m.eos;
    const int K = gp->spec_k < 1 ? 1 : gp->spec_k;
    p.spec_k = K;
    p.ngram_n = gp->ngram_n < 1 ? 3 : gp->ngram_n;
    p.history_has_current = gp->history_has_current;
    p.bonus_mode = gp->bonus_mode == SD_BONUS_REFERENCE ? SD_BONUS_REF_UNIFORM : SD_BONUS_ARGMAX_FIXED;
    p.gen_limit = p.mode == SD_MODE_GREEDY ? gp->max_tokens : gp->max_tokens - 1;
    p.max_seq = b->max_seq;
    *K_out = K;
    return p;
}

int iteration_graph(sd_batch* b, const GenParamsDev& p, int T) {
    if (b->iter_graph && b->iter_T == T && memcmp(&b->iter_p, &p, sizeof(p)) == 0) return SD_OK;
    if (b->iter_graph) cudaGraphExecDestroy(b->iter_graph);
    b->iter_graph = nullptr;
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal), "capture");
    int rc = ck(launch_bgen_prepare(b->gs, b->ctrl, b->B, p, b->st), "prepare");
    if (!rc) rc = enqueue_bforward(b, T, true);
    if (!rc) rc = ck(launch_bgen_commit(b->gs, b->ctrl, b->B, b->logits, b->probs, b->argmax, p, b->m.vocab, T, 0, b->st), "commit");
    if (!rc) rc = ck(launch_bcount_done(b->gs, b->B, p.gen_limit, b->ndone, b->st), "count");
    const cudaError_t e = cudaStreamEndCapture(b->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    CK(e, "capture end");
    const cudaError_t ie = cudaGraphInstantiate(&b->iter_graph, g, 0);
    cudaGraphDestroy(g);
    CK(ie, "graph instantiate");
    b->iter_T = T;
    b->iter_p = p;
    return SD_OK;
}

// Decode loop over every stream from the generation states already on the device.
int decode_loop(sd_batch* b, const GenParamsDev& p, int K, int32_t* out, int out_cap, int32_t* n_out, sd_batch_stats* stats) {
    const int T = p.mode == SD_MODE_GREEDY ? 1 : K + 1;
    int rc = iteration_graph(b, p, T);
    if (rc) return rc;
    const double t0 = now_ms();
    long long iters = 0;
    CK(launch_bcount_done(b->gs, b->B, p.gen_limit, b->ndone, b->st), "count");
    CK(cudaMemcpyAsync(b->ndone_h, b->ndone, 2 * sizeof(int), cudaMemcpyDeviceToHost, b->st), "count");
    CK(cudaStreamSynchronize(b->st), "decode");
    while (b->ndone_h[0] < b->B) {
        // an iteration emits 1 .. T tokens per live stream: every stream is still live after
        // ceil(most remaining / T) more iterations, so launch that many before looking again
        const int batch = std::max(1, (b->ndone_h[1] + T - 1) / T);
        for (int i = 0; i < batch; ++i) CK(cudaGraphLaunch(b->iter_graph, b->st), "iteration");
        iters += batch;
        CK(cudaMemcpyAsync(b->ndone_h, b->ndone, 2 * sizeof(int), cudaMemcpyDeviceToHost, b->st), "count");
        CK(cudaStreamSynchronize(b->st), "decode");
        if (iters > 4LL * (p.gen_limit + 4) + 64) return fail(SD_ERR_TIMEOUT, "batched decode did not terminate");
    }
    const double t1 = now_ms();
    if ((rc = finish(b))) return rc;
    CK(cudaMemcpy(b->gs_h, b->gs, sizeof(GenState) * b->B, cudaMemcpyDeviceToHost), "state");
    sd_batch_stats s{};
    for (int i = 0; i < b->B; ++i) {
        const GenState& g = b->gs_h[i];
        const int n = std::min(g.n_out, std::min(out_cap, b->g_cap));
        if (n > 0) CK(cudaMemcpy(out + (size_t)i * out_cap, b->g_out + (size_t)i * b->g_cap, (size_t)n * 4, cudaMemcpyDeviceToHost), "download");
        n_out[i] = n;
        s.n_generated += g.n_out;
        s.total_draft += g.total_draft;
        s.total_accepted += g.total_accepted;
        s.total_iterations += g.total_iterations;
    }
    s.verify_forwards = iters;
    s.ms_decode = t1 - t0;
    if (stats) {
        const double pre = stats->ms_prefill;
        *stats = s;
        stats->ms_prefill = pre;
    }
    return SD_OK;
}

int check_gen(sd_batch* b, const sd_gen_params* gp, int n_hist) {
    if (gp->mode == SD_GEN_SELF_SPEC) return fail(SD_ERR_UNSUPPORTED, "batched streams: greedy or n-gram drafting");
    const int K = gp->spec_k < 1 ? 1 : gp->spec_k;
    const int T = gp->mode == SD_GEN_GREEDY ? 1 : K + 1;
    if (T > b->W) return fail(SD_ERR_UNSUPPORTED, "verify width %d above the batch width %d", T, b->W);
    const int vw = std::max(kMaxS, T);
    if (n_hist + gp->max_tokens + vw + 1 > b->max_seq) return fail(SD_ERR_INVALID, "history + tokens exceed the KV ring");
    return SD_OK;
}

}  // namespace

extern "C" {

void sd_batch_free(sd_batch* b) {
    if (!b) return;
    cudaSetDevice(b->dev);
    if (b->st) cudaStreamSynchronize(b->st);
    for (auto& row : b->fwd_graph)
        for (auto& g : row)
            if (g) cudaGraphExecDestroy(g);
    if (b->iter_graph) cudaGraphExecDestroy(b->iter_graph);
    for (auto* v : {&b->wqkv, &b->wwo, &b->ww13, &b->ww2})
        for (uint8_t* p : *v) cudaFree(p);
    cudaFree(b->wlm);
    if (!b->shared_ring) {
        cudaFree(b->kc);
        cudaFree(b->vc);
    }
    cudaFree(b->x); cudaFree(b->y); cudaFree(b->qkv); cudaFree(b->q);
    cudaFree(b->img_x); cudaFree(b->img_attn); cudaFree(b->img_h); cudaFree(b->part_ml); cudaFree(b->part_acc);
    cudaFree(b->logits); cudaFree(b->argmax); cudaFree(b->probs); cudaFree(b->ctrl); cudaFree(b->tok);
    cudaFree(b->pos_dev); cudaFree(b->gs); cudaFree(b->g_out); cudaFree(b->g_hist); cudaFree(b->ndone);
    if (b->gs_h) cudaFreeHost(b->gs_h);
    if (b->ndone_h) cudaFreeHost(b->ndone_h);
    if (b->st && !b->shared_ring) cudaStreamDestroy(b->st);
    delete b;
}

void* sd_batch_stream(sd_batch* b) { return b ? (void*)b->st : nullptr; }

int sd_batch_set_gemm(sd_batch* b, int mode) {
    if (!b || mode < SD_BATCH_GEMM_AUTO || mode > SD_BATCH_GEMM_TC) return fail(SD_ERR_INVALID, "bad batch or gemm mode");
    clear_error();
    if (mode == b->gemm_mode) return SD_OK;
    cudaSetDevice(b->dev);
    CK(cudaStreamSynchronize(b->st), "sync");
    b->gemm_mode = mode;
    for (auto& P : b->plans) P.ready = false;
    for (auto& row : b->fwd_graph)
        for (auto& gr : row)
            if (gr) {
                cudaGraphExecDestroy(gr);
                gr = nullptr;
            }
    if (b->iter_graph) cudaGraphExecDestroy(b->iter_graph);
    b->iter_graph = nullptr;
    return SD_OK;
}

}  // extern "C"

namespace {

// The context's K/V ring and stream, for a batch whose streams are slices of one prompt.
struct SharedRing {
    __half *kc, *vc;
    cudaStream_t st;
};

int batch_create(sd_ctx* ctx, int n_streams, int max_seq, int max_width, const SharedRing* shared, sd_batch** out) {
    *out = nullptr;
    sd_batch* b = new sd_batch();
    int rc = sd_ctx_model_view(ctx, &b->m);
    auto bail = [&](int code) { sd_batch_free(b); return code; };
    if (rc) return bail(rc);
    const ModelView& m = b->m;
    if (m.tp_size != 1) return bail(fail(SD_ERR_UNSUPPORTED, "batched streams run on single-GPU contexts"));
    if (m.lm_type != 2 || m.embd_type != 2)
        return bail(fail(SD_ERR_UNSUPPORTED, "batched streams need a Q4_0 embedding and LM head (this model has "
                                             "K-quant ones; sd_forward / sd_generate serve it)"));
    if (m.dim > 4096 || m.dim % 1024) return bail(fail(SD_ERR_UNSUPPORTED, "dim %d", m.dim));
    b->ctx = ctx;
    b->dev = m.dev;
    b->B = n_streams;
    b->W = max_width;
    b->max_seq = max_seq;
    b->M_max = n_streams * max_width;
    b->sms = device_sm_count(b->dev);
    b->max_smem = device_max_smem(b->dev) - 1024;  // room for the GEMM's static shared memory
    b->max_chunks = (max_seq + b->chunk - 1) / b->chunk;
    if (cudaSetDevice(b->dev) != cudaSuccess) return bail(fail(SD_ERR_INVALID, "bad device %d", b->dev));
    if (shared) {
        b->shared_ring = true;
        b->st = shared->st;
        b->kc = shared->kc;
        b->vc = shared->vc;
    } else if ((rc = ck(cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking), "stream"))) {
        return bail(rc);
    }
    if ((rc = ck(wgemm_init_attrs(b->max_smem), "gemm attributes"))) return bail(rc);
    if ((rc = ck(tcgemm_init_attrs(b->max_smem), "tcgen05 gemm attributes"))) return bail(rc);
    if ((rc = ck(cudaFuncSetAttribute(k_battn_partial, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)battn_smem_bytes()),
                 "attention attributes")))
        return bail(rc);
    // a shared ring is the context's [layer][max_seq][kv_rows]: every stream of the batch addresses the same rows
    b->kv_stream = shared ? 0 : (size_t)max_seq * m.kv_rows;
    b->kv_layer = shared ? (size_t)max_seq * m.kv_rows : (size_t)n_streams * b->kv_stream;
    const size_t M = b->M_max;
    const size_t parts = (size_t)M * m.n_heads * b->max_chunks;
    if ((!shared && ((rc = dalloc(&b->kc, (size_t)m.n_layers * b->kv_layer)) ||
                     (rc = dalloc(&b->vc, (size_t)m.n_layers * b->kv_layer)))) ||
        (rc = dalloc(&b->x, M * m.dim)) || (rc = dalloc(&b->y, (size_t)b->kp_max * M * m.dim)) ||
        (rc = dalloc(&b->qkv, (size_t)b->kp_max * M * m.qkv_rows)) || (rc = dalloc(&b->q, M * m.q_rows)) ||
        (rc = dalloc(&b->img_x, wimg_bytes((int)M, m.dim))) || (rc = dalloc(&b->img_attn, wimg_bytes((int)M, m.q_rows))) ||
        (rc = dalloc(&b->img_h, wimg_bytes((int)M, m.hidden))) || (rc = dalloc(&b->part_ml, parts)) ||
        (rc = dalloc(&b->part_acc, parts * kHD)) || (rc = dalloc(&b->logits, M * m.vocab)) ||
        (rc = dalloc(&b->argmax, M)) || (rc = dalloc(&b->probs, (size_t)n_streams * m.vocab)) ||
        (rc = dalloc(&b->ctrl, (size_t)n_streams)) || (rc = dalloc(&b->pos_dev, (size_t)n_streams)) ||
        (rc = dalloc(&b->gs, (size_t)n_streams)) || (rc = dalloc(&b->ndone, 2)))
        return bail(rc);
    // weights in the wide GEMM layout (the context keeps its tile16x4 copies for the single-stream path)
    auto wide = [&](const uint8_t* tiles, int rows, int cols, uint8_t** out_w) {
        int r = dalloc(out_w, wide_bytes(rows, cols));
        if (!r) r = ck(launch_wide_repack(tiles, qmat_row_groups(rows), cols / 128, *out_w, b->st), "wide repack");
        return r;
    };
    b->wqkv.assign(m.n_layers, nullptr);
    b->wwo.assign(m.n_layers, nullptr);
    b->ww13.assign(m.n_layers, nullptr);
    b->ww2.assign(m.n_layers, nullptr);
    for (int l = 0; l < m.n_layers; ++l)
        if ((rc = wide(m.qkv[l], m.qkv_rows, m.dim, &b->wqkv[l])) || (rc = wide(m.wo[l], m.dim, m.q_rows, &b->wwo[l])) ||
            (rc = wide(m.w13[l], 2 * m.hidden, m.dim, &b->ww13[l])) || (rc = wide(m.w2[l], m.dim, m.hidden, &b->ww2[l])))
            return bail(rc);
    if ((rc = wide(m.lm, m.vocab, m.dim, &b->wlm))) return bail(rc);
    if ((rc = ck(cudaMallocHost((void**)&b->gs_h, sizeof(GenState) * n_streams), "pinned state"))) return bail(rc);
    if ((rc = ck(cudaMallocHost((void**)&b->ndone_h, 2 * sizeof(int)), "pinned counter"))) return bail(rc);
    // images start zeroed: tokens past a forward's count read zeros, never uninitialised bytes
    cudaMemsetAsync(b->img_x, 0, wimg_bytes((int)M, m.dim), b->st);
    cudaMemsetAsync(b->img_attn, 0, wimg_bytes((int)M, m.q_rows), b->st);
    cudaMemsetAsync(b->img_h, 0, wimg_bytes((int)M, m.hidden), b->st);
    cudaMemsetAsync(b->x, 0, M * m.dim * sizeof(float), b->st);
    cudaMemsetAsync(b->ctrl, 0, sizeof(DevCtrl) * n_streams, b->st);
    // rings start as fp16 zeros (positions never written read as zeros, never as stale bytes)
    if (!shared) {
        cudaMemsetAsync(b->kc, 0, (size_t)m.n_layers * b->kv_layer * sizeof(__half), b->st);
        cudaMemsetAsync(b->vc, 0, (size_t)m.n_layers * b->kv_layer * sizeof(__half), b->st);
    }
    cudaMemsetAsync(b->gs, 0, sizeof(GenState) * n_streams, b->st);
    if ((rc = finish(b))) return bail(rc);
    *out = b;
    return SD_OK;
}

}  // namespace

extern "C" {

int sd_batch_create(sd_ctx* ctx, int n_streams, int max_seq, int max_width, sd_batch** out) {
    clear_error();
    if (!ctx || !out || n_streams < 1 || max_seq < 16 || max_width < 1 || max_width > SD_BATCH_MAX_WIDTH)
        return fail(SD_ERR_INVALID, "sd_batch_create: bad arguments");
    return batch_create(ctx, n_streams, max_seq, max_width, nullptr, out);
}

}  // extern "C"

namespace sd {

int batch_create_prefill(sd_ctx* ctx, int n_slices, int width, void* kc, void* vc, int max_seq, cudaStream_t st,
                         sd_batch** out) {
    const SharedRing sr{reinterpret_cast<__half*>(kc), reinterpret_cast<__half*>(vc), st};
    return batch_create(ctx, n_slices, max_seq, width, &sr, out);
}

// Chunks of n_slices x width prompt tokens; slice v of a chunk starting at prompt index i takes tokens
// [i + width v, i + width v + width) at position start_pos + i + width v (a short last slice has fewer valid
// tokens, slices past the prompt are marked done).  The RoPE kernel writes every valid token's K/V into the
// context's ring before the attention kernel reads it, so each slice attends to the whole prefix before it.
int batch_prefill_ring(sd_batch* b, const int32_t* tokens, int n, int start_pos) {
    const int W = b->W, chunk = b->B * W;
    std::vector<DevCtrl> hc(b->B);
    for (int i = 0; i < n; i += chunk) {
        for (int v = 0; v < b->B; ++v) {
            DevCtrl& c = hc[v];
            memset(&c, 0, sizeof(c));
            const int first = i + v * W, nv = std::max(0, std::min(W, n - first));
            c.pos = start_pos + first;
            c.n_valid = nv;
            c.done = nv == 0;
            for (int j = 0; j < nv; ++j) c.tokens[j] = tokens[first + j];
        }
        // from pageable memory: the call returns once the host array has been read
        CK(cudaMemcpyAsync(b->ctrl, hc.data(), sizeof(DevCtrl) * b->B, cudaMemcpyHostToDevice, b->st), "prefill ctrl");
        int rc = run_bforward(b, W, false);
        if (rc) return rc;
    }
    return SD_OK;
}

}  // namespace sd

extern "C" {

int sd_batch_forward(sd_batch* b, const int32_t* tokens, int T, const int32_t* pos, float* logits) {
    clear_error();
    if (!b || !tokens || !pos || T < 1 || T > b->W) return fail(SD_ERR_INVALID, "sd_batch_forward: bad arguments");
    int rc = check_host_tokens(b, tokens, (size_t)b->B * T);
    if (rc) return rc;
    for (int i = 0; i < b->B; ++i)
        if (pos[i] < 0 || pos[i] + T > b->max_seq) return fail(SD_ERR_INVALID, "stream %d: positions past the ring", i);
    cudaSetDevice(b->dev);
    if ((rc = ensure_tok(b, (size_t)b->B * T))) return rc;
    CK(cudaMemcpyAsync(b->tok, tokens, (size_t)b->B * T * 4, cudaMemcpyHostToDevice, b->st), "tokens");
    CK(cudaMemcpyAsync(b->pos_dev, pos, (size_t)b->B * 4, cudaMemcpyHostToDevice, b->st), "positions");
    k_bset_ctrl<<<(b->B + 127) / 128, 128, 0, b->st>>>(b->ctrl, b->B, b->tok, T, 0, T, b->pos_dev);
    CK(cudaGetLastError(), "ctrl");
    if ((rc = run_bforward(b, T, logits != nullptr))) return rc;
    if (logits)
        CK(cudaMemcpyAsync(logits, b->logits, (size_t)b->B * T * b->m.vocab * 4, cudaMemcpyDeviceToHost, b->st), "logits");
    return finish(b);
}

int sd_batch_prefill(sd_batch* b, const int32_t* tokens, int n) {
    clear_error();
    if (!b || !tokens || n < 1 || n > b->max_seq) return fail(SD_ERR_INVALID, "sd_batch_prefill: bad arguments");
    int rc = check_host_tokens(b, tokens, (size_t)b->B * n);
    if (rc) return rc;
    cudaSetDevice(b->dev);
    if ((rc = ensure_tok(b, (size_t)b->B * n))) return rc;
    CK(cudaMemcpyAsync(b->tok, tokens, (size_t)b->B * n * 4, cudaMemcpyHostToDevice, b->st), "tokens");
    if ((rc = prefill_dev(b, n, n, false))) return rc;
    return finish(b);
}

int sd_batch_decode(sd_batch* b, const sd_gen_params* gp, const int32_t* history, int n_hist, const int32_t* first,
                    int32_t* out, int out_cap, int32_t* n_out, sd_batch_stats* stats) {
    clear_error();
    if (!b || !gp || !history || n_hist < 1 || !first || !out || out_cap < 1 || !n_out)
        return fail(SD_ERR_INVALID, "sd_batch_decode: bad arguments");
    int rc = check_gen(b, gp, n_hist);
    if (rc) return rc;
    if ((rc = check_host_tokens(b, history, (size_t)b->B * n_hist)) || (rc = check_host_tokens(b, first, (size_t)b->B)))
        return rc;
    cudaSetDevice(b->dev);
    const int cap = n_hist + gp->max_tokens + 2 * kMaxVerify + 16;
    if ((rc = ensure_gen(b, cap)) || (rc = ensure_tok(b, (size_t)b->B * n_hist + b->B))) return rc;
    int K = 1;
    const GenParamsDev p = gen_params_dev(b, gp, &K);
    CK(cudaMemcpyAsync(b->tok, history, (size_t)b->B * n_hist * 4, cudaMemcpyHostToDevice, b->st), "history");
    int* cur = b->tok + (size_t)b->B * n_hist;
    CK(cudaMemcpyAsync(cur, first, (size_t)b->B * 4, cudaMemcpyHostToDevice, b->st), "first");
    GenState t{};
    t.pos = n_hist;  // the fix-up below moves it to n_hist - 1, where the first token (history's last) sits
    t.out_cap = cap;
    t.hist_cap = cap;
    t.hlen = n_hist;
    t.rng_counter = 1ull << 20;
    k_binit_gen<<<b->B, 256, 0, b->st>>>(b->gs, b->B, t, b->g_out, b->g_hist, cap, b->tok, n_hist, n_hist, cur, gp->seed);
    CK(cudaGetLastError(), "state");
    // the first token counts as generated but is not in the output (sd_decode semantics)
    CK(launch_bgen_first_fixup(b->gs, b->B, p.gen_limit, p.ignore_eos, p.eos_id, b->st), "state");
    if (stats) stats->ms_prefill = 0.0;
    return decode_loop(b, p, K, out, out_cap, n_out, stats);
}

int sd_batch_generate(sd_batch* b, const sd_gen_params* gp, const int32_t* prompts, int n_prompt, int32_t* out,
                      int out_cap, int32_t* n_out, sd_batch_stats* stats) {
    clear_error();
    if (!b || !gp || !prompts || n_prompt < 1 || !out || out_cap < 1 || !n_out)
        return fail(SD_ERR_INVALID, "sd_batch_generate: bad arguments");
    int rc = check_gen(b, gp, n_prompt);
    if (rc) return rc;
    if ((rc = check_host_tokens(b, prompts, (size_t)b->B * n_prompt))) return rc;
    cudaSetDevice(b->dev);
    const double t0 = now_ms();
    const int cap = n_prompt + gp->max_tokens + 2 * kMaxVerify + 16;
    if ((rc = ensure_gen(b, cap)) || (rc = ensure_tok(b, (size_t)b->B * n_prompt))) return rc;
    CK(cudaMemcpyAsync(b->tok, prompts, (size_t)b->B * n_prompt * 4, cudaMemcpyHostToDevice, b->st), "prompts");
    if ((rc = prefill_dev(b, n_prompt, n_prompt, true))) return rc;
    const int Tl = n_prompt - (n_prompt - 1) / b->W * b->W;  // tokens in the last chunk
    // first token: sample_token with the repetition penalty over the prompt window, from each stream's last
    // prompt row (mistral/mistral_infer.m:610-621)
    GenParamsDev p1{};
    p1.mode = SD_MODE_GREEDY;
    p1.temp = gp->temp;
    p1.top_k = gp->top_k;
    p1.top_p = gp->top_p;
    p1.rep_penalty = gp->rep_penalty;
    p1.rep_window = gp->rep_window;
    p1.ignore_eos = 1;
    p1.eos_id = b->m.eos;
    p1.gen_limit = 1;
    p1.max_seq = b->max_seq;
    GenState t{};
    t.pos = n_prompt;
    t.out_cap = cap;
    t.hist_cap = cap;
    t.hlen = n_prompt;
    k_binit_gen<<<b->B, 256, 0, b->st>>>(b->gs, b->B, t, b->g_out, b->g_hist, cap, b->tok, n_prompt, n_prompt, nullptr,
                                         gp->seed);
    CK(cudaGetLastError(), "state");
    CK(launch_bgen_commit(b->gs, b->ctrl, b->B, b->logits, b->probs, b->argmax, p1, b->m.vocab, Tl, Tl - 1, b->st), "first token");
    int K = 1;
    const GenParamsDev p = gen_params_dev(b, gp, &K);
    CK(launch_bgen_first_fixup(b->gs, b->B, p.gen_limit, p.ignore_eos, p.eos_id, b->st), "state");
    if ((rc = finish(b))) return rc;
    sd_batch_stats s{};
    s.ms_prefill = now_ms() - t0;
    rc = decode_loop(b, p, K, out, out_cap, n_out, &s);
    if (rc) return rc;
    if (stats) *stats = s;
    return SD_OK;
}

}  // extern "C"
