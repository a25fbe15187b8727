// sd_quant.cu -- Q8_0 activation quantizer, residual add + RMSNorm + quantise, token embedding.
//
// Quantizer: mistral/dequant.h:545-599 (bit-exact: IEEE d = amax/127, id = 1/d, RNE, saturate).
// RMSNorm:   mistral/mistral_model.h:202-208 (s = 1/sqrt(sum(x^2)/dim + eps); out = (x*s)*w).
// Embedding: Q4_0 row dequant d*((q&15)-8), mistral/mistral_model.h:134-145 (exact).
// Outputs are Q8 planes: codes [S][n], fp32 scales [S][n/32] and per-block code sums [S][n/32]
// (the sum feeds the -8*sum accumulator init of the u8 x s8 MMA in the matvec).
#include "sd_dev.cuh"

namespace sd {

// One warp per 32-value block; grid-stride over S * n/32 blocks.
__global__ void k_quantize(const float* __restrict__ x, Q8Planes out, int S, int n) {
    const int nb = n >> 5;
    const int lane = threadIdx.x & 31;
    const long long wid = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long blk = wid; blk < (long long)S * nb; blk += nw) {
        const float v = x[blk * 32 + lane];
        float d;
        int sum;
        const int q = q8_quant_lane(v, &d, &sum);
        out.qs[blk * 32 + lane] = (int8_t)q;
        if (lane == 0) {
            out.d[blk] = d;
            out.sum[blk] = sum;
        }
    }
}

cudaError_t launch_quantize(const float* x, Q8Planes out, int S, int n, cudaStream_t st) {
    long long blocks = (long long)S * (n / 32);
    int grid = (int)((blocks * 32 + 255) / 256);
    if (grid > 4096) grid = 4096;
    k_quantize<<<grid, 256, 0, st>>>(x, out, S, n);
    return cudaGetLastError();
}

// Planes <-> reference AoS block_q8_0 (fp32 d + 32 int8, 36 bytes).
__global__ void k_q8_to_blocks(Q8Planes in, uint8_t* blocks, long long nblk) {
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblk; b += (long long)gridDim.x * blockDim.x) {
        uint8_t* o = blocks + b * 36;
        float d = in.d[b];
        memcpy(o, &d, 4);
        for (int j = 0; j < 32; ++j) o[4 + j] = (uint8_t)in.qs[b * 32 + j];
    }
}

__global__ void k_blocks_to_q8(const uint8_t* blocks, Q8Planes out, long long nblk) {
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblk; b += (long long)gridDim.x * blockDim.x) {
        const uint8_t* o = blocks + b * 36;
        float d;
        memcpy(&d, o, 4);
        int s = 0;
        for (int j = 0; j < 32; ++j) {
            const int8_t q = (int8_t)o[4 + j];
            out.qs[b * 32 + j] = q;
            s += q;
        }
        out.d[b] = d;
        out.sum[b] = s;
    }
}

cudaError_t launch_q8_to_blocks(Q8Planes in, void* blocks, int S, int n, cudaStream_t st) {
    long long nblk = (long long)S * (n / 32);
    int grid = (int)((nblk + 255) / 256);
    k_q8_to_blocks<<<grid > 4096 ? 4096 : grid, 256, 0, st>>>(in, (uint8_t*)blocks, nblk);
    return cudaGetLastError();
}

cudaError_t launch_blocks_to_q8(const void* blocks, Q8Planes out, int S, int n, cudaStream_t st) {
    long long nblk = (long long)S * (n / 32);
    int grid = (int)((nblk + 255) / 256);
    k_blocks_to_q8<<<grid > 4096 ? 4096 : grid, 256, 0, st>>>((const uint8_t*)blocks, out, nblk);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Residual add / embed + RMSNorm + Q8_0 quantisation, one CTA (1024 threads) per token.
// Warp w owns Q8_0 blocks w, w+32, ... (up to kNormMaxBPW of them); lane j owns element j of each
// block.  Every global load of a thread is issued before any is consumed (x, all K-split partials of
// y, the norm weight), so a token costs about one memory round trip.  The sum of squares is
// accumulated in a fixed order per lane, reduced by a butterfly within the warp and then across the
// 32 warps in order -- identical for every S (batch invariant).
// ---------------------------------------------------------------------------------------------
constexpr int kNormThreads = 1024;
constexpr int kNormWarps = kNormThreads / 32;
constexpr int kNormMaxBPW = 4;          // dim <= 32 * 32 * 4 = 4096
constexpr int kNormMaxParts = 8;

template <int MODE>
__global__ void __launch_bounds__(kNormThreads) k_norm_quant(const NormArgs a) {
    __shared__ __align__(16) float vs[kNormWarps * 32 * kNormMaxBPW];
    __shared__ float gss[kNormMaxBPW * kNormWarps * 32 / 16];
    __shared__ float scale;
    const int tok = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (a.ctrl && a.ctrl->done) return;
    pdl_trigger();
    pdl_wait();
    const int nv = a.ctrl ? min(a.ctrl->n_valid, a.S) : a.S;
    if (tok >= nv) return;
    const int nb = a.dim >> 5;
    const int bpw = nb / kNormWarps;      // blocks per warp (dim % 1024 == 0)
    float* x = a.x + (size_t)tok * a.dim;

    float v[kNormMaxBPW];
    float wv[kNormMaxBPW];
#pragma unroll
    for (int k = 0; k < kNormMaxBPW; ++k) {
        v[k] = 0.f;
        wv[k] = 0.f;
        if (k < bpw) {
            const int e = (warp + kNormWarps * k) * 32 + lane;
            wv[k] = a.w[e];
            if constexpr (MODE == 0) {
                const int token = a.tokens ? a.tokens[tok] : a.ctrl->tokens[tok];
                v[k] = embed_value(a.embd, a.embd_type, token, a.dim, warp + kNormWarps * k, lane);
            } else {
                v[k] = x[e];
            }
        }
    }
    if constexpr (MODE == 1) {
        float yv[kNormMaxBPW];
#pragma unroll
        for (int k = 0; k < kNormMaxBPW; ++k) yv[k] = 0.f;
        if (a.tp.n > 1) {
            // tensor parallel: every rank's partial outputs of this reduction, in rank order then slice
            // order, read from the ranks' own memory once their flags show this sequence number
            const unsigned long long seq = *a.tp.base + a.tp.idx + 1;
            if (tok == 0 && threadIdx.x < a.tp.n) {
                // this rank's slice is complete (previous kernel, stream order): publish it to every rank
                __threadfence_system();
                asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.tp.flags[threadIdx.x] + a.tp.rank), "l"(seq)
                             : "memory");
            }
            if (threadIdx.x == 0) {
                bool ok = true;
                const uint64_t t0 = global_ns();
                for (int r = 0; r < a.tp.n && ok; ++r) {
                    const unsigned long long* f = a.tp.flags[a.tp.rank] + r;
                    unsigned long long v;
                    while (true) {
                        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
                        if (v >= seq) break;
                        if (global_ns() - t0 > kWaitLimitNs) {
                            set_dev_error(a.err, DEV_ERR_PEER_WAIT);
                            ok = false;
                            break;
                        }
                    }
                }
            }
            __syncthreads();
            const size_t boff = (size_t)(seq & 1) * a.tp.buf;
            for (int r = 0; r < a.tp.n; ++r) {
#pragma unroll
                for (int p = 0; p < kNormMaxParts; ++p) {
                    if (p < a.yparts) {
#pragma unroll
                        for (int k = 0; k < kNormMaxBPW; ++k)
                            if (k < bpw)
                                yv[k] += __ldcg(a.tp.y[r] + boff + (size_t)p * a.ystride + (size_t)tok * a.dim +
                                                (warp + kNormWarps * k) * 32 + lane);
                    }
                }
            }
        } else {
            // partial slices summed in slice order (K-split matvec outputs)
#pragma unroll
            for (int p = 0; p < kNormMaxParts; ++p) {
                if (p < a.yparts) {
#pragma unroll
                    for (int k = 0; k < kNormMaxBPW; ++k)
                        if (k < bpw) yv[k] += a.y[(size_t)p * a.ystride + (size_t)tok * a.dim + (warp + kNormWarps * k) * 32 + lane];
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kNormMaxBPW; ++k) v[k] = v[k] + yv[k];
    }
#pragma unroll
    for (int k = 0; k < kNormMaxBPW; ++k)
        if (k < bpw) {
            const int e = (warp + kNormWarps * k) * 32 + lane;
            vs[e] = v[k];
            if constexpr (MODE != 2) x[e] = v[k];
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
    for (int k = 0; k < kNormMaxBPW; ++k) {
        if (k >= bpw) continue;
        const int b = warp + kNormWarps * k;
        // Q8_0 of the normalised row (x*s)*w, taken as Q8_0 of u = x*w with the block scale times s:
        // s > 0 is common to the block, so the codes do not depend on it and whichever kernel produces x
        // can quantise u before s is known (the persistent forward does; this kernel matches it).
        const float u = v[k] * wv[k];
        if (a.xn_out) a.xn_out[(size_t)tok * a.dim + b * 32 + lane] = u * s;
        float du;
        int sum;
        const int q = q8_quant_lane(u, &du, &sum);
        a.out.qs[(size_t)tok * a.dim + b * 32 + lane] = (int8_t)q;
        if (lane == 0) {
            a.out.d[(size_t)tok * nb + b] = du * s;
            a.out.sum[(size_t)tok * nb + b] = sum;
        }
    }
}

__global__ void k_tp_advance(unsigned long long* base, int n) { *base += (unsigned long long)n; }

cudaError_t launch_tp_advance(unsigned long long* base, int n, cudaStream_t st) {
    k_tp_advance<<<1, 1, 0, st>>>(base, n);
    return cudaGetLastError();
}

cudaError_t launch_norm_quant(int mode, const NormArgs& a, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.S);
    cfg.blockDim = dim3(kNormThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (mode) {
        case 0: return cudaLaunchKernelEx(&cfg, k_norm_quant<0>, a);
        case 1: return cudaLaunchKernelEx(&cfg, k_norm_quant<1>, a);
        default: return cudaLaunchKernelEx(&cfg, k_norm_quant<2>, a);
    }
}

}  // namespace sd
