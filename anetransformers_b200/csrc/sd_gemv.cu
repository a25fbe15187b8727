// sd_gemv.cu -- W4A8 Q4_0 x Q8_0 matvec for S <= 8 tokens on sm_100a.
//
// Replaces the reference's row-parallel SDOT matvec (mistral/dequant.h:1022-1137) and its fused
// QKV / gate-up variants (mistral/mistral_model.h:676-814) for the S=1 decode step and the S=K+1
// batched verify (mistral/mistral_infer.m:103-179).
//
// Per row r, token s:  y[s][r] = sum_b (wd[r,b] * xd[s,b]) * isum[r,s,b]
//   isum = sum_j (q_j - 8) * x8_j  -- exact int32, the same value SDOT produces.
// isum comes from the int8 tensor core (mma.m16n8k32, u8 nibbles x s8 codes) with the accumulator
// initialised to -8 * sum_j x8_j, so the MMA result IS the block sum; the fp32 scale is applied per
// block exactly as the reference does.  Weights stream HBM -> shared memory through a ring of
// 9216-byte stages filled by 1-D bulk copies (TMA engine) issued by a producer warp; 8 consumer warps
// each take one 1152-byte tile (16 rows x 4 blocks) per stage.  The weight stream does not depend
// on the previous kernel, so the producer starts before griddepcontrol.wait (PDL overlap).
//
// Determinism / batch invariance: every (row, token) value is accumulated in a fixed order (per warp
// over its tiles, then warps 0..7), independent of S and of the other tokens, so a token's result in
// an S=5 verify is bit-identical to its S=1 decode result.
#include "sd_common.cuh"

namespace sd {

namespace {

struct SmemLayout {
    size_t ring, act_b, act_c, act_x, red, ubuf, bars, total;
};

__host__ __device__ inline SmemLayout smem_layout(int K, int nstage) {
    SmemLayout L;
    size_t nb = (size_t)K / 32;
    L.ring = 0;
    L.act_b = L.ring + (size_t)nstage * kStageBytes;
    L.act_c = L.act_b + nb * 64 * 4;
    L.act_x = L.act_c + nb * 4 * 8;
    L.red = L.act_x + nb * 4 * 8;
    L.ubuf = L.red + 2 * kConsumerWarps * 128 * 4;
    L.bars = L.ubuf + 4 * 128 * 4;
    L.total = L.bars + 2 * kMaxStages * 8;
    return L;
}

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float h2f_lane(uint2 v, int blk) {
    uint32_t w = blk < 2 ? v.x : v.y;
    uint16_t h = (blk & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFF);
    return __half2float(__ushort_as_half(h));
}

}  // namespace

template <int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemLayout L = smem_layout(a.K, a.nstage);
    uint8_t* ring = smem + L.ring;
    uint32_t* act_b = reinterpret_cast<uint32_t*>(smem + L.act_b);
    int2* act_c = reinterpret_cast<int2*>(smem + L.act_c);
    float2* act_x = reinterpret_cast<float2*>(smem + L.act_x);
    float* red = reinterpret_cast<float*>(smem + L.red);
    float* ubuf = reinterpret_cast<float*>(smem + L.ubuf);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + kMaxStages;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nstage = a.nstage;
    const int nb = a.K >> 5;

    if (a.ctrl && a.ctrl->done) return;  // uniform across the grid

    // CTA's contiguous range of units (a unit is rg_per_unit row-groups).
    const int G = gridDim.x, c = blockIdx.x;
    const int u0 = (int)((long long)c * a.n_units / G), u1 = (int)((long long)(c + 1) * a.n_units / G);
    const int rg0 = u0 * a.rg_per_unit, rg1 = u1 * a.rg_per_unit;
    const int cpr = a.nq / kChunkQuads;  // ring stages per row-group
    const int n_stages_total = (rg1 - rg0) * cpr;
    const uint8_t* wbase = a.w + (size_t)rg0 * a.nq * kTileBytes;

    if (tid == 0) {
        for (int i = 0; i < nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kConsumerWarps) {
        // ---------------- producer: stream this CTA's weight range through the ring ----------------
        if (lane == 0) {
            for (int s = 0; s < n_stages_total; ++s) {
                const int slot = s % nstage;
                if (s >= nstage && !mbar_wait(&empty[slot], ((s / nstage) - 1) & 1)) {
                    set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
                    break;  // consumers time out on the stages never issued
                }
                mbar_arrive_expect_tx(&full[slot], kStageBytes);
                bulk_g2s(ring + (size_t)slot * kStageBytes, wbase + (size_t)s * kStageBytes, kStageBytes,
                         &full[slot]);
            }
        }
        return;
    }

    // ---------------- consumers: stage activations (depends on the previous kernel) ----------------
    pdl_wait();
    const int S = a.S;
    int nv = S;
    int pos = 0;
    if (a.ctrl) {
        nv = min(a.ctrl->n_valid, S);
        pos = a.ctrl->pos;
    }
    {
        // codes: global [s][K] -> act_b[(b*8 + j)*8 + s] (word j of block b of token s)
        const int words_per_tok = a.K >> 2;
        const int n16 = kMaxS * (words_per_tok >> 2);  // 16-byte pieces over 8 token slots
        for (int i = tid; i < n16; i += kConsumerWarps * 32) {
            const int s = i / (words_per_tok >> 2);
            const int w4 = (i - s * (words_per_tok >> 2)) * 4;  // first word index within the token
            uint4 v = make_uint4(0, 0, 0, 0);
            if (s < nv) v = *reinterpret_cast<const uint4*>(a.act.qs + (size_t)s * a.K + (size_t)w4 * 4);
            const int b = w4 >> 3, j = w4 & 7;
            act_b[(b * 8 + j + 0) * 8 + s] = v.x;
            act_b[(b * 8 + j + 1) * 8 + s] = v.y;
            act_b[(b * 8 + j + 2) * 8 + s] = v.z;
            act_b[(b * 8 + j + 3) * 8 + s] = v.w;
        }
        for (int i = tid; i < nb * kMaxS; i += kConsumerWarps * 32) {
            const int s = i / nb, b = i - s * nb;
            int cs = 0;
            float xd = 0.f;
            if (s < nv) {
                cs = -8 * a.act.sum[(size_t)s * nb + b];
                xd = a.act.d[(size_t)s * nb + b];
            }
            int* cp = reinterpret_cast<int*>(&act_c[b * 4 + (s >> 1)]);
            float* xp = reinterpret_cast<float*>(&act_x[b * 4 + (s >> 1)]);
            cp[s & 1] = cs;
            xp[s & 1] = xd;
        }
    }
    named_sync(1, kConsumerWarps * 32);

    // ---------------- main loop ----------------
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    int sidx = 0;
    // A stage that never arrives (only possible if the producer gave up) marks the warp aborted: it
    // stops waiting and computing but still takes part in every named barrier, so no warp is left
    // waiting on a barrier a returned warp would never reach.  Every stage issued before the give-up
    // has been waited for, so no bulk copy is in flight when the CTA exits.
    bool aborted = false;
    for (int rg = rg0; rg < rg1; ++rg) {
        for (int ch = 0; ch < cpr; ++ch, ++sidx) {
            const int slot = sidx % nstage;
            if (!aborted && !mbar_wait(&full[slot], (sidx / nstage) & 1)) {
                set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                aborted = true;
            }
            if (aborted) continue;
            const uint8_t* tile = ring + (size_t)slot * kStageBytes + warp * kTileBytes;
            const uint4 wl = *reinterpret_cast<const uint4*>(tile + lane * 16);
            const uint4 wh = *reinterpret_cast<const uint4*>(tile + 512 + lane * 16);
            const uint2 sl = *reinterpret_cast<const uint2*>(tile + 1024 + g * 8);
            const uint2 sh = *reinterpret_cast<const uint2*>(tile + 1088 + g * 8);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);

            const int bbase = (ch * kChunkQuads + warp) * 4;
#pragma unroll
            for (int blk = 0; blk < 4; ++blk) {
                const uint32_t wlo = blk == 0 ? wl.x : blk == 1 ? wl.y : blk == 2 ? wl.z : wl.w;
                const uint32_t whi = blk == 0 ? wh.x : blk == 1 ? wh.y : blk == 2 ? wh.z : wh.w;
                const uint32_t a0 = wlo & 0x0F0F0F0Fu, a2 = (wlo >> 4) & 0x0F0F0F0Fu;
                const uint32_t a1 = whi & 0x0F0F0F0Fu, a3 = (whi >> 4) & 0x0F0F0F0Fu;
                const int b = bbase + blk;
                const uint32_t b0 = act_b[(b * 8 + t) * 8 + g];
                const uint32_t b1 = act_b[(b * 8 + 4 + t) * 8 + g];
                const int2 ci = act_c[b * 4 + t];
                int d[4];
                mma_u8s8(d, a0, a1, a2, a3, b0, b1, ci.x, ci.y, ci.x, ci.y);
                if constexpr (EPI == EPI_BLOCKSUMS) {
                    if (t == 0) {
                        const int r0 = rg * kTileRows + g;
                        a.isum[(size_t)r0 * nb + b] = d[0];
                        a.isum[(size_t)(r0 + 8) * nb + b] = d[2];
                    }
                } else {
                    const float2 xd = act_x[b * 4 + t];
                    const float wdl = h2f_lane(sl, blk), wdh = h2f_lane(sh, blk);
                    acc0 = fmaf(wdl * xd.x, (float)d[0], acc0);
                    acc1 = fmaf(wdl * xd.y, (float)d[1], acc1);
                    acc2 = fmaf(wdh * xd.x, (float)d[2], acc2);
                    acc3 = fmaf(wdh * xd.y, (float)d[3], acc3);
                }
            }
        }
        if constexpr (EPI == EPI_BLOCKSUMS) continue;

        // ---- cross-warp reduction of this row-group (fixed order) ----
        float* rb = red + (rg & 1) * (kConsumerWarps * 128);
        rb[warp * 128 + g * 8 + 2 * t] = acc0;
        rb[warp * 128 + g * 8 + 2 * t + 1] = acc1;
        rb[warp * 128 + (g + 8) * 8 + 2 * t] = acc2;
        rb[warp * 128 + (g + 8) * 8 + 2 * t + 1] = acc3;
        acc0 = acc1 = acc2 = acc3 = 0.f;
        named_sync(1, kConsumerWarps * 32);

        if constexpr (EPI == EPI_STORE) {
            if (tid < 128) {
                const int row = tid >> 3, tok = tid & 7;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) v += rb[w * 128 + tid];
                const int gr = rg * kTileRows + row;
                if (gr < a.out_rows && tok < nv) a.out[(size_t)tok * a.out_ld + gr] = v;
            }
        } else if constexpr (EPI == EPI_QKV) {
            if (tid < 64) {
                const int p = tid >> 3, tok = tid & 7;
                float ve = 0.f, vo = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) {
                    ve += rb[w * 128 + (2 * p) * 8 + tok];
                    vo += rb[w * 128 + (2 * p + 1) * 8 + tok];
                }
                const int gr = rg * kTileRows + 2 * p;
                if (tok < nv) {
                    const int tpos = pos + tok;
                    if (gr < a.q_rows + a.kv_rows) {
                        // RoPE on q and k rows (mistral/mistral_model.h:79-122)
                        const int i = (gr % a.head_dim) >> 1;
                        const float ang = a.theta_inv[i] * (float)tpos;
                        float sn, cs;
                        sincosf(ang, &sn, &cs);
                        const float e2 = fmaf(-vo, sn, ve * cs);
                        const float o2 = fmaf(ve, sn, vo * cs);
                        if (gr < a.q_rows) {
                            a.q_out[(size_t)tok * a.q_rows + gr] = e2 * a.q_scale;
                            a.q_out[(size_t)tok * a.q_rows + gr + 1] = o2 * a.q_scale;
                        } else {
                            const size_t slot = (size_t)(tpos % a.max_seq) * a.kv_rows + (gr - a.q_rows);
                            a.k_cache[slot] = __float2half_rn(e2);
                            a.k_cache[slot + 1] = __float2half_rn(o2);
                        }
                    } else if (gr < a.q_rows + 2 * a.kv_rows) {
                        const size_t slot = (size_t)(tpos % a.max_seq) * a.kv_rows + (gr - a.q_rows - a.kv_rows);
                        a.v_cache[slot] = __float2half_rn(ve);
                        a.v_cache[slot + 1] = __float2half_rn(vo);
                    }
                }
            }
        } else if constexpr (EPI == EPI_SILU_Q8) {
            const int part = rg & 3;  // 0 gate lo, 1 gate hi, 2 up lo, 3 up hi (unit-aligned ranges)
            if (tid < 128) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) v += rb[w * 128 + tid];
                ubuf[part * 128 + tid] = v;
            }
            if (part == 3) {
                if (tid < 128) named_sync(2, 128);
                if (tid < 128) {
                    const int unit = rg >> 2;
                    const int nbh = a.hidden >> 5;
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int tok = warp * 2 + k;
                        const int r = lane & 15, hsel = lane >> 4;
                        const float gv = ubuf[(hsel)*128 + r * 8 + tok];
                        const float uv = ubuf[(2 + hsel) * 128 + r * 8 + tok];
                        // SiLU(g) * u (mistral/mistral_model.h:174-199)
                        const float e = expf(-gv);
                        const float sig = 1.0f / (1.0f + e);
                        const float hv = (gv * sig) * uv;
                        float dq;
                        int sq;
                        const int q = q8_quant_lane(hv, &dq, &sq);
                        if (tok < nv) {
                            a.h.qs[(size_t)tok * a.hidden + unit * 32 + lane] = (int8_t)q;
                            if (lane == 0) {
                                a.h.d[(size_t)tok * nbh + unit] = dq;
                                a.h.sum[(size_t)tok * nbh + unit] = sq;
                            }
                        }
                    }
                }
            }
        }
    }
}

size_t gemv_smem_bytes(int K, int nstage) { return smem_layout(K, nstage).total; }

int gemv_pick_stages(int K, int max_smem) {
    for (int n = kMaxStages; n >= 2; --n)
        if (smem_layout(K, n).total <= (size_t)max_smem) return n;
    return 0;
}

template <int EPI>
static cudaError_t launch_t(const GemvArgs& a, int grid, size_t smem, cudaStream_t st, bool pdl) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemv<EPI>, a);
}

cudaError_t launch_gemv(int epi, const GemvArgs& a, int grid, size_t smem, cudaStream_t st, bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_t<EPI_STORE>(a, grid, smem, st, pdl);
        case EPI_QKV: return launch_t<EPI_QKV>(a, grid, smem, st, pdl);
        case EPI_SILU_Q8: return launch_t<EPI_SILU_Q8>(a, grid, smem, st, pdl);
        case EPI_BLOCKSUMS: return launch_t<EPI_BLOCKSUMS>(a, grid, smem, st, pdl);
    }
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------------------------
// Repack 18-byte AoS Q4_0 blocks (device copy of the GGUF tensor) into the tile16x4 layout.
// One thread per (source row, quad, word t): writes the 16-byte nibble piece; t == 0 also writes
// the row's 4 scales for that quad.
// ---------------------------------------------------------------------------------------------
__global__ void k_repack(const uint8_t* __restrict__ aos, int rows, int cols, RowMap map, uint8_t* __restrict__ dst) {
    const int nq = cols / 128, bpr = cols / 32;
    const long long n = (long long)rows * nq * 4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i & 3);
        const long long rq = i >> 2;
        const int q = (int)(rq % nq);
        const int r = (int)(rq / nq);
        const int dr = (r / map.unit) * map.stride + map.offset + (r % map.unit);
        const int rg = dr / kTileRows, h = (dr % kTileRows) / 8, gg = dr % 8;
        uint8_t* tile = dst + ((size_t)rg * nq + q) * kTileBytes;
        uint32_t words[4];
        uint16_t sc[4];
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
            const uint8_t* b = aos + ((size_t)r * bpr + q * 4 + blk) * 18;
            words[blk] = (uint32_t)b[2 + 4 * t] | ((uint32_t)b[3 + 4 * t] << 8) | ((uint32_t)b[4 + 4 * t] << 16) |
                         ((uint32_t)b[5 + 4 * t] << 24);
            sc[blk] = (uint16_t)(b[0] | (b[1] << 8));
        }
        *reinterpret_cast<uint4*>(tile + h * 512 + (4 * gg + t) * 16) = make_uint4(words[0], words[1], words[2], words[3]);
        if (t == 0) {
            uint2 s2 = make_uint2((uint32_t)sc[0] | ((uint32_t)sc[1] << 16), (uint32_t)sc[2] | ((uint32_t)sc[3] << 16));
            *reinterpret_cast<uint2*>(tile + 1024 + (h * 8 + gg) * 8) = s2;
        }
    }
}

cudaError_t launch_repack(const uint8_t* aos, int rows, int cols, RowMap map, uint8_t* dst, cudaStream_t st) {
    long long n = (long long)rows * (cols / 128) * 4;
    int blocks = (int)((n + 255) / 256);
    if (blocks > 65535 * 8) blocks = 65535 * 8;
    k_repack<<<blocks, 256, 0, st>>>(aos, rows, cols, map, dst);
    return cudaGetLastError();
}

}  // namespace sd
