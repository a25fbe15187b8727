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
// stages of up to 16 x 1152-byte tiles filled by 1-D bulk copies (TMA engine) issued by a producer
// warp; 16 consumer warps each take one tile (16 rows x 4 blocks) per stage.  The weight stream does not depend
// on the previous kernel, so the producer starts before griddepcontrol.wait (PDL overlap).
//
// Determinism / batch invariance: every (row, token) value is accumulated in a fixed order (per warp
// over its tiles, then warps 0..15), independent of S and of the other tokens, so a token's result in
// an S=5 verify is bit-identical to its S=1 decode result.
#include "sd_common.cuh"

namespace sd {

namespace {

// Shared memory: weight ring | B fragments (+ zero pad) | C quads | activation scales |
//                partial-sum slots | SiLU unit | mbarriers
struct SmemLayout {
    size_t ring, act_b, act_zero, act_c, act_x, red, ubuf, bars, total;
};

// Kp = the K range one CTA covers (K / kparts).
__host__ __device__ inline SmemLayout smem_layout(int Kp, int S, int chunk, int nstage) {
    SmemLayout L;
    const size_t nb = (size_t)Kp / 32;
    L.ring = 0;
    L.act_b = L.ring + (size_t)nstage * kRPW * chunk * kTileBytes;
    L.act_zero = L.act_b + nb * (size_t)(4 * S) * 8;   // uint2 per (block, lane < 4S)
    L.act_c = L.act_zero + (size_t)4 * (4 * S) * 8;    // zeros read by lanes whose token g >= S
    L.act_x = L.act_c + nb * 4 * 16;                   // int4 C quad per (block, t)
    L.red = L.act_x + nb * 4 * 8;                      // float2 scales per (block, t)
    L.ubuf = L.red + (size_t)kRedSlots * kRPW * kConsumerWarps * 128 * 4;
    L.bars = L.ubuf + 4 * 128 * 4;
    L.total = L.bars + (2 * kMaxStages + 2 * kRedSlots) * 8;
    return L;
}

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float2 h2x2f(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// The MMA accumulator is initialised with -8*sum(codes) + kMagic: the result bits are then the fp32
// value 1.5*2^23 + isum (exact for |isum| < 2^22; |isum| <= 32*8*128 here), so one exact FADD
// recovers (float)isum without the quarter-rate I2F conversion.
constexpr int kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

}  // namespace

template <int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = a.S;
    const int chunk = a.chunk;
    const int nq_p = a.nq / a.kparts;          // quads of this CTA's K slice
    const int Kp = nq_p * 128;
    const int nb = Kp >> 5;                    // blocks of the slice
    const SmemLayout L = smem_layout(Kp, S, chunk, a.nstage);
    uint8_t* ring = smem + L.ring;
    uint2* act_b = reinterpret_cast<uint2*>(smem + L.act_b);
    uint2* act_zero = reinterpret_cast<uint2*>(smem + L.act_zero);
    int4* act_c = reinterpret_cast<int4*>(smem + L.act_c);
    float2* act_x = reinterpret_cast<float2*>(smem + L.act_x);
    float* red = reinterpret_cast<float*>(smem + L.red);
    float* ubuf = reinterpret_cast<float*>(smem + L.ubuf);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + kMaxStages;
    uint64_t* red_full = empty + kMaxStages;    // consumers -> epilogue (count: consumer warps)
    uint64_t* red_empty = red_full + kRedSlots; // epilogue -> consumers (count: epilogue warps)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nstage = a.nstage;
    const uint32_t half_bytes = (uint32_t)chunk * kTileBytes;   // one row-group's share of a stage
    const uint32_t stage_bytes = kRPW * half_bytes;

    if (a.ctrl && a.ctrl->done) return;  // advisory early exit (the flag only ever goes 0 -> 1)

    // CTAs are split evenly over the K slices; within a slice each CTA takes a contiguous unit range.
    const int G = gridDim.x;
    const int part = (int)((long long)blockIdx.x * a.kparts / G);
    const int c0p = (int)(((long long)part * G + a.kparts - 1) / a.kparts);       // first CTA of slice
    const int c1p = (int)(((long long)(part + 1) * G + a.kparts - 1) / a.kparts);
    const int cpp = c1p - c0p, ci = blockIdx.x - c0p;
    const int u0 = (int)((long long)ci * a.n_units / cpp), u1 = (int)((long long)(ci + 1) * a.n_units / cpp);
    const int rg0 = u0 * a.rg_per_unit, rg1 = u1 * a.rg_per_unit;
    const int cpr = nq_p / chunk;              // ring stages per row-group pair
    const int n_pairs = (rg1 - rg0) / kRPW;
    const int n_stages_total = n_pairs * cpr;
    const int q0 = part * nq_p;                // first quad of the slice
    const int kb0 = q0 * 4;                    // first block of the slice

    if (tid == 0) {
        for (int i = 0; i < nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        for (int i = 0; i < kRedSlots; ++i) {
            mbar_init(&red_full[i], kConsumerWarps);
            mbar_init(&red_empty[i], kEpiWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kConsumerWarps + kEpiWarps) {
        // -------- producer: stream this CTA's row-group pairs through the ring (2 bulk copies/stage) --------
        // Weights do not depend on the previous kernel, so this runs before griddepcontrol.wait.
        if (lane == 0) {
            for (int s = 0; s < n_stages_total; ++s) {
                const int slot = s % nstage;
                if (s >= nstage && !mbar_wait(&empty[slot], ((s / nstage) - 1) & 1)) {
                    set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
                    break;  // consumers give up on the stages never issued
                }
                const int rg = rg0 + (s / cpr) * kRPW, ch = s % cpr;
                const uint8_t* src = a.w + ((size_t)rg * a.nq + q0 + (size_t)ch * chunk) * kTileBytes;
                uint8_t* dst = ring + (size_t)slot * stage_bytes;
                mbar_arrive_expect_tx(&full[slot], stage_bytes);
#pragma unroll
                for (int r = 0; r < kRPW; ++r)
                    bulk_g2s(dst + r * half_bytes, src + (size_t)r * a.nq * kTileBytes, half_bytes, &full[slot]);
            }
        }
        return;
    }

    // ---------------- stage activations of the slice (depends on the previous kernel) ----------------
    pdl_wait();
    int nv = S;
    int pos = 0;
    if (a.ctrl) {
        nv = min(a.ctrl->n_valid, S);
        pos = a.ctrl->pos;
    }
    const int nthr = (kConsumerWarps + kEpiWarps) * 32;
    {
        // B fragments: act_b[b*4S + 4s + tt] = (word tt of token s, word 4+tt of token s) of block b
        const int n16 = S * nb * 2;
        for (int i = tid; i < n16; i += nthr) {
            const int s = i / (nb * 2), rem = i - s * (nb * 2);
            const int b = rem >> 1, half = rem & 1;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (s < nv)
                v = *reinterpret_cast<const uint4*>(a.act.qs + (size_t)s * a.K + (size_t)(kb0 + b) * 32 + half * 16);
            uint32_t* base = reinterpret_cast<uint32_t*>(act_b + (size_t)b * 4 * S + 4 * s) + half;
            base[0] = v.x;
            base[2] = v.y;
            base[4] = v.z;
            base[6] = v.w;
        }
        for (int i = tid; i < 4 * 4 * S; i += nthr) act_zero[i] = make_uint2(0, 0);
        // C quad (-8*sum + magic for tokens 2t, 2t+1, repeated for rows g+8) and scales (xd pair)
        const int nbK = a.K >> 5;
        for (int i = tid; i < nb * 4; i += nthr) {
            const int b = i >> 2, tt = i & 3;
            const int s0 = 2 * tt, s1 = 2 * tt + 1;
            int c0 = kMagicI, c1 = kMagicI;
            float x0 = 0.f, x1 = 0.f;
            if (s0 < nv) {
                c0 = kMagicI - 8 * a.act.sum[(size_t)s0 * nbK + kb0 + b];
                x0 = a.act.d[(size_t)s0 * nbK + kb0 + b];
            }
            if (s1 < nv) {
                c1 = kMagicI - 8 * a.act.sum[(size_t)s1 * nbK + kb0 + b];
                x1 = a.act.d[(size_t)s1 * nbK + kb0 + b];
            }
            act_c[i] = make_int4(c0, c1, c0, c1);
            act_x[i] = make_float2(x0, x1);
        }
    }
    named_sync(1, nthr);

    if (warp >= kConsumerWarps) {
        if constexpr (EPI == EPI_BLOCKSUMS) return;  // consumers write the block sums themselves
        // ================= epilogue warps: reduce the partials of one row-group, apply the epilogue ======
        const int r = warp - kConsumerWarps;  // row-group of the pair this warp finishes
        bool ab = false;
        for (int pi = 0; pi < n_pairs; ++pi) {
            const int slot = pi % kRedSlots;
            if (!ab && !mbar_wait(&red_full[slot], (pi / kRedSlots) & 1)) {
                set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                ab = true;
            }
            const int rg = rg0 + pi * kRPW + r;
            const float* rr = red + ((size_t)slot * kRPW + r) * kConsumerWarps * 128;
            float v[4] = {0.f, 0.f, 0.f, 0.f};  // elements lane + 32*k: row = e>>3, tok = e&7
            if (!ab) {
                for (int w = 0; w < chunk; ++w) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) v[k] += rr[w * 128 + lane + 32 * k];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_empty[slot]);
            if (ab) continue;
            if constexpr (EPI == EPI_STORE) {
                float* out = a.out + (size_t)part * a.part_stride;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int e = lane + 32 * k, row = e >> 3, tok = e & 7;
                    const int gr = rg * kTileRows + row;
                    if (gr < a.out_rows && tok < nv) out[(size_t)tok * a.out_ld + gr] = v[k];
                }
            } else if constexpr (EPI == EPI_QKV) {
                // element (row, tok) lives in lane (row*8 + tok) % 32, register (row*8 + tok) / 32;
                // the partner row (row ^ 1) of a RoPE pair is the same register of lane ^ 8
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int e = lane + 32 * k;
                    const int row = e >> 3, tok = e & 7;
                    const float other = __shfl_xor_sync(0xffffffffu, v[k], 8);
                    if ((row & 1) == 0 && tok < nv) {
                        const float ve = v[k], vo = other;
                        const int gr = rg * kTileRows + row;
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
                                const size_t sl = (size_t)(tpos % a.max_seq) * a.kv_rows + (gr - a.q_rows);
                                a.k_cache[sl] = __float2half_rn(e2);
                                a.k_cache[sl + 1] = __float2half_rn(o2);
                            }
                        } else if (gr < a.q_rows + 2 * a.kv_rows) {
                            const size_t sl = (size_t)(tpos % a.max_seq) * a.kv_rows + (gr - a.q_rows - a.kv_rows);
                            a.v_cache[sl] = __float2half_rn(ve);
                            a.v_cache[sl + 1] = __float2half_rn(vo);
                        }
                    }
                }
            } else if constexpr (EPI == EPI_SILU_Q8) {
                // unit of 4 row-groups = 2 pairs: (gate lo, gate hi), (up lo, up hi)
                const int pair_in_unit = ((rg0 / kRPW) + pi) & 1;
#pragma unroll
                for (int k = 0; k < 4; ++k) ubuf[(pair_in_unit * 2 + r) * 128 + lane + 32 * k] = v[k];
                if (pair_in_unit == 1) {
                    named_sync(2, kEpiWarps * 32);
                    const int unit = rg >> 2;
                    const int nbh = a.hidden >> 5;
                    for (int k = 0; k < 4; ++k) {
                        const int tok = r * 4 + k;
                        const int rr2 = lane & 15, hsel = lane >> 4;
                        const float gv = ubuf[hsel * 128 + rr2 * 8 + tok];
                        const float uv = ubuf[(2 + hsel) * 128 + rr2 * 8 + tok];
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
                    named_sync(2, kEpiWarps * 32);  // ubuf reused by the next unit
                }
            }
        }
        return;
    }

    // ================= consumer warps: int8 MMA over one tile of each row-group of the pair ==========
    float2 accL[kRPW], accH[kRPW];
#pragma unroll
    for (int r = 0; r < kRPW; ++r) accL[r] = accH[r] = make_float2(0.f, 0.f);
    const bool has_tile = warp < chunk;
    const bool zero_lane = g >= S;             // token column g beyond the launch's S reads zeros
    const uint2* bf_lane = zero_lane ? act_zero + t : act_b + lane;
    int sidx = 0;
    // A stage that never arrives (only possible if the producer gave up) marks the warp aborted: it
    // stops waiting and computing but keeps its place in every handshake, so no warp is left waiting
    // on one that returned.  Every stage issued before the give-up has been waited for, so no bulk
    // copy is in flight when the CTA exits.
    bool aborted = false;
    for (int pi = 0; pi < n_pairs; ++pi) {
        const int rg = rg0 + pi * kRPW;
        for (int ch = 0; ch < cpr; ++ch, ++sidx) {
            const int slot = sidx % nstage;
            if (!aborted && !mbar_wait(&full[slot], (sidx / nstage) & 1)) {
                set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                aborted = true;
            }
            if (aborted) continue;
            uint4 wl[kRPW], wh[kRPW];
            uint2 sl[kRPW], sh[kRPW];
            if (has_tile) {
#pragma unroll
                for (int r = 0; r < kRPW; ++r) {
                    const uint8_t* tile = ring + (size_t)slot * stage_bytes + r * half_bytes + warp * kTileBytes;
                    wl[r] = *reinterpret_cast<const uint4*>(tile + lane * 16);
                    wh[r] = *reinterpret_cast<const uint4*>(tile + 512 + lane * 16);
                    sl[r] = *reinterpret_cast<const uint2*>(tile + 1024 + g * 8);
                    sh[r] = *reinterpret_cast<const uint2*>(tile + 1088 + g * 8);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (!has_tile) continue;

            float2 dl[kRPW][2], dh[kRPW][2];
#pragma unroll
            for (int r = 0; r < kRPW; ++r) {
                dl[r][0] = h2x2f(sl[r].x);
                dl[r][1] = h2x2f(sl[r].y);
                dh[r][0] = h2x2f(sh[r].x);
                dh[r][1] = h2x2f(sh[r].y);
            }
            const int bbase = (ch * chunk + warp) * 4;   // block index within the slice
            const uint2* bf_p = zero_lane ? bf_lane : bf_lane + (size_t)bbase * 4 * S;
            const int4* c_p = act_c + bbase * 4 + t;
            const float2* x_p = act_x + bbase * 4 + t;
#pragma unroll
            for (int blk = 0; blk < 4; ++blk) {
                const uint2 bf = bf_p[blk * 4 * S];
                const int4 cq = c_p[blk * 4];
                const float2 xd = x_p[blk * 4];
#pragma unroll
                for (int r = 0; r < kRPW; ++r) {
                    const uint32_t wlo = blk == 0 ? wl[r].x : blk == 1 ? wl[r].y : blk == 2 ? wl[r].z : wl[r].w;
                    const uint32_t whi = blk == 0 ? wh[r].x : blk == 1 ? wh[r].y : blk == 2 ? wh[r].z : wh[r].w;
                    const uint32_t a0 = wlo & 0x0F0F0F0Fu, a2 = (wlo >> 4) & 0x0F0F0F0Fu;
                    const uint32_t a1 = whi & 0x0F0F0F0Fu, a3 = (whi >> 4) & 0x0F0F0F0Fu;
                    int d[4];
                    mma_u8s8(d, a0, a1, a2, a3, bf.x, bf.y, cq.x, cq.y, cq.z, cq.w);
                    if constexpr (EPI == EPI_BLOCKSUMS) {
                        if (t == 0 && (rg + r) * kTileRows < a.out_rows) {
                            const int r0 = (rg + r) * kTileRows + g;
                            const size_t nbK = (size_t)(a.K >> 5);
                            a.isum[(size_t)r0 * nbK + kb0 + bbase + blk] = d[0] - kMagicI;
                            a.isum[(size_t)(r0 + 8) * nbK + kb0 + bbase + blk] = d[2] - kMagicI;
                        }
                    } else {
                        const float wdl = (blk & 1) ? dl[r][blk >> 1].y : dl[r][blk >> 1].x;
                        const float wdh = (blk & 1) ? dh[r][blk >> 1].y : dh[r][blk >> 1].x;
                        const float2 fL = __fadd2_rn(make_float2(__int_as_float(d[0]), __int_as_float(d[1])),
                                                     make_float2(-kMagicF, -kMagicF));
                        const float2 fH = __fadd2_rn(make_float2(__int_as_float(d[2]), __int_as_float(d[3])),
                                                     make_float2(-kMagicF, -kMagicF));
                        // (wd*xd) * (float)isum accumulated per block, as mistral/dequant.h:1085
                        const float2 sL = __fmul2_rn(make_float2(wdl, wdl), xd);
                        const float2 sH = __fmul2_rn(make_float2(wdh, wdh), xd);
                        accL[r] = __ffma2_rn(sL, fL, accL[r]);
                        accH[r] = __ffma2_rn(sH, fH, accH[r]);
                    }
                }
            }
        }
        if constexpr (EPI == EPI_BLOCKSUMS) continue;
        // ---- hand the pair's partials to the epilogue warps ----
        const int rs = pi % kRedSlots;
        if (pi >= kRedSlots && !aborted && !mbar_wait(&red_empty[rs], ((pi / kRedSlots) - 1) & 1)) {
            set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
            aborted = true;
        }
        if (has_tile && !aborted) {
#pragma unroll
            for (int r = 0; r < kRPW; ++r) {
                float* rr = red + (((size_t)rs * kRPW + r) * kConsumerWarps + warp) * 128;
                *reinterpret_cast<float2*>(&rr[g * 8 + 2 * t]) = accL[r];
                *reinterpret_cast<float2*>(&rr[(g + 8) * 8 + 2 * t]) = accH[r];
            }
        }
#pragma unroll
        for (int r = 0; r < kRPW; ++r) accL[r] = accH[r] = make_float2(0.f, 0.f);
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_full[rs]);
    }
}

size_t gemv_smem_bytes(int Kp, int S, int chunk, int nstage) { return smem_layout(Kp, S, chunk, nstage).total; }

int gemv_pick_stages(int Kp, int S, int chunk, int max_smem) {
    for (int n = kMaxStages; n >= 2; --n)
        if (smem_layout(Kp, S, chunk, n).total <= (size_t)max_smem) return n;
    return 0;
}

// Allow the full opt-in shared memory for every matvec variant on the current device.  Called before
// any launch (and before stream capture: it is not a stream operation but is kept out of captures).
cudaError_t gemv_init_attrs(int max_smem) {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_gemv<EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(k_gemv<EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(k_gemv<EPI_SILU_Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    return cudaFuncSetAttribute(k_gemv<EPI_BLOCKSUMS>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

template <int EPI>
static cudaError_t launch_t(const GemvArgs& a, int grid, size_t smem, cudaStream_t st, bool pdl) {
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

__global__ void k_sum_parts(const float* __restrict__ parts, float* __restrict__ out, int n, int kparts, size_t stride) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float v = 0.f;
        for (int p = 0; p < kparts; ++p) v += parts[(size_t)p * stride + i];
        out[i] = v;
    }
}

cudaError_t launch_sum_parts(const float* parts, float* out, int n, int kparts, size_t stride, cudaStream_t st) {
    int grid = (n + 255) / 256;
    k_sum_parts<<<grid > 1024 ? 1024 : grid, 256, 0, st>>>(parts, out, n, kparts, stride);
    return cudaGetLastError();
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
__global__ void k_repack(const uint8_t* __restrict__ aos, int rows, int cols, size_t src_row_bytes, RowMap map,
                         uint8_t* __restrict__ dst) {
    const int nq = cols / 128;
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
            const uint8_t* b = aos + (size_t)r * src_row_bytes + ((size_t)q * 4 + blk) * 18;
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

// aos points at row 0, column block 0 of the (sub)matrix; consecutive rows are src_row_bytes apart
// (a column slice of a wider matrix for tensor-parallel shards).
cudaError_t launch_repack(const uint8_t* aos, int rows, int cols, size_t src_row_bytes, RowMap map, uint8_t* dst,
                          cudaStream_t st) {
    long long n = (long long)rows * (cols / 128) * 4;
    int blocks = (int)((n + 255) / 256);
    if (blocks > 65535 * 8) blocks = 65535 * 8;
    k_repack<<<blocks, 256, 0, st>>>(aos, rows, cols, src_row_bytes, map, dst);
    return cudaGetLastError();
}

}  // namespace sd
