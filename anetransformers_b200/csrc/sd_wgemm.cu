// sd_wgemm.cu -- wide-token W4A8 GEMM (Q4_0 weights x Q8_0 activations of M tokens) for the batched
// verify / prefill of many streams.
//
// Per row r, token m:  Y[m][r] = sum_b (wd[r,b] * xd[m,b]) * isum[r,m,b]
//   isum = sum_j (q_j - 8) * x8_j (exact int32, the reference's SDOT block sum, mistral/dequant.h:1068-1087)
// with the same per-block fp32 arithmetic as the matvec (sd_gemv.cu), so a token's value over a K slice does
// not depend on the batch.  The matvec reads every weight once per 8 tokens; here a weight tile is read once
// per token tile of up to 160 tokens, which turns the M = (streams x verify width) contraction of batched
// serving from weight-bandwidth bound into a dense int8 contraction.
//
// CTA = 8 consumer warps + 1 producer warp, one CTA per SM, persistent over units.  Unit = (row tile of 128
// rows, K slice, token tile of tt_n8 n8 tiles); units that share weights are adjacent so their weight reads
// meet in L2.  Per quad (128 columns) a ring stage holds the row tile's 8 weight tiles (1152-byte tile16x4
// tiles, one bulk copy each) and the token tile's activation segments (one bulk copy; sd_internal.h wide
// image).  Consumer warp (wr, wt) owns rows 64 wr .. +63 (row-groups 4wr .. 4wr+3) and n8 tiles
// [wt * per, wt * per + per) of the token tile: per block it unpacks the A fragments of its 4 row-groups once
// and uses each B fragment for 4 MMAs (m16n8k32, u8 nibbles x s8 codes, accumulator started at the bits of
// kMagic so one FADD recovers the exact block sum).
#include "sd_dev.cuh"

namespace sd {

size_t wgemm_smem_bytes(int tt_n8, int nstage) {
    return (size_t)nstage * (kWgWStage + (size_t)tt_n8 * kWSeg) + 2 * kWgMaxStages * 8;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

// Unit u -> (row tile, K slice, token tile); quads [q0, q1) of the slice.
struct WgUnit {
    int rt, kp, tt, q0, q1;
};

__device__ __forceinline__ WgUnit wg_unit(const WGemmArgs& a, int u) {
    WgUnit w;
    const int per_rt = a.kparts * a.n_tt;
    w.rt = u / per_rt;
    const int r2 = u - w.rt * per_rt;
    w.kp = r2 / a.n_tt;
    w.tt = r2 - w.kp * a.n_tt;
    w.q0 = (int)((long long)w.kp * a.nq / a.kparts);
    w.q1 = (int)((long long)(w.kp + 1) * a.nq / a.kparts);
    return w;
}

template <int EPI>
__global__ void __launch_bounds__(kWgThreads, 1) k_wgemm(const WGemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int nstage = a.nstage;
    const uint32_t SB = (uint32_t)a.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nstage * SB);
    uint64_t* empty = full + kWgMaxStages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_units = a.n_rt * a.kparts * a.n_tt;

    if (tid == 0) {
        for (int i = 0; i < nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kWgWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();

    if (warp == kWgWarps) {
        // ---------------- producer: one weight copy per row-group and one activation copy per stage ----------------
        if (lane == 0) {
            RingPos rp;
            int s = 0;
            for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
                const WgUnit w = wg_unit(a, u);
                const int nrg = min(kWgRG, a.n_rg - w.rt * kWgRG);
                const int n0 = w.tt * a.tt_n8, nn = min(a.tt_n8, a.NT - n0);
                const uint32_t bytes = (uint32_t)(nrg * kTileBytes + nn * kWSeg);
                const uint8_t* wsrc = a.w + (size_t)w.rt * kWgRG * a.nq * kTileBytes;
                for (int q = w.q0; q < w.q1; ++q, ++s, rp.advance(nstage)) {
                    if (s >= nstage && !mbar_wait(&empty[rp.slot], rp.phase ^ 1)) {
                        set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
                        return;  // the consumers run out their bounded waits on the stages never issued
                    }
                    uint8_t* dst = smem + (size_t)rp.slot * SB;
                    mbar_arrive_expect_tx(&full[rp.slot], bytes);
                    for (int r = 0; r < nrg; ++r)
                        bulk_g2s(dst + r * kTileBytes, wsrc + ((size_t)r * a.nq + q) * kTileBytes, kTileBytes, &full[rp.slot]);
                    bulk_g2s(dst + kWgWStage, a.act + ((size_t)q * a.NT + n0) * kWSeg, (uint32_t)(nn * kWSeg),
                             &full[rp.slot]);
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int wr = warp >> 2, wt = warp & 3;
    const int g = lane >> 2, t = lane & 3;
    const int per = (a.tt_n8 + 3) >> 2;  // n8 tiles per warp
    RingPos rp;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const WgUnit w = wg_unit(a, u);
        const int n0 = w.tt * a.tt_n8, nn = min(a.tt_n8, a.NT - n0);
        const int nb0 = wt * per;
        const int nw = max(0, min(per, nn - nb0));  // n8 tiles this warp computes
        float2 accL[4][kWgMaxN8], accH[4][kWgMaxN8];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int n = 0; n < kWgMaxN8; ++n) accL[r][n] = accH[r][n] = make_float2(0.f, 0.f);
        for (int q = w.q0; q < w.q1; ++q, rp.advance(nstage)) {
            if (!mbar_wait(&full[rp.slot], rp.phase)) {
                set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                return;
            }
            const uint32_t st = smem_u32(smem + (size_t)rp.slot * SB);
            if (nw > 0) {
                // scales once per quad; nibble words per block (fewer live registers: 9 warps share the
                // 4 x 16K-register scheduler partitions, 3 on one, so a thread has at most 168)
                uint4 sc[4];
                const uint32_t tile0 = st + 4 * wr * kTileBytes + lane * 16;
#pragma unroll
                for (int r = 0; r < 4; ++r) sc[r] = lds128(st + (4 * wr + r) * kTileBytes + 1024 + g * 16);
                const uint32_t ab = st + kWgWStage + nb0 * kWSeg + lane * 8;
                const uint32_t mb = st + kWgWStage + nb0 * kWSeg + 1024 + t * 16;
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) {
                    uint32_t A[4][4];
                    float wdl[4], wdh[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const uint32_t wlo = lds32(tile0 + r * kTileBytes + blk * 4);
                        const uint32_t whi = lds32(tile0 + r * kTileBytes + 512 + blk * 4);
                        A[r][0] = wlo & 0x0F0F0F0Fu;
                        A[r][1] = whi & 0x0F0F0F0Fu;
                        A[r][2] = (wlo >> 4) & 0x0F0F0F0Fu;
                        A[r][3] = (whi >> 4) & 0x0F0F0F0Fu;
                        // scales [g][h][blk]: x = row g blocks 0,1; y = row g blocks 2,3; z, w = row g + 8
                        const float2 dl = h2x2f(blk < 2 ? sc[r].x : sc[r].y);
                        const float2 dh = h2x2f(blk < 2 ? sc[r].z : sc[r].w);
                        wdl[r] = (blk & 1) ? dl.y : dl.x;
                        wdh[r] = (blk & 1) ? dh.y : dh.x;
                    }
#pragma unroll
                    for (int n = 0; n < kWgMaxN8; ++n) {
                        if (n < nw) {
                            const uint2 bf = lds64(ab + n * kWSeg + blk * 256);
                            const uint4 mu = lds128(mb + n * kWSeg + blk * 64);
                            const float2 xd = make_float2(__uint_as_float(mu.x), __uint_as_float(mu.y));
                            const float2 off = make_float2(__uint_as_float(mu.z), __uint_as_float(mu.w));
#pragma unroll
                            for (int r = 0; r < 4; ++r) {
                                int d[4];
                                mma_u8s8(d, A[r][0], A[r][1], A[r][2], A[r][3], bf.x, bf.y, kMagicI, kMagicI, kMagicI, kMagicI);
                                const float2 fL = __fadd2_rn(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), off);
                                const float2 fH = __fadd2_rn(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), off);
                                // (wd*xd) * (float)isum accumulated per block, as mistral/dequant.h:1085
                                const float2 sL = __fmul2_rn(make_float2(wdl[r], wdl[r]), xd);
                                const float2 sH = __fmul2_rn(make_float2(wdh[r], wdh[r]), xd);
                                accL[r][n] = __ffma2_rn(sL, fL, accL[r][n]);
                                accH[r][n] = __ffma2_rn(sH, fH, accH[r][n]);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[rp.slot]);
        }
        if (nw <= 0) continue;
        const int mbase = (n0 + nb0) * 8 + 2 * t;  // token of .x in n8 tile 0 of this warp
        if constexpr (EPI == WG_STORE) {
            float* out = a.out + (size_t)w.kp * a.part_stride;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int row0 = ((w.rt * kWgRG + 4 * wr + r) << 4) + g;
#pragma unroll
                for (int n = 0; n < kWgMaxN8; ++n) {
                    if (n >= nw) break;
                    const int m0 = mbase + 8 * n;
                    if (m0 < a.M) {
                        if (row0 < a.out_rows) out[(size_t)m0 * a.ld + row0] = accL[r][n].x;
                        if (row0 + 8 < a.out_rows) out[(size_t)m0 * a.ld + row0 + 8] = accH[r][n].x;
                    }
                    if (m0 + 1 < a.M) {
                        if (row0 < a.out_rows) out[(size_t)(m0 + 1) * a.ld + row0] = accL[r][n].y;
                        if (row0 + 8 < a.out_rows) out[(size_t)(m0 + 1) * a.ld + row0 + 8] = accH[r][n].y;
                    }
                }
            }
        } else {
            // gate|up unit (64 rows: gate row-groups 0, 1, up row-groups 2, 3 of this warp's half) = one Q8_0
            // block hb of h.  Lane holds hidden units g, g + 8 (row-group 0 / 2 rows g, g + 8) and 16 + g, 24 + g
            // (row-group 1 / 3) for tokens m0 (.x) and m0 + 1 (.y).
            const int hb = w.rt * 2 + wr;
            const bool unit_ok = hb < (a.hidden >> 5);
#pragma unroll
            for (int n = 0; n < kWgMaxN8; ++n) {
                if (n >= nw) break;
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int m = mbase + 8 * n + k;
                    float gv[4], uv[4];
                    gv[0] = k ? accL[0][n].y : accL[0][n].x;
                    gv[1] = k ? accH[0][n].y : accH[0][n].x;
                    gv[2] = k ? accL[1][n].y : accL[1][n].x;
                    gv[3] = k ? accH[1][n].y : accH[1][n].x;
                    uv[0] = k ? accL[2][n].y : accL[2][n].x;
                    uv[1] = k ? accH[2][n].y : accH[2][n].x;
                    uv[2] = k ? accL[3][n].y : accL[3][n].x;
                    uv[3] = k ? accH[3][n].y : accH[3][n].x;
                    float hv[4];
                    float am = 0.f;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // SiLU(g) * u (mistral/mistral_model.h:174-199), as the matvec epilogue computes it
                        const float e = expf(-gv[j]);
                        const float sig = 1.0f / (1.0f + e);
                        hv[j] = (gv[j] * sig) * uv[j];
                        am = fmaxf(am, fabsf(hv[j]));
                    }
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                    // Q8_0 of the block (mistral/dequant.h:545-599)
                    const float d = __fdiv_rn(am, 127.0f);
                    int qv[4] = {0, 0, 0, 0};
                    if (am != 0.0f) {
                        const float id = __fdiv_rn(1.0f, d);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int rq = __float2int_rn(__fmul_rn(hv[j], id));
                            qv[j] = rq > 127 ? 127 : (rq < -128 ? -128 : rq);
                        }
                    }
                    int sum = (qv[0] + qv[1]) + (qv[2] + qv[3]);
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                    // element u = g + 8j is byte (g & 3) of code word (g >> 2) + 2j
                    uint32_t words[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t v = (uint32_t)(qv[j] & 0xFF) << (8 * (g & 3));
                        v |= __shfl_xor_sync(0xffffffffu, v, 4);
                        v |= __shfl_xor_sync(0xffffffffu, v, 8);
                        words[j] = v;
                    }
                    if (unit_ok && m < a.M && (g & 3) == 0) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) wimg_put_word(a.h, m, hb, (g >> 2) + 2 * j, words[j]);
                        if (g == 0) wimg_put_meta(a.h, m, hb, d, sum);
                    }
                }
            }
        }
    }
}

cudaError_t wgemm_init_attrs(int max_smem) {
    cudaError_t e = cudaFuncSetAttribute(k_wgemm<WG_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_wgemm<WG_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

cudaError_t launch_wgemm(int epi, const WGemmArgs& a, int grid, size_t smem, cudaStream_t st) {
    if (epi == WG_SILU)
        k_wgemm<WG_SILU><<<grid, kWgThreads, smem, st>>>(a);
    else
        k_wgemm<WG_STORE><<<grid, kWgThreads, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace sd
