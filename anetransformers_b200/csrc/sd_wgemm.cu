// sd_wgemm.cu -- wide-token W4A8 GEMM (Q4_0 weights x Q8_0 activations of M tokens) for the batched
// verify / prefill of many streams.
//
// Per row r, token m:  Y[m][r] = sum_b (wd[r,b] * xd[m,b]) * isum[r,m,b]
//   isum = sum_j (q_j - 8) * x8_j (exact int32, the reference's SDOT block sum, mistral/dequant.h:1068-1087)
// with the same per-block fp32 arithmetic as the matvec (sd_gemv.cu), so a token's value over a K slice does
// not depend on the batch.  The matvec reads every weight once per 8 tokens; here a weight tile is read once
// per token tile of up to 128 tokens, which turns the M = (streams x verify width) contraction of batched
// serving from weight-bandwidth bound into a dense int8 contraction.
//
// CTA = 16 warps, one CTA per SM, persistent over units.  Unit = (row tile of 128 rows, K slice, token tile
// of tt_n8 n8 tiles); units that share weights are adjacent so their weight reads meet in L2.  Per quad (128
// columns) a ring stage holds the row tile's weights in the wide layout (sd_batch.h; one bulk copy) and the
// token tile's activation segments (one bulk copy; sd_internal.h wide image); lane 0 of warp 0 keeps the ring
// filled ahead of the stage it consumes.  Warp (wr, wt) owns rows 64 wr .. +63 (row-groups 4wr .. 4wr+3) and
// n8 tiles [wt * per, wt * per + per) of the token tile: per block it loads its B fragments once and the A
// words of its four row-groups with two conflict-free 16-byte loads, and runs 4 x per MMAs (m16n8k32, u8
// nibbles x s8 codes, accumulator started at the bits of kMagic so one FADD recovers the exact block sum).
#include "sd_dev.cuh"

namespace sd {

size_t wgemm_smem_bytes(int tt_n8, int nstage) {
    return (size_t)nstage * (kWgWStage + (size_t)tt_n8 * kWSeg) + 2 * kWgMaxStages * 8;
}

// The int8 MMA as a pure register operation (no volatile): the compiler may interleave it with the shared
// loads and the fp32 epilogue of other fragments.
__device__ __forceinline__ void mma_u8s8_pure(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(kMagicI));
}

__device__ __forceinline__ uint32_t pick4(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
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

// The ring's producer (lane 0 of warp 0): walks the same (unit, quad) sequence as the consumers.
struct WgProducer {
    int u, q, q1, s;  // next unit / quad to issue, its slice end, stages issued
    const uint8_t* wsrc;
    const uint8_t* asrc;
    uint32_t bytes, abytes;
    RingPos rp;
    bool live;

    __device__ __forceinline__ void start_unit(const WGemmArgs& a, int n_units) {
        live = u < n_units;
        if (!live) return;
        const WgUnit w = wg_unit(a, u);
        q = w.q0;
        q1 = w.q1;
        const int n0 = w.tt * a.tt_n8, nn = min(a.tt_n8, a.NT - n0);
        abytes = (uint32_t)(nn * kWSeg);
        bytes = (uint32_t)kWgWStage + abytes;
        wsrc = a.w + (size_t)w.rt * a.nq * kWgWStage;
        asrc = a.act + (size_t)n0 * kWSeg;
    }

    // Issue stages while fewer than `limit` have been issued.  block: wait (bounded) for a free slot, false if
    // the wait ran out; otherwise stop at the first slot still in use.
    __device__ __forceinline__ bool fill(const WGemmArgs& a, int n_units, int limit, uint8_t* smem, uint32_t SB,
                                         uint64_t* full, uint64_t* empty, int nstage, bool block = true) {
        while (live && s < limit) {
            if (s >= nstage) {
                if (!block) {
                    if (!mbar_try_wait(&empty[rp.slot], rp.phase ^ 1)) return true;
                } else if (!mbar_wait(&empty[rp.slot], rp.phase ^ 1)) {
                    live = false;
                    return false;
                }
            }
            uint8_t* dst = smem + (size_t)rp.slot * SB;
            mbar_arrive_expect_tx(&full[rp.slot], bytes);
            bulk_g2s(dst, wsrc + (size_t)q * kWgWStage, kWgWStage, &full[rp.slot]);
            bulk_g2s(dst + kWgWStage, asrc + (size_t)q * a.NT * kWSeg, abytes, &full[rp.slot]);
            ++s;
            rp.advance(nstage);
            if (++q == q1) {
                u += gridDim.x;
                start_unit(a, n_units);
            }
        }
        return true;
    }
};

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

    // the producer's cursor lives in shared memory: registers are the scarce resource of the consumer loop
    __shared__ WgProducer P;
    const bool producer = tid == 0;
    if (producer) {
        P.u = blockIdx.x;
        P.s = 0;
        P.rp = RingPos{};
        P.start_unit(a, n_units);
        if (!P.fill(a, n_units, nstage, smem, SB, full, empty, nstage)) set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
    }

    const int wr = warp >> 3, wt = warp & 7;
    const int g = lane >> 2, t = lane & 3;
    const int per = (a.tt_n8 + kWgTokGroups - 1) / kWgTokGroups;  // n8 tiles per warp
    RingPos rp;
    int s = 0;
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
        for (int q = w.q0; q < w.q1; ++q, ++s, rp.advance(nstage)) {
            // the stage this warp consumes next must be issued (a bounded wait only if the ring fell behind);
            // beyond it, issue into whatever slots the slowest warp has already released
            if (producer) {
                if (!P.fill(a, n_units, s + 1, smem, SB, full, empty, nstage))
                    set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
                else
                    P.fill(a, n_units, s + nstage, smem, SB, full, empty, nstage, false);
            }
            __syncwarp();
            if (!mbar_wait(&full[rp.slot], rp.phase)) {
                set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                return;
            }
            const uint32_t st = smem_u32(smem + (size_t)rp.slot * SB);
            if (nw > 0) {
                const uint32_t ab = st + kWgWStage + nb0 * kWSeg + lane * 8;
                const uint32_t mb = st + kWgWStage + nb0 * kWSeg + 1024 + t * 16;
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) {
                    // A fragments and scales of the four row-groups, unpacked once per block
                    const uint32_t seg = st + (wr * 4 + blk) * kTileBytes;
                    const uint4 lo = lds128(seg + lane * 16);
                    const uint4 hi = lds128(seg + 512 + lane * 16);
                    const uint4 sc = lds128(seg + 1024 + g * 16);
                    uint32_t A[4][4];
                    float2 wd[4];  // (row g, row g + 8) of row-group r
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const uint32_t wlo = pick4(lo, r), whi = pick4(hi, r);
                        A[r][0] = wlo & 0x0F0F0F0Fu;
                        A[r][1] = whi & 0x0F0F0F0Fu;
                        A[r][2] = (wlo >> 4) & 0x0F0F0F0Fu;
                        A[r][3] = (whi >> 4) & 0x0F0F0F0Fu;
                        wd[r] = h2x2f(pick4(sc, r));
                    }
                    uint2 bf[kWgMaxN8];
                    float2 xd[kWgMaxN8], off[kWgMaxN8];
                    int d[kWgMaxN8][4][4];
#pragma unroll
                    for (int n = 0; n < kWgMaxN8; ++n) {
                        if (n < nw) {
                            bf[n] = lds64(ab + n * kWSeg + blk * 256);
                            const uint4 mu = lds128(mb + n * kWSeg + blk * 64);
                            xd[n] = make_float2(__uint_as_float(mu.x), __uint_as_float(mu.y));
                            off[n] = make_float2(__uint_as_float(mu.z), __uint_as_float(mu.w));
#pragma unroll
                            for (int r = 0; r < 4; ++r)
                                mma_u8s8_pure(d[n][r], A[r][0], A[r][1], A[r][2], A[r][3], bf[n].x, bf[n].y);
                        }
                    }
#pragma unroll
                    for (int n = 0; n < kWgMaxN8; ++n) {
                        if (n < nw) {
#pragma unroll
                            for (int r = 0; r < 4; ++r) {
                                const float2 fL = __fadd2_rn(make_float2(__int_as_float(d[n][r][0]), __int_as_float(d[n][r][1])), off[n]);
                                const float2 fH = __fadd2_rn(make_float2(__int_as_float(d[n][r][2]), __int_as_float(d[n][r][3])), off[n]);
                                // (wd*xd) * (float)isum accumulated per block, as mistral/dequant.h:1085
                                const float2 sL = __fmul2_rn(make_float2(wd[r].x, wd[r].x), xd[n]);
                                const float2 sH = __fmul2_rn(make_float2(wd[r].y, wd[r].y), xd[n]);
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

// One thread per 4-byte word of the wide layout.
__global__ void k_wide_repack(const uint8_t* __restrict__ tiles, int n_rg, int nq, uint8_t* __restrict__ wide,
                              long long n_words) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_words;
         i += (long long)gridDim.x * blockDim.x) {
        const long long byte = i * 4;
        const long long seg_i = byte / kTileBytes;  // ((rt * nq + q) * 2 + hh) * 4 + bq
        const int off = (int)(byte - seg_i * kTileBytes);
        const int bq = (int)(seg_i & 3), hh = (int)((seg_i >> 2) & 1);
        const long long rq = seg_i >> 3;
        const int q = (int)(rq % nq);
        const long long rt = rq / nq;
        uint32_t v = 0;
        if (off < 1024) {
            // lane L's 16 bytes: word bq of row-groups 4hh .. 4hh+3 (tile16x4: half h, lane L at h*512 + L*16)
            const int h = off >> 9, L = (off & 511) >> 4, r = (off >> 2) & 3;
            const long long rg = rt * kWgRG + hh * 4 + r;
            if (rg < n_rg)
                v = *reinterpret_cast<const uint32_t*>(tiles + ((size_t)rg * nq + q) * kTileBytes + h * 512 + L * 16 + bq * 4);
        } else {
            // g's 16 bytes: (wd row g, wd row g + 8) of block bq for row-groups 4hh .. 4hh+3
            const int gg = (off - 1024) >> 4, r = ((off - 1024) >> 2) & 3;
            const long long rg = rt * kWgRG + hh * 4 + r;
            if (rg < n_rg) {
                const uint8_t* sc = tiles + ((size_t)rg * nq + q) * kTileBytes + 1024 + gg * 16;  // [g][h][blk] fp16
                const uint32_t lo = *reinterpret_cast<const uint16_t*>(sc + bq * 2);
                const uint32_t hi = *reinterpret_cast<const uint16_t*>(sc + 8 + bq * 2);
                v = lo | (hi << 16);
            }
        }
        reinterpret_cast<uint32_t*>(wide)[i] = v;
    }
}

cudaError_t launch_wide_repack(const uint8_t* tiles, int n_rg, int nq, uint8_t* wide, cudaStream_t st) {
    const long long n_rt = (n_rg + kWgRG - 1) / kWgRG;
    const long long n_words = n_rt * nq * kWgWStage / 4;
    long long grid = (n_words + 255) / 256;
    if (grid > 65536) grid = 65536;
    k_wide_repack<<<(int)grid, 256, 0, st>>>(tiles, n_rg, nq, wide, n_words);
    return cudaGetLastError();
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
