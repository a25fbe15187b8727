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
#include "sd_dev.cuh"

namespace sd {

namespace {

// Shared memory: weight ring | B fragments (+ zero pad) | C quads | activation scales |
//                partial-sum slots | SiLU unit | mbarriers
struct SmemLayout {
    size_t ring, act, red, ubuf, bars, total;
};

// Kp = the K range one CTA covers (K / kparts).
__host__ __device__ inline SmemLayout smem_layout(int Kp, int S, int chunk, int nstage) {
    SmemLayout L;
    const size_t nb = (size_t)Kp / 32;
    L.ring = 0;
    L.act = L.ring + (size_t)nstage * kRPW * chunk * kTileBytes;
    L.red = L.act + act_smem_bytes((int)nb);  // B fragments, C quads, scales (sd_dev.cuh)
    L.ubuf = L.red + (size_t)kRedSlots * kRPW * kConsumerWarps * 128 * 4;
    L.bars = L.ubuf + 4 * 128 * 4;
    L.total = L.bars + (2 * kMaxStages + 2 * kRedSlots) * 8;
    return L;
}

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
    float* red = reinterpret_cast<float*>(smem + L.red);
    float* ubuf = reinterpret_cast<float*>(smem + L.ubuf);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + kMaxStages;
    uint64_t* red_full = empty + kMaxStages;    // consumers -> epilogue (count: consumer warps)
    uint64_t* red_empty = red_full + kRedSlots; // epilogue -> consumers (count: epilogue warps)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
            RingPos rp;
            for (int s = 0; s < n_stages_total; ++s, rp.advance(nstage)) {
                const int slot = rp.slot;
                if (s >= nstage && !mbar_wait(&empty[slot], rp.phase ^ 1)) {
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
    const ActSmem A = act_smem_at(smem + L.act, nb);
    stage_act_from_planes(A, a.act, a.K, kb0, nb, S, nv, tid, nthr);
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
            if (!ab) reduce_partials(rr, chunk, lane, v);
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
                epi_qkv(v, rg, lane, nv, pos, a.q_out, a.k_cache, a.v_cache, a.q_rows, a.kv_rows, a.max_seq, a.head_dim,
                        a.theta_inv, a.q_scale);
            } else if constexpr (EPI == EPI_SILU_Q8) {
                // unit of 4 row-groups = 2 pairs: (gate lo, gate hi), (up lo, up hi)
                const int pair_in_unit = ((rg0 / kRPW) + pi) & 1;
#pragma unroll
                for (int k = 0; k < 4; ++k) ubuf[(pair_in_unit * 2 + r) * 128 + lane + 32 * k] = v[k];
                if (pair_in_unit == 1) {
                    named_sync(2, kEpiWarps * 32);
                    epi_silu_q8(ubuf, r, lane, rg >> 2, nv, a.h, a.hidden);
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
    RingPos rp;
    // A stage that never arrives (only possible if the producer gave up) marks the warp aborted: it
    // stops waiting and computing but keeps its place in every handshake, so no warp is left waiting
    // on one that returned.  Every stage issued before the give-up has been waited for, so no bulk
    // copy is in flight when the CTA exits.
    bool aborted = false;
    for (int pi = 0; pi < n_pairs; ++pi) {
        const int rg = rg0 + pi * kRPW;
        for (int ch = 0; ch < cpr; ++ch, rp.advance(nstage)) {
            const int slot = rp.slot;
            if (!aborted && !mbar_wait(&full[slot], rp.phase)) {
                set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                aborted = true;
            }
            if (aborted) continue;
            const uint8_t* slot_p = ring + (size_t)slot * stage_bytes;
            if (has_tile) {
                // tile registers are loaded before the slot is released
                TileRegs tr;
                load_tiles(slot_p, half_bytes, warp, lane, tr);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                consume_tiles<EPI == EPI_BLOCKSUMS>(tr, lane, A, S, (ch * chunk + warp) * 4, accL, accH, a.isum, rg,
                                                    a.out_rows, (size_t)(a.K >> 5), kb0);
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
        }
        if constexpr (EPI == EPI_BLOCKSUMS) continue;
        // ---- hand the pair's partials to the epilogue warps ----
        const int rs = pi % kRedSlots;
        if (pi >= kRedSlots && !aborted && !mbar_wait(&red_empty[rs], ((pi / kRedSlots) - 1) & 1)) {
            set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
            aborted = true;
        }
        if (has_tile && !aborted) write_partials(red + (size_t)rs * kRPW * kConsumerWarps * 128, warp, lane, accL, accH);
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
            *reinterpret_cast<uint2*>(tile + 1024 + gg * 16 + h * 8) = s2;
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
