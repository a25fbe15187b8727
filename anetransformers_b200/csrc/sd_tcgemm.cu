// sd_tcgemm.cu -- the wide-token W4A8 GEMM of the batched verify / prefill on the 5th-generation tensor
// cores: tcgen05.mma kind::i8 with the accumulators in tensor memory (TMEM).
//
// Same contract and arithmetic as k_wgemm (sd_wgemm.cu), which stays the path for narrow forwards:
//   Y[m][r] = sum_b (wd[r,b] * xd[m,b]) * isum[r,m,b],  isum = sum_j (q_j - 8) * x8_j
// (the reference's per-block SDOT sum and fp32 scale, mistral/dequant.h:1068-1087).  One MMA of M = 128
// weight rows x N tokens x K = 32 is exactly one Q4_0 block, so the int32 block sums come out of the tensor
// core exact and separate: each MMA overwrites its TMEM accumulator slot with sum(q * x) (q the 0..15 nibbles).
// The epilogue adds the bits of kMagic with one integer add, so the word reads as the fp32 value
// kMagic + sum(q * x), and then runs k_wgemm's three fp32 operations per element (one exact FADD of the
// image's offset, the scale product, the FMA into the running sum), block by block in K order.  Both GEMMs
// therefore give bit-identical outputs for the same K split.  (Presetting the slots to kMagic instead, by
// tcgen05.cp from shared memory, cost the MMA thread ~900 cycles per block and measured 16 % slower; 16
// epilogue warps of at most 32 columns instead of 8 of at most 64 measured 12 % slower.)
//
// Shapes.  A unit is (row tile of 128 rows, K slice, token tile of N <= 128 tokens); CTAs are persistent
// (one per SM) and walk units u = blockIdx.x, += gridDim.x, with the token tiles of a row tile adjacent so
// their weight reads meet in L2.  Per quad (4 blocks, 128 columns) a shared-memory stage holds:
//   W  9216 B   the row tile's quad in the wide layout (sd_batch.h), one bulk copy
//   X  N/8 x 1280 B   the token tile's segments of the activation image in the tensor-core arrangement
//                (sd_internal.h), one bulk copy; block bq of token group g: [kc][8 tokens][16 B] at
//                g * 1280 + bq * 256 -- the canonical K-major no-swizzle operand (8 x 16 B core matrices,
//                K-chunk stride 128 B, token-group stride 1280 B)
//   A  4 x 4096 B    the quad's weights unpacked to u8 nibbles, block bq: [kc][128 rows][16 B]
//                (K-chunk stride 2048 B, row-group stride 128 B)
// Warp roles (12 warps):
//   warp 0      lane 0 issues the bulk copies of each stage
//   warp 1      allocates the 512 TMEM columns; lane 0 issues the MMAs (4 accumulator slots of 128 columns)
//   warps 2-3   unpack each stage's nibbles into A (a generic-proxy write, fenced for the async proxy)
//   warps 4-11  epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (the tile's rows) and token columns
//               [c * N/2, (c + 1) * N/2), c = (w - 4) / 4; it keeps that row x column block's fp32 sums
//               in registers over the unit's blocks, releases each slot once it is read, and at the
//               end of the unit stores the K-slice partial (WG_STORE) or, for gate|up units, hands the gate
//               sums to the warp holding the matching up rows, which forms SiLU(g) * u and writes its Q8_0
//               block into the next image (WG_SILU).
// Every wait is an mbarrier wait bounded in time; a wait that runs out sets the context's error word, the
// kernel stops issuing work, waits (bounded) for its copies and MMAs in flight, frees its TMEM and returns.
#include "sd_dev.cuh"

namespace sd {

namespace {

constexpr int kTcWarps = 12;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcUnpackWarp0 = 2, kTcUnpackWarps = 2;
constexpr int kTcEpiWarp0 = 4, kTcEpiWarps = 8;
constexpr int kTcSlots = 4;                      // TMEM accumulator slots
constexpr int kTcSlotCols = 128;                 // columns per slot = tokens of a tile at most
constexpr uint32_t kTcCols = kTcSlots * kTcSlotCols;  // 512: the whole TMEM of the SM
constexpr int kTcABytes = kTcAStage;             // unpacked A tiles of a stage
constexpr int kTcPairs = 4;                      // (gate warp, up warp) pairs of a gate|up unit
constexpr int kTcXchgBytes = kTcPairs * 2 * 32 * 33 * 4;  // per pair: two halves of <= 32 token rows of 33 floats

// Shared-memory matrix descriptor of a K-major operand without swizzle: start address, leading byte offset
// (distance between the two 16-byte K chunks of a 32-byte K step) and stride byte offset (distance between
// groups of 8 rows), each in 16-byte units; bit 46 = descriptor version of sm_100.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::i8: D s32 (bits 4-5 = 2), A u8 (bits 7-9 = 0), B s8 (bits 10-12 = 1),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24 (M = 128).
__host__ __device__ constexpr uint32_t idesc_u8s8(int n) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] = A[smem] x B[smem] (u8 x s8 -> s32, the accumulator overwritten), issued by one thread.
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, 0, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc)
        : "memory");
}
// The mbarrier receives one arrival once every MMA this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 consecutive columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
// Wait for this thread's TMEM loads; the registers of the last load pass through the statement so that no
// use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&v)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                   "+r"(v[15]), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]),
                   "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]),
                   "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
                 :
                 : "memory");
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}

__device__ __forceinline__ uint32_t pick4u(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

struct TcUnit {
    int rt, kp, tt, q0, q1;
};

__device__ __forceinline__ TcUnit tc_unit(const WGemmArgs& a, int u) {
    TcUnit w;
    const int per_rt = a.kparts * a.n_tt;
    w.rt = u / per_rt;
    const int r2 = u - w.rt * per_rt;
    w.kp = r2 / a.n_tt;
    w.tt = r2 - w.kp * a.n_tt;
    w.q0 = (int)((long long)w.kp * a.nq / a.kparts);
    w.q1 = (int)((long long)(w.kp + 1) * a.nq / a.kparts);
    return w;
}

// Shared control block (after the stages and the gate exchange).
struct TcCtl {
    uint64_t full[kTcMaxStages];    // stage landed (1 arrival + transaction bytes)
    uint64_t aready[kTcMaxStages];  // stage's A unpacked (64 unpack threads)
    uint64_t sempty[kTcMaxStages];  // stage free again (MMA commit + 8 epilogue warps)
    uint64_t tfull[kTcSlots];       // accumulator slot holds a finished block (MMA commit)
    uint64_t tempty[kTcSlots];      // accumulator slot read (8 epilogue warps)
    uint64_t xg[kTcPairs];          // gate warp's hand-over written (32 lanes)
    uint64_t xu[kTcPairs];          // up warp's hand-over written (32 lanes)
    uint64_t xempty[kTcPairs];      // both warps of the pair done with the exchange rows (64 lanes)
    uint64_t done;                  // every MMA of the CTA has completed
    uint32_t tmem;                  // TMEM base address from tcgen05.alloc
    int abort;                      // a wait ran out: stop issuing work
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, TcCtl* ctl, int* err, int code) {
    if (*(volatile int*)&ctl->abort) return false;
    if (mbar_wait(bar, parity)) return true;
    set_dev_error(err, code);
    *(volatile int*)&ctl->abort = 1;
    return false;
}

}  // namespace

size_t tcgemm_smem_bytes(int tt_n8, int nstage, int epi) {
    return (size_t)nstage * ((size_t)kWgWStage + (size_t)tt_n8 * kWSeg + kTcABytes) +
           (epi == WG_SILU ? (size_t)kTcXchgBytes : 0) + sizeof(TcCtl) + 128;
}

// NG = 8-token groups per epilogue warp (N = 16 NG tokens per tile).
template <int EPI, int NG>
__global__ void __launch_bounds__(kTcThreads, 1) k_tcgemm(const WGemmArgs a) {
    static_assert(NG >= 1 && NG <= 8, "token groups per epilogue warp");
    constexpr int N = 16 * NG;     // tokens of a tile = MMA N
    constexpr int HALF = 8 * NG;   // columns per epilogue warp
    constexpr int NA = NG < 4 ? NG : 4, NB = NG - NA;  // groups in the first / second 32-column load
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nstage = a.nstage;
    const uint32_t SB = (uint32_t)a.stage_bytes;  // kWgWStage + tt_n8 * kWSeg + kTcABytes
    const uint32_t xoff = kWgWStage, aoff = kWgWStage + (uint32_t)a.tt_n8 * kWSeg;
    float* xchg = reinterpret_cast<float*>(smem + (size_t)nstage * SB);
    TcCtl* ctl = reinterpret_cast<TcCtl*>(smem + (size_t)nstage * SB + (EPI == WG_SILU ? kTcXchgBytes : 0));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_units = a.n_rt * a.kparts * a.n_tt;
    const uint32_t sbase = smem_u32(smem);

    if (tid == 0) {
        for (int i = 0; i < nstage; ++i) {
            mbar_init(&ctl->full[i], 1);
            mbar_init(&ctl->aready[i], kTcUnpackWarps * 32);
            mbar_init(&ctl->sempty[i], 1 + kTcEpiWarps);
        }
        for (int i = 0; i < kTcSlots; ++i) {
            mbar_init(&ctl->tfull[i], 1);
            mbar_init(&ctl->tempty[i], kTcEpiWarps);
        }
        for (int i = 0; i < kTcPairs; ++i) {
            mbar_init(&ctl->xg[i], 32);
            mbar_init(&ctl->xu[i], 32);
            mbar_init(&ctl->xempty[i], 64);
        }
        mbar_init(&ctl->done, 1);
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&ctl->tmem, kTcCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    pdl_trigger();
    pdl_wait();

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            RingPos rp;
            int issued = 0;
            uint32_t last_phase[kTcMaxStages];
            for (int u = blockIdx.x; u < n_units && !ctl->abort; u += gridDim.x) {
                const TcUnit w = tc_unit(a, u);
                const int n0 = w.tt * a.tt_n8, nn = min(a.tt_n8, a.NT - n0);
                const uint32_t abytes = (uint32_t)(nn * kWSeg);
                const uint8_t* wsrc = a.w + (size_t)w.rt * a.nq * kWgWStage;
                const uint8_t* asrc = a.act + (size_t)n0 * kWSeg;
                for (int q = w.q0; q < w.q1; ++q) {
                    if (issued >= nstage && !tc_wait(&ctl->sempty[rp.slot], rp.phase ^ 1, ctl, a.err, DEV_ERR_EMPTY_WAIT))
                        break;
                    uint8_t* dst = smem + (size_t)rp.slot * SB;
                    mbar_arrive_expect_tx(&ctl->full[rp.slot], (uint32_t)kWgWStage + abytes);
                    bulk_g2s(dst, wsrc + (size_t)q * kWgWStage, kWgWStage, &ctl->full[rp.slot]);
                    bulk_g2s(dst + xoff, asrc + (size_t)q * a.NT * kWSeg, abytes, &ctl->full[rp.slot]);
                    last_phase[rp.slot] = rp.phase;
                    ++issued;
                    rp.advance(nstage);
                }
            }
            // no copy may still be landing when the CTA exits
            for (int i = 0; i < nstage && i < issued; ++i) mbar_wait(&ctl->full[i], last_phase[i]);
        }
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            RingPos rp, ts;
            constexpr uint32_t idesc = idesc_u8s8(N);
            bool ok = true;
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
                const TcUnit w = tc_unit(a, u);
                for (int q = w.q0; q < w.q1 && ok; ++q) {
                    ok = tc_wait(&ctl->aready[rp.slot], rp.phase, ctl, a.err, DEV_ERR_FULL_WAIT) &&
                         tc_wait(&ctl->full[rp.slot], rp.phase, ctl, a.err, DEV_ERR_FULL_WAIT);
                    if (!ok) break;
                    const uint32_t st = sbase + rp.slot * SB;
#pragma unroll
                    for (int bq = 0; bq < 4; ++bq) {
                        if (!tc_wait(&ctl->tempty[ts.slot], ts.phase, ctl, a.err, DEV_ERR_EMPTY_WAIT)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = tmem + ts.slot * kTcSlotCols;
                        const uint64_t ad = kmajor_desc(st + aoff + bq * 4096, 2048, 128);
                        const uint64_t bd = kmajor_desc(st + xoff + bq * 256, 128, kWSeg);
                        tc_mma(d, ad, bd, idesc);
                        tc_commit(&ctl->tfull[ts.slot]);
                        ts.advance(kTcSlots);
                    }
                    tc_commit(&ctl->sempty[rp.slot]);
                    rp.advance(nstage);
                }
            }
            // every MMA issued above has completed before TMEM is released
            tc_commit(&ctl->done);
            if (!mbar_wait(&ctl->done, 0)) set_dev_error(a.err, DEV_ERR_FULL_WAIT);
        }
        __syncwarp();
    } else if (warp < kTcEpiWarp0) {
        // ---------------- nibble unpack ----------------
        // lane L = 4g + t of combo (hh, bq, high): the wide layout's 16 bytes at L hold word t of rows
        // 16r + 8high + g (r = 0..3) of half hh; the low nibbles are K chunk 0 of those rows (elements 4t..4t+3),
        // the high nibbles K chunk 1 (elements 16+4t..).  Stores are bank-conflict free (bank = L).
        const int uw = warp - kTcUnpackWarp0;
        const int g = lane >> 2, t = lane & 3;
        RingPos rp;
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const TcUnit w = tc_unit(a, u);
            for (int q = w.q0; q < w.q1; ++q) {
                if (!tc_wait(&ctl->full[rp.slot], rp.phase, ctl, a.err, DEV_ERR_FULL_WAIT)) {
                    ok = false;
                    break;
                }
                const uint32_t st = sbase + rp.slot * SB;
#pragma unroll
                for (int i = 0; i < 16 / kTcUnpackWarps; ++i) {
                    const int c = uw + i * kTcUnpackWarps;
                    const int hh = c >> 3, bq = (c >> 1) & 3, high = c & 1;
                    const uint4 v = lds128(st + (hh * 4 + bq) * 1152 + high * 512 + lane * 16);
                    const uint32_t ab = st + aoff + bq * 4096 + t * 4;
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int R = hh * 64 + r * 16 + high * 8 + g;
                        const uint32_t wv = pick4u(v, r);
                        sts32(ab + R * 16, wv & 0x0F0F0F0Fu);
                        sts32(ab + 2048 + R * 16, (wv >> 4) & 0x0F0F0F0Fu);
                    }
                }
                fence_async_smem();
                mbar_arrive(&ctl->aready[rp.slot]);
                rp.advance(nstage);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - kTcEpiWarp0;
        const int quarter = warp & 3;          // TMEM lanes 32 quarter .. +31 = tile rows
        const int ch = ew >> 2;                // column half
        const int col0 = ch * HALF;
        const int R = quarter * 32 + lane;     // tile row of this thread
        // wide-layout scale of row R: half hh, row-group r, high, g
        const int hh = R >> 6, rr = (R >> 4) & 3, hi8 = (R >> 3) & 1, gg = R & 7;
        const uint32_t wd_off = 1024 + gg * 16 + rr * 4 + hi8 * 2;
        const uint32_t tlane = (uint32_t)(quarter * 32) << 16;
        // the slots start free
        __syncwarp();
        if (lane == 0)
            for (int s = 0; s < kTcSlots; ++s) mbar_arrive(&ctl->tempty[s]);
        RingPos rp, ts;
        bool ok = true;
        int unit_i = 0;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++unit_i) {
            const TcUnit w = tc_unit(a, u);
            float2 acc[4 * NG];
#pragma unroll
            for (int i = 0; i < 4 * NG; ++i) acc[i] = make_float2(0.f, 0.f);
            for (int q = w.q0; q < w.q1 && ok; ++q) {
                if (!tc_wait(&ctl->full[rp.slot], rp.phase, ctl, a.err, DEV_ERR_FULL_WAIT)) {
                    ok = false;
                    break;
                }
                const uint32_t st = sbase + rp.slot * SB;
#pragma unroll 1
                for (int bq = 0; bq < 4; ++bq) {
                    if (!tc_wait(&ctl->tfull[ts.slot], ts.phase, ctl, a.err, DEV_ERR_FULL_WAIT)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ta = tmem + tlane + ts.slot * kTcSlotCols + col0;
                    const float wd = __half2float(__ushort_as_half((unsigned short)lds_u16(st + (hh * 4 + bq) * 1152 + wd_off)));
                    const float2 wd2 = make_float2(wd, wd);
                    const uint32_t mb = st + xoff + (col0 >> 3) * kWSeg + 1024 + bq * 64;
                    // as k_wgemm: exact block sum, then (wd*xd) * isum accumulated per block
                    auto group = [&](int gi, const uint32_t(&v)[32]) {
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const uint4 mu = lds128(mb + gi * kWSeg + t * 16);
                            const float2 xd = make_float2(__uint_as_float(mu.x), __uint_as_float(mu.y));
                            const float2 off = make_float2(__uint_as_float(mu.z), __uint_as_float(mu.w));
                            const int j = (gi & 3) * 8 + 2 * t;
                            // the bits of kMagic + sum(q * x): exact while |sum| < 2^22 (|sum| <= 32 * 15 * 128)
                            const float2 f = __fadd2_rn(make_float2(__uint_as_float(v[j] + (uint32_t)kMagicI),
                                                                    __uint_as_float(v[j + 1] + (uint32_t)kMagicI)), off);
                            const float2 sc = __fmul2_rn(wd2, xd);
                            acc[gi * 4 + t] = __ffma2_rn(sc, f, acc[gi * 4 + t]);
                        }
                    };
                    // columns col0 .. col0 + 63 stay inside the slot (col0 + 64 <= HALF + 64 <= 128)
                    uint32_t va[32];
                    tmem_ld32(ta, va);
                    tmem_wait_ld(va);
                    if constexpr (NB > 0) {
                        uint32_t vb[32];
                        tmem_ld32(ta + 32, vb);
#pragma unroll
                        for (int gi = 0; gi < NA; ++gi) group(gi, va);
                        tmem_wait_ld(vb);
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&ctl->tempty[ts.slot]);
#pragma unroll
                        for (int gi = NA; gi < NG; ++gi) group(gi, vb);
                    } else {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&ctl->tempty[ts.slot]);
#pragma unroll
                        for (int gi = 0; gi < NA; ++gi) group(gi, va);
                    }
                    ts.advance(kTcSlots);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->sempty[rp.slot]);
                rp.advance(nstage);
            }
            if (!ok) break;
            const int n0 = w.tt * N;  // first token of the tile
            if constexpr (EPI == WG_STORE) {
                const int row = w.rt * 128 + R;
                if (row < a.out_rows) {
                    float* out = a.out + (size_t)w.kp * a.part_stride + row;
#pragma unroll
                    for (int i = 0; i < 4 * NG; ++i) {
                        const int m = n0 + col0 + 2 * i;
                        if (m < a.M) out[(size_t)m * a.ld] = acc[i].x;
                        if (m + 1 < a.M) out[(size_t)(m + 1) * a.ld] = acc[i].y;
                    }
                }
            } else {
                // Gate rows of hidden block hb sit in quarter 2p (p = 0, 1), its up rows in quarter 2p + 1; lane j is
                // hidden unit 32 hb + j in both.  The pair splits the warp's tokens: the gate warp finishes the
                // first half, the up warp the second.  Each hands the other the sums it needs through shared
                // memory (rows of 33 floats: conflict-free by lane in both directions), forms h = SiLU(g) * u for
                // its half with lane = hidden unit, then quantises it with lane = token (one Q8_0 block per lane).
                constexpr int HT = HALF / 2;  // tokens per warp of the pair (<= 32)
                const int pair = (quarter >> 1) + 2 * ch;
                const int hb = w.rt * 2 + (quarter >> 1);
                const bool gate = (quarter & 1) == 0;
                float* bufA = xchg + pair * (2 * 32 * 33);  // first-half tokens: up sums, then h (gate warp)
                float* bufB = bufA + 32 * 33;               // second-half tokens: gate sums, then h (up warp)
                if (unit_i > 0 && !tc_wait(&ctl->xempty[pair], (unit_i - 1) & 1, ctl, a.err, DEV_ERR_FULL_WAIT)) break;
                float* mine = gate ? bufA : bufB;   // the half this warp finishes
                float* other = gate ? bufB : bufA;  // the half the partner finishes
                // acc pairs [0, HT/2) hold the first-half tokens, [HT/2, HT) the second half (indices stay
                // compile-time constants so that acc lives in registers)
#pragma unroll
                for (int i = 0; i < HT / 2; ++i) {
                    const float2 ov = gate ? acc[HT / 2 + i] : acc[i];
                    other[(2 * i) * 33 + lane] = ov.x;
                    other[(2 * i + 1) * 33 + lane] = ov.y;
                }
                mbar_arrive(gate ? &ctl->xg[pair] : &ctl->xu[pair]);
                if (!tc_wait(gate ? &ctl->xu[pair] : &ctl->xg[pair], unit_i & 1, ctl, a.err, DEV_ERR_FULL_WAIT)) break;
#pragma unroll
                for (int i = 0; i < HT / 2; ++i) {
                    const float2 mv = gate ? acc[i] : acc[HT / 2 + i];
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const float own = k ? mv.y : mv.x;
                        const float par = mine[(2 * i + k) * 33 + lane];
                        const float gv = gate ? own : par, uv = gate ? par : own;
                        // SiLU(g) * u (mistral/mistral_model.h:174-199), as the matvec epilogue computes it
                        const float e = expf(-gv);
                        const float sig = 1.0f / (1.0f + e);
                        mine[(2 * i + k) * 33 + lane] = (gv * sig) * uv;
                    }
                }
                __syncwarp();
                if (lane < HT) {
                    // Q8_0 of token lane's 32 values (mistral/dequant.h:545-599, as q8_quant_lane)
                    const float* hrow = mine + lane * 33;
                    float amax = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(hrow[j]));
                    const float d = __fdiv_rn(amax, 127.0f);
                    const float id = amax != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                    const int m = n0 + col0 + (gate ? 0 : HT) + lane;
                    int sum = 0;
                    uint32_t words[8];
#pragma unroll
                    for (int wq = 0; wq < 8; ++wq) {
                        uint32_t wv = 0;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            int q = 0;
                            if (amax != 0.0f) {
                                const int r = __float2int_rn(__fmul_rn(hrow[wq * 4 + k], id));
                                q = r > 127 ? 127 : (r < -128 ? -128 : r);
                            }
                            sum += q;
                            wv |= (uint32_t)(q & 0xFF) << (8 * k);
                        }
                        words[wq] = wv;
                    }
                    if (hb < (a.hidden >> 5) && m < a.M) {
#pragma unroll
                        for (int wq = 0; wq < 8; ++wq) wimg_put_word(a.h, m, hb, wq, words[wq]);
                        wimg_put_meta(a.h, m, hb, d, sum);
                    }
                }
                mbar_arrive(&ctl->xempty[pair]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTcCols);
}

template <int EPI, int NG>
cudaError_t tc_attr(int max_smem) {
    return cudaFuncSetAttribute(k_tcgemm<EPI, NG>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

template <int EPI>
cudaError_t tc_attrs(int max_smem) {
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = tc_attr<EPI, 1>(max_smem);
    if (e == cudaSuccess) e = tc_attr<EPI, 2>(max_smem);
    if (e == cudaSuccess) e = tc_attr<EPI, 3>(max_smem);
    if (e == cudaSuccess) e = tc_attr<EPI, 4>(max_smem);
    if (e == cudaSuccess) e = tc_attr<EPI, 5>(max_smem);
    if (e == cudaSuccess) e = tc_attr<EPI, 6>(max_smem);
    if (e == cudaSuccess) e = tc_attr<EPI, 7>(max_smem);
    if (e == cudaSuccess) e = tc_attr<EPI, 8>(max_smem);
    return e;
}

template <int EPI>
void tc_launch(int ng, const WGemmArgs& a, int grid, size_t smem, cudaStream_t st) {
    switch (ng) {
        case 1: k_tcgemm<EPI, 1><<<grid, kTcThreads, smem, st>>>(a); break;
        case 2: k_tcgemm<EPI, 2><<<grid, kTcThreads, smem, st>>>(a); break;
        case 3: k_tcgemm<EPI, 3><<<grid, kTcThreads, smem, st>>>(a); break;
        case 4: k_tcgemm<EPI, 4><<<grid, kTcThreads, smem, st>>>(a); break;
        case 5: k_tcgemm<EPI, 5><<<grid, kTcThreads, smem, st>>>(a); break;
        case 6: k_tcgemm<EPI, 6><<<grid, kTcThreads, smem, st>>>(a); break;
        case 7: k_tcgemm<EPI, 7><<<grid, kTcThreads, smem, st>>>(a); break;
        default: k_tcgemm<EPI, 8><<<grid, kTcThreads, smem, st>>>(a); break;
    }
}

cudaError_t tcgemm_init_attrs(int max_smem) {
    cudaError_t e = tc_attrs<WG_STORE>(max_smem);
    return e == cudaSuccess ? tc_attrs<WG_SILU>(max_smem) : e;
}

cudaError_t launch_tcgemm(int epi, const WGemmArgs& a, int grid, size_t smem, cudaStream_t st) {
    // the tile width is a whole number of 16-token MMA columns: tt_n8 even, 2..kTcMaxTT
    if (a.tt_n8 < 2 || a.tt_n8 > kTcMaxTT || (a.tt_n8 & 1)) return cudaErrorInvalidValue;
    if (epi == WG_SILU)
        tc_launch<WG_SILU>(a.tt_n8 / 2, a, grid, smem, st);
    else
        tc_launch<WG_STORE>(a.tt_n8 / 2, a, grid, smem, st);
    return cudaGetLastError();
}

}  // namespace sd
