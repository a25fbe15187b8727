// sd_fwd.cu -- the whole forward of S <= 8 tokens (decode step or S = K+1 verify) as one persistent
// kernel: one CTA per SM, launched cooperatively so that every CTA is resident and grid-wide barriers
// are safe.
//
// Replaces the per-layer kernel sequence of the reference's batched forward (mistral/mistral_infer.m:
// 103-179 driving mistral/mistral_model.h:490-560): embedding, RMSNorm + Q8_0, fused QKV matvec with
// RoPE and the KV-ring write, 4:1 GQA attention, o-proj + residual, RMSNorm + Q8_0, gate|up matvec with
// SiLU and Q8_0, down projection + residual, final norm and LM head.
//
// Why one kernel: at S <= 8 every matvec streams its weights once and does little math, so a forward
// is a ~3.9 GB weight stream interrupted by small latency-bound steps.  Here a producer warp per CTA
// streams the weight tiles of every matvec of the forward, in order, through a shared-memory ring (1-D
// bulk copies, no multicast); weights do not depend on activations, so the ring keeps filling with the
// next matvec's tiles while the CTA waits in a grid barrier, runs attention or normalises.
//
// Warp roles (608 threads): warps 0-15 consume tiles (int8 MMA), 16-17 reduce the 16 partials of a
// row-group and apply the epilogue, 18 is the producer.  Warps 0-17 also run the non-matvec phases.
//
// Phases of a layer, each ended by a grid barrier:
//   QKV    Q8_0 planes of x*w (written by the phase that produced x) staged with the RMSNorm scale;
//          matvec, RoPE, KV write
//   ATTN   (kv head, chunk) partials, two 128-thread groups per CTA
//   COMB   merge of the chunk partials and Q8_0 of the head outputs
//   WO     matvec, outputs to slice buffers
//   RED    warp per (token, 32-row block): x += slices, 16-row sums of squares, Q8_0 of x*w for the
//          next norm
//   W13    gate|up matvec, SiLU(gate)*up, Q8_0
//   W2     K-split matvec, outputs to slice buffers
//   RED    as above
// then the LM head.  The kernel is driven by this phase table with one call site per phase kind, so
// its code stays small enough for the instruction cache.  The arithmetic (tile math, reduction orders,
// norms, attention) is the same device code as the per-op kernels, so both paths give bit-identical
// logits.
#include "sd_dev.cuh"
#include "sd_fwd.h"

namespace sd {

namespace {

constexpr int kComputeWarps = kConsumerWarps + kEpiWarps;   // 18
constexpr int kComputeThreads = kComputeWarps * 32;         // 576
constexpr int kConsumerThreads = kConsumerWarps * 32;       // 512
constexpr int kProducerWarp = kComputeWarps;
constexpr int kMaxChunk = 16;
constexpr uint32_t kStageBytes = kRPW * kMaxChunk * kTileBytes;  // 36864
constexpr int kActMaxNb = 128;                                   // K slice <= 4096 columns

// named barrier ids: 0 = __syncthreads, 1 = compute warps, 2 = the two epilogue warps,
// 3 = consumer warps (staging), 4.. = attention groups
constexpr int kBarCompute = 1, kBarEpi = 2, kBarStage = 3, kBarAttn0 = 4;

struct FwdSmem {
    size_t ring, act, red, ubuf, misc, bars, total;
};

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline FwdSmem fwd_layout(int nstage) {
    FwdSmem L{};
    L.ring = 0;
    L.act = L.ring + (size_t)nstage * kStageBytes;
    const size_t act_bytes = act_smem_bytes(kActMaxNb);
    const size_t red_bytes = (size_t)kRedSlots * kRPW * kConsumerWarps * 128 * 4;
    L.red = L.act + align_up(act_bytes, 128);
    L.ubuf = L.red + red_bytes;
    size_t uni = (L.ubuf + 4 * 128 * 4) - L.act;
    const size_t attn = (size_t)kFwdAttnGroups * attn_smem_bytes();
    if (attn > uni) uni = attn;
    L.misc = L.act + align_up(uni, 128);
    L.bars = L.misc + 128;  // misc: scale[kMaxS], abort, producer issued/done, argmax keys
    L.total = L.bars + (2 * kMaxStages + 2 * kRedSlots + 1) * 8;
    return L;
}

struct Misc {
    float scale[kMaxS];
    int abort;
    int grid_ok;
    uint32_t issued;
    int pdone;
    uint32_t act_issued;  // activation stagings issued (bulk copies completing on the act barrier)
    unsigned long long best[kMaxS];  // LM head: this CTA's best (logit, row) key per token
};
static_assert(sizeof(Misc) <= 128, "Misc fits its 128-byte slot");

struct Ring {
    uint64_t* act_full;  // activation staging copies
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    uint64_t* red_full;
    uint64_t* red_empty;
    float* red;
    float* ubuf;
    int nstage;
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const unsigned* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Single-thread wait that also gives up as soon as another warp of the CTA has aborted.
__device__ __forceinline__ bool wait_or_abort_1(uint64_t* bar, uint32_t parity, const volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag || global_ns() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// Whole-warp form: every lane waits (each lane then sees the data the phase guards) and the result
// is made warp-uniform, so the warp never diverges on a give-up.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const volatile int* abort_flag) {
    const bool ok = wait_or_abort_1(bar, parity, abort_flag);
    return __all_sync(0xffffffffu, ok);
}

struct Items {
    int i0, i1;
};

__device__ __forceinline__ Items my_items(const MvPhase& p) {
    const int n = p.n_units * p.kparts, G = gridDim.x, c = blockIdx.x;
    return Items{(int)((long long)c * n / G), (int)((long long)(c + 1) * n / G)};
}

// Grid barrier of the compute warps (CTA-wide arrive by thread 0, as cooperative groups do).  A CTA
// that has aborted stops synchronising; the others then run out their bounded wait and abort too.
__device__ void grid_barrier(const FwdArgs& a, Misc* m, uint32_t& target) {
    named_sync(kBarCompute, kComputeThreads);
    if (threadIdx.x == 0) {
        target += gridDim.x;
        volatile int* ab = &m->abort;
        if (!*ab) {
            // release: this CTA's writes (ordered before by the CTA barrier) are visible to a CTA that
            // acquires the count; the acquiring load does the same for the others' writes
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&a.sync[0]) : "memory");
            if (ld_acquire_u32(&a.sync[0]) < target) {
                const uint64_t t0 = global_ns();
                while (ld_acquire_u32(&a.sync[0]) < target) {
                    if (global_ns() - t0 > kWaitLimitNs) {
                        set_dev_error(a.err, DEV_ERR_PEER_WAIT);
                        *ab = 1;
                        break;
                    }
                }
            }
        }
    }
    named_sync(kBarCompute, kComputeThreads);
}

// ---------------------------------------------------------------------------------------------
// Activation staging (consumer warps only)
// ---------------------------------------------------------------------------------------------

// Stage blocks [kb0, kb0 + nb) of an activation image into A (consumer warps): two bulk copies on the
// act barrier.  While they land, warps < nv form the RMSNorm scale s of their token from the 16-row sums of
// squares (norm phases only).  Then, for norm phases, the block scales of tokens < nv become d_u * s -- the
// same values the per-op staging builds from Q8 planes.  Token slots >= nv keep whatever an earlier forward
// left there: each MMA output column depends only on its own token's fragments, and no epilogue reads the
// columns of tokens >= nv (clearing them cost 3 % of a forward).
__device__ void stage_image(const FwdArgs& a, const ActImage& im, const ActSmem& A, const Ring& R, Misc* m, uint32_t& nstg,
                            int kb0, int nb, int nv, bool norm, bool& ab, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        // the image was written by ordinary stores of other CTAs (ordered before us by a grid barrier);
        // order those with this thread's async-proxy reads
        asm volatile("fence.proxy.async.global;" ::: "memory");
        const uint32_t bb = (uint32_t)nb * kActStride * 8, mb = (uint32_t)nb * 64;
        mbar_arrive_expect_tx(R.act_full, bb + mb);
        bulk_g2s(A.b, im.b + (size_t)kb0 * kActStride, bb, R.act_full);
        bulk_g2s(A.m, im.m + (size_t)kb0 * 4, mb, R.act_full);
        reinterpret_cast<volatile uint32_t*>(&m->act_issued)[0] = nstg + 1;
    }
    if (norm && warp < nv) {
        const int ngroups = a.dim >> 4;
        const float tot = row_sumsq(a.ssq + (size_t)warp * ngroups, ngroups, lane);
        if (lane == 0) m->scale[warp] = rms_scale(tot, a.dim, a.eps);
    }
    named_sync(kBarStage, kConsumerThreads);
    if (!ab && !wait_or_abort(R.act_full, nstg & 1, &m->abort)) {
        set_dev_error(a.err, DEV_ERR_FULL_WAIT);
        ab = true;
        m->abort = 1;
    }
    ++nstg;
    if (norm)
        for (int i = tid; i < nb * 4; i += kConsumerThreads) {
            float* mp = reinterpret_cast<float*>(&A.m[i]);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int s = 2 * (i & 3) + hh;
                if (s < nv) mp[hh] = mp[hh] * m->scale[s];
            }
        }
}

// ---------------------------------------------------------------------------------------------
// Phase kinds
// ---------------------------------------------------------------------------------------------
enum PhaseKind : int { PH_QKV = 0, PH_WO = 1, PH_W13 = 2, PH_W2 = 3, PH_LM = 4 };
constexpr int kMaxParts = 8;  // K slices of a matvec whose outputs a residual phase adds
constexpr int kGather = 8;    // (rank, slice) values a reduction lane loads before adding


// Argmax key of logit v at row `row`: larger keys for larger logits, and for equal logits for the smaller
// row (first index on ties, mistral/mistral_model.h:1136-1143).
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
    const uint32_t b = __float_as_uint(v);
    const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)row);
}

// Finish one (token s, 32-row block b) of the residual stream, one warp, lane = row: store the new x
// value xv, the block's two 16-row sums of squares (the canonical order of group16_sumsq), and Q8_0 of
// u = x*wn for the next RMSNorm (wn its weight; the norm scale is applied when the image is staged).
__device__ __forceinline__ void finish_block(const FwdArgs& a, int s, int b, float xv, float w, int lane) {
    a.x[(size_t)s * a.dim + b * 32 + lane] = xv;
    const int gb = lane & 16, j = lane & 3;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float e = __shfl_sync(0xffffffffu, xv, gb + 4 * k + j);
        q = fmaf(e, e, q);
    }
    q += __shfl_xor_sync(0xffffffffu, q, 1);
    q += __shfl_xor_sync(0xffffffffu, q, 2);
    if ((lane & 15) == 0) a.ssq[(size_t)s * (a.dim >> 4) + 2 * b + (lane >> 4)] = q;
    float d;
    int sum;
    const int code = q8_quant_lane(xv * w, &d, &sum);
    image_put_codes_lane(a.un_img, s, b, lane, code);
    if (lane == 0) image_put_meta(a.un_img, s, b, d, sum);
}

// Residual update of one (token, block): x += the matvec's slice outputs, added in slice order as the
// per-op norm kernel adds them.
// With tensor parallelism the slices of every rank are added, rank by rank (each rank's own memory, read
// over NVLink), as the per-op norm kernel adds them.
__device__ void red_block(const FwdArgs& a, const float* const* ysrc, int nsrc, int s, int b, int kparts, const float* wn,
                          int lane) {
    const int row = b * 32 + lane;
    const float xv = a.x[(size_t)s * a.dim + row];
    const float w = wn[row];
    const size_t off = (size_t)s * a.dim + row;
    float t = 0.f;
    const int nl = nsrc * kparts;
    if (nl <= kGather) {
        // every (rank, slice) value requested before the first add: one NVLink round trip per reduction instead
        // of one per rank; the adds keep the rank-major, slice-minor order
        float yv[kGather];
#pragma unroll
        for (int i = 0; i < kGather; ++i) {
            const int r = i / kparts, p = i - r * kparts;
            yv[i] = i < nl ? __ldcg(ysrc[r] + (size_t)p * a.ypart_stride + off) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kGather; ++i)
            if (i < nl) t += yv[i];
    } else {
        for (int r = 0; r < nsrc; ++r) {
            float yv[kMaxParts];
#pragma unroll
            for (int p = 0; p < kMaxParts; ++p) yv[p] = p < kparts ? __ldcg(ysrc[r] + (size_t)p * a.ypart_stride + off) : 0.f;
#pragma unroll
            for (int p = 0; p < kMaxParts; ++p)
                if (p < kparts) t += yv[p];
        }
    }
    finish_block(a, s, b, xv + t, w, lane);
}

__device__ __forceinline__ AttnArgs attn_args(const FwdArgs& a, int l, int pos) {
    AttnArgs aa{};
    aa.q = a.q;
    aa.q_ld = a.q_rows;
    aa.k = a.k_cache + (size_t)l * a.kv_layer;
    aa.v = a.v_cache + (size_t)l * a.kv_layer;
    aa.kv_ld = a.kv_rows;
    aa.n_heads = a.n_heads;
    aa.n_kvh = a.n_kvh;
    aa.S = a.S;
    aa.pos = pos;
    aa.max_seq = a.max_seq;
    aa.chunk = a.attn_chunk;
    aa.max_chunks = a.max_chunks;
    aa.part_ml = a.part_ml;
    aa.part_acc = a.part_acc;
    aa.out = a.attn;
    aa.img = a.attn_img;
    aa.out_f32 = nullptr;
    aa.ctrl = nullptr;
    return aa;
}

// One matvec phase for the compute warps (consumer and epilogue roles).  kind is a runtime value so that
// the tile loop exists once in the kernel.
__device__ __forceinline__ void mv_phase(const FwdArgs& a, int kind, int layer, const Ring& R, Misc* m, RingPos& rp,
                                      uint32_t& pidx, uint32_t& nstg, bool& ab, int nv, int pos, int tid) {
    const MvPhase& p = kind == PH_QKV ? a.qkv : kind == PH_WO ? a.wo : kind == PH_W13 ? a.w13 : kind == PH_W2 ? a.w2 : a.lmp;
    const int warp = tid >> 5, lane = tid & 31;
    const Items it = my_items(p);
    const int nq_p = p.nq / p.kparts, cpr = nq_p / p.chunk, pairs = p.rpu / kRPW;
    const int nb = nq_p * 4;
    const uint32_t half = (uint32_t)p.chunk * kTileBytes;
    const ActSmem A = act_smem_at(R.ring + (size_t)R.nstage * kStageBytes, nb);
    const volatile int* abort_flag = &m->abort;

    if (warp < kConsumerWarps) {
        // ============================ consumers ============================
        int cur_part = -1;
        const bool has_tile = warp < p.chunk;
        for (int i = it.i0; i < it.i1; ++i) {
            const int part = i / p.n_units, unit = i % p.n_units;
            if (part != cur_part) {
                named_sync(kBarStage, kConsumerThreads);  // every consumer is done with the previous slice
                const ActImage& im = kind == PH_WO ? a.attn_img : kind == PH_W2 ? a.h_img : a.un_img;
                stage_image(a, im, A, R, m, nstg, part * nb, nb, nv, kind != PH_WO && kind != PH_W2, ab, tid);
                named_sync(kBarStage, kConsumerThreads);
                cur_part = part;
            }
            float2 accL[kRPW], accH[kRPW];
            for (int pr = 0; pr < pairs; ++pr) {
                const int rg = unit * p.rpu + pr * kRPW;
#pragma unroll
                for (int r = 0; r < kRPW; ++r) accL[r] = accH[r] = make_float2(0.f, 0.f);
                for (int ch = 0; ch < cpr; ++ch, rp.advance(R.nstage)) {
                    const int slot = rp.slot;
                    if (!ab && !wait_or_abort(&R.full[slot], rp.phase, abort_flag)) {
                        set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                        ab = true;
                        m->abort = 1;
                    }
                    if (ab) continue;  // an aborted warp releases nothing more (see the drain)
                    if (has_tile) {
                        TileRegs tr;
                        load_tiles(R.ring + (size_t)slot * kStageBytes, half, warp, lane, tr);
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&R.empty[slot]);
                        consume_tiles<false>(tr, lane, A, a.S, (ch * p.chunk + warp) * 4, accL, accH, nullptr, rg, 0,
                                             0, 0);
                    } else {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&R.empty[slot]);
                    }
                }
                const int rs = pidx % kRedSlots;
                if (pidx >= kRedSlots && !ab &&
                    !wait_or_abort(&R.red_empty[rs], ((pidx / kRedSlots) - 1) & 1, abort_flag)) {
                    set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
                    ab = true;
                    m->abort = 1;
                }
                ++pidx;
                if (ab) continue;
                if (has_tile) write_partials(R.red + (size_t)rs * kRPW * kConsumerWarps * 128, warp, lane, accL, accH);
                __syncwarp();
                if (lane == 0) mbar_arrive(&R.red_full[rs]);
            }
        }
        return;
    }

    // ============================ epilogue warps ============================
    const int r = warp - kConsumerWarps;
    for (int i = it.i0; i < it.i1; ++i) {
        const int part = i / p.n_units, unit = i % p.n_units;
        for (int pr = 0; pr < pairs; ++pr, ++pidx) {
            const int slot = pidx % kRedSlots;
            if (!ab && !wait_or_abort(&R.red_full[slot], (pidx / kRedSlots) & 1, abort_flag)) {
                set_dev_error(a.err, DEV_ERR_FULL_WAIT);
                ab = true;
                m->abort = 1;
            }
            const int rg = unit * p.rpu + pr * kRPW + r;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (!ab) {
                reduce_partials(R.red + ((size_t)slot * kRPW + r) * kConsumerWarps * 128, p.chunk, lane, v);
                __syncwarp();
                if (lane == 0) mbar_arrive(&R.red_empty[slot]);
            }
            if (kind == PH_W13) {
                // unit of 4 row-groups = 2 pairs: (gate lo, gate hi), (up lo, up hi)
#pragma unroll
                for (int k = 0; k < 4; ++k) R.ubuf[(pr * 2 + r) * 128 + lane + 32 * k] = v[k];
                if (pr == 1) {
                    named_sync(kBarEpi, kEpiWarps * 32);
                    if (!ab) epi_silu_q8(R.ubuf, r, lane, unit, nv, a.h, a.hidden, &a.h_img);
                    named_sync(kBarEpi, kEpiWarps * 32);
                }
            } else if (kind == PH_WO && p.kparts == 1 && a.tp.n <= 1) {
                // the pair is one 32-row block (unit): finish it here for every token, warp r taking
                // tokens r, r + 2, ... (lane = row); x and the norm weight are loaded up front
#pragma unroll
                for (int k = 0; k < 4; ++k) R.ubuf[r * 128 + lane + 32 * k] = v[k];
                const int row = unit * 32 + lane;
                const float w = a.layers[layer].rms_ffn[row];
                float xo[kMaxS / 2];
#pragma unroll
                for (int q = 0; q < kMaxS / 2; ++q) {
                    const int s = r + 2 * q;
                    xo[q] = s < nv ? a.x[(size_t)s * a.dim + row] : 0.f;
                }
                named_sync(kBarEpi, kEpiWarps * 32);
                if (!ab) {
#pragma unroll
                    for (int q = 0; q < kMaxS / 2; ++q) {
                        const int s = r + 2 * q;
                        if (s >= nv) break;
                        const float y = R.ubuf[(lane >> 4) * 128 + (lane & 15) * 8 + s];
                        finish_block(a, s, unit, xo[q] + (0.f + y), w, lane);
                    }
                }
                named_sync(kBarEpi, kEpiWarps * 32);  // ubuf free again
            } else if (ab) {
                continue;
            } else if (kind == PH_QKV) {
                epi_qkv(v, rg, lane, nv, pos, a.q, a.k_cache + (size_t)layer * a.kv_layer,
                        a.v_cache + (size_t)layer * a.kv_layer, a.q_rows, a.kv_rows, a.max_seq, a.head_dim, a.theta_inv,
                        a.q_scale);
            } else {
                // WO / W2: this slice's outputs (the residual add runs in the following phase); LM: logits
                float* ybase = a.yparts;
                if (a.tp.n > 1) ybase = a.tp.y[a.tp.rank] + (size_t)(((2 * layer + (kind == PH_W2)) + 1) & 1) * a.tp.buf;
                float* out = kind == PH_LM ? a.logits : ybase + (size_t)part * a.ypart_stride;
                const int ld = kind == PH_LM ? a.vocab : a.dim;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int e = lane + 32 * k, row = e >> 3, tok = e & 7;
                    const int gr = rg * kTileRows + row;
                    if (gr < ld && tok < nv) out[(size_t)tok * ld + gr] = v[k];
                }
                if (kind == PH_LM) {
                    // token lane & 7 of rows (lane >> 3) + 4k: best of the four, then of the four lanes of the
                    // token, into this CTA's best
                    unsigned long long key = 0;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int gr = rg * kTileRows + (lane >> 3) + 4 * k;
                        if (gr < ld) key = max(key, argmax_key(v[k], gr));
                    }
                    key = max(key, __shfl_xor_sync(0xffffffffu, key, 8));
                    key = max(key, __shfl_xor_sync(0xffffffffu, key, 16));
                    if (lane < 8 && lane < nv) atomicMax(&m->best[lane], key);
                }
            }
        }
    }
}

__device__ __forceinline__ void attention_phase(const FwdArgs& a, int l, uint8_t* uni, int nv, int pos, int tid) {
    const int warp = tid >> 5;
    const int G = gridDim.x;
    const AttnArgs aa = attn_args(a, l, pos);
    const int grp = warp >> 3;  // two 8-warp groups per CTA over the (kv head, chunk) items
    if (grp >= kFwdAttnGroups || nv <= 0) return;
    const int hi_max = pos + nv - 1, lo_min = max(0, pos + 1 - a.max_seq);
    const int c_first = lo_min / aa.chunk, c_last = hi_max / aa.chunk;
    const int n_items = (c_last - c_first + 1) * a.n_kvh;
    const AttnSmem sm = attn_smem_at(uni + (size_t)grp * attn_smem_bytes());
    const int bar_id = kBarAttn0 + grp;
    for (int item = blockIdx.x * kFwdAttnGroups + grp; item < n_items; item += G * kFwdAttnGroups) {
        const int nx = item + G * kFwdAttnGroups;  // this group's next item, prefetched into L2 during this one
        attn_item(aa, nv, pos, lo_min, hi_max, item % a.n_kvh, c_first + item / a.n_kvh, nx % a.n_kvh,
                  nx < n_items ? c_first + nx / a.n_kvh : -1, sm, tid & 255, [bar_id] { named_sync(bar_id, 256); });
    }
}

// combine_warps(max_seq) warps per (token, head) row; warps 0-15 hold 16 / that many rows at a time.
__device__ __forceinline__ void combine_phase(const FwdArgs& a, int l, uint8_t* uni, int nv, int pos, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const int nwc = combine_warps(a.max_seq), slots = 16 / nwc;
    const int slot = warp / nwc;
    if (slot >= slots) return;
    const AttnArgs aa = attn_args(a, l, pos);
    float* obuf = reinterpret_cast<float*>(uni) + slot * nwc * kHD;
    const int bar_id = kBarAttn0 + slot;
    const int nthr = nwc * 32;
    for (int row = blockIdx.x * slots + slot; row < nv * a.n_heads; row += gridDim.x * slots)
        attn_combine_row(aa, nwc, pos, row / a.n_heads, row % a.n_heads, warp % nwc, lane, obuf,
                         [bar_id, nthr] { named_sync(bar_id, nthr); });
}

// idx: the reduction's index in the forward (2 per layer).  Tensor parallel: after the grid barrier this
// rank's slices are complete; CTA 0 publishes the reduction's sequence number to every rank's flags, and
// every CTA waits (bounded) until all ranks have published before reading their slices.
__device__ __forceinline__ void red_phase(const FwdArgs& a, Misc* m, int idx, unsigned long long seq0, int kparts,
                                          const float* wn, int nv, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const int nbd = a.dim >> 5;
    const float* src[kMaxTp];
    int nsrc = 1;
    src[0] = a.yparts;
    if (a.tp.n > 1) {
        const unsigned long long seq = seq0 + idx + 1;
        const size_t boff = (size_t)(seq & 1) * a.tp.buf;
        nsrc = a.tp.n;
        for (int r = 0; r < kMaxTp; ++r) src[r] = r < nsrc ? a.tp.y[r] + boff : nullptr;
        if (blockIdx.x == 0 && tid < a.tp.n) {
            __threadfence_system();
            asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.tp.flags[tid] + a.tp.rank), "l"(seq) : "memory");
        }
        if (tid == 0 && !m->abort) {
            const uint64_t t0 = global_ns();
            for (int r = 0; r < a.tp.n; ++r) {
                const unsigned long long* fl = a.tp.flags[a.tp.rank] + r;
                unsigned long long v;
                while (true) {
                    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(fl) : "memory");
                    if (v >= seq) break;
                    if (global_ns() - t0 > kWaitLimitNs) {
                        set_dev_error(a.err, DEV_ERR_PEER_WAIT);
                        m->abort = 1;
                        break;
                    }
                }
            }
        }
        named_sync(kBarCompute, kComputeThreads);
    }
    for (int wt = blockIdx.x * kComputeWarps + warp; wt < nv * nbd; wt += gridDim.x * kComputeWarps)
        red_block(a, src, nsrc, wt / nbd, wt % nbd, kparts, wn, lane);
}

// embedding: x rows, their 16-row sums of squares and Q8_0 of x * (layer 0 attention norm weight); one
// warp per (token, 32-value block)
__device__ __forceinline__ void embed_phase(const FwdArgs& a, int nv, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const int nbd = a.dim >> 5;
    const float* w0 = a.layers[0].rms_att;
    for (int wt = blockIdx.x * kComputeWarps + warp; wt < nv * nbd; wt += gridDim.x * kComputeWarps) {
        const int s = wt / nbd, b = wt % nbd;
        const int token = a.tokens ? a.tokens[s] : a.ctrl->tokens[s];
        const float v = embed_value(a.embd, a.embd_type, token, a.dim, b, lane);
        finish_block(a, s, b, v, w0[b * 32 + lane], lane);
    }
}

}  // namespace

__global__ void __launch_bounds__(kGemvThreads, 1) k_forward(const FwdArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const FwdSmem L = fwd_layout(a.nstage);
    Misc* m = reinterpret_cast<Misc*>(smem + L.misc);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + kMaxStages;
    uint64_t* red_full = empty + kMaxStages;
    uint64_t* red_empty = red_full + kRedSlots;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (a.ctrl && a.ctrl->done) return;  // uniform: nothing writes ctrl while the kernel runs
    const int nv = a.ctrl ? min(a.ctrl->n_valid, a.S) : a.S;
    const int pos = a.ctrl ? a.ctrl->pos : 0;
    if (nv <= 0) return;  // a slice of a verify batch with no valid token (uniform, as above)

    if (tid == 0) {
        for (int i = 0; i < a.nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        for (int i = 0; i < kRedSlots; ++i) {
            mbar_init(&red_full[i], kConsumerWarps);
            mbar_init(&red_empty[i], kEpiWarps);
        }
        mbar_init(&red_empty[kRedSlots], 1);  // act barrier (after the red slots)
        m->abort = 0;
        m->issued = 0;
        m->pdone = 0;
        m->act_issued = 0;
        for (int i = 0; i < kMaxS; ++i) m->best[i] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    Ring R;
    R.act_full = &red_empty[kRedSlots];
    R.ring = smem + L.ring;
    R.full = full;
    R.empty = empty;
    R.red_full = red_full;
    R.red_empty = red_empty;
    R.red = reinterpret_cast<float*>(smem + L.red);
    R.ubuf = reinterpret_cast<float*>(smem + L.ubuf);
    R.nstage = a.nstage;

    if (warp == kProducerWarp) {
        // ---------------- producer: every matvec tile of the forward, in consumption order ----------------
        if (lane == 0) {
            const volatile int* abort_flag = &m->abort;
            uint32_t sidx = 0;
            RingPos pp;
            bool ok = true;
            auto stream = [&](const MvPhase& p, const uint8_t* w) {
                const Items it = my_items(p);
                const int nq_p = p.nq / p.kparts, cpr = nq_p / p.chunk, pairs = p.rpu / kRPW;
                const uint32_t half = (uint32_t)p.chunk * kTileBytes;
                for (int i = it.i0; i < it.i1 && ok; ++i) {
                    const int part = i / p.n_units, unit = i % p.n_units;
                    for (int pr = 0; pr < pairs && ok; ++pr) {
                        const int rg = unit * p.rpu + pr * kRPW;
                        for (int ch = 0; ch < cpr; ++ch) {
                            const int slot = pp.slot;
                            if (sidx >= (uint32_t)a.nstage && !wait_or_abort_1(&empty[slot], pp.phase ^ 1, abort_flag)) {
                                if (!*abort_flag) set_dev_error(a.err, DEV_ERR_EMPTY_WAIT);
                                m->abort = 1;
                                ok = false;
                                break;
                            }
                            const uint8_t* src =
                                w + ((size_t)rg * p.nq + (size_t)part * nq_p + (size_t)ch * p.chunk) * kTileBytes;
                            uint8_t* dst = R.ring + (size_t)slot * kStageBytes;
                            mbar_arrive_expect_tx(&full[slot], 2 * half);
                            bulk_g2s(dst, src, half, &full[slot]);
                            bulk_g2s(dst + half, src + (size_t)p.nq * kTileBytes, half, &full[slot]);
                            ++sidx;
                            pp.advance(a.nstage);
                        }
                    }
                }
            };
            for (int l = 0; l < a.n_layers && ok; ++l) {
                const FwdLayer& W = a.layers[l];
                stream(a.qkv, W.qkv);
                if (ok) stream(a.wo, W.wo);
                if (ok) stream(a.w13, W.w13);
                if (ok) stream(a.w2, W.w2);
            }
            if (a.lm && ok) stream(a.lmp, a.lm);
            reinterpret_cast<volatile uint32_t*>(&m->issued)[0] = sidx;
            __threadfence_block();
            reinterpret_cast<volatile int*>(&m->pdone)[0] = 1;
        }
        return;
    }

    // ---------------- compute warps: the phase table ----------------
    uint32_t target = 0, pidx = 0, nstg = 0;
    RingPos rp;
    bool ab = false;
    embed_phase(a, nv, tid);
    grid_barrier(a, m, target);
    uint8_t* uni = smem + L.act;
    const int n_ph = 8 * a.n_layers + (a.lm ? 1 : 0);
    // the o-proj epilogue finishes the residual itself when its sums are complete locally
    const bool wo_fused = a.wo.kparts == 1 && a.tp.n <= 1;
    // reductions done before this forward (tensor parallel; read before any CTA can advance it)
    const unsigned long long seq0 = a.tp.n > 1 ? *a.tp.base : 0ull;
    for (int ph = 0; ph < n_ph; ++ph) {
        const int l = ph >> 3, k = ph & 7;
        if (k == 1 && l < a.n_layers) {
            attention_phase(a, l, uni, nv, pos, tid);
        } else if (k == 2) {
            combine_phase(a, l, uni, nv, pos, tid);
        } else if (k == 4 && wo_fused) {
            // done by the o-proj epilogue
        } else if (k == 4 || k == 7) {
            const int kp = k == 4 ? a.wo.kparts : a.w2.kparts;
            const float* wn = k == 4 ? a.layers[l].rms_ffn : l + 1 < a.n_layers ? a.layers[l + 1].rms_att : a.rms_out;
            red_phase(a, m, 2 * l + (k == 7), seq0, kp, wn, nv, tid);
        } else {
            const int kind = l == a.n_layers ? PH_LM : k == 0 ? PH_QKV : k == 3 ? PH_WO : k == 5 ? PH_W13 : PH_W2;
            mv_phase(a, kind, l, R, m, rp, pidx, nstg, ab, nv, pos, tid);
        }
        // no barrier after the o-proj when it finished the residual itself
        if (ph + 1 < n_ph && !(k == 3 && wo_fused && l < a.n_layers)) grid_barrier(a, m, target);
    }

    // Drain: no bulk copy may still be landing in shared memory when the CTA exits.  Only the last
    // nstage issued stages can be in flight (a slot is reissued only after every consumer waited for it).
    named_sync(kBarCompute, kComputeThreads);
    // the LM head's argmax: this CTA's best key per token into the forward's keys
    if (a.lm && tid < nv && m->best[tid]) atomicMax(reinterpret_cast<unsigned long long*>(a.sync + 32) + tid, m->best[tid]);
    if (tid == 0) {
        const volatile int* pd = &m->pdone;
        uint32_t n = 0;
        while (!*pd && ++n < kSpinLimit) __nanosleep(32);
        const uint32_t issued = reinterpret_cast<volatile uint32_t*>(&m->issued)[0];
        const uint32_t first = issued > (uint32_t)a.nstage ? issued - a.nstage : 0;
        for (uint32_t s = first; s < issued; ++s) mbar_wait(&full[s % a.nstage], (s / a.nstage) & 1);
        const uint32_t acts = reinterpret_cast<volatile uint32_t*>(&m->act_issued)[0];
        if (acts > 0) mbar_wait(R.act_full, (acts - 1) & 1);
    }
}

size_t fwd_smem_bytes(int nstage) { return fwd_layout(nstage).total; }

int fwd_pick_stages(int max_smem) {
    for (int n = kMaxStages; n >= 2; --n)
        if (fwd_layout(n).total <= (size_t)max_smem) return n;
    return 0;
}

// word 0: the grid barrier counter; words 32..: the argmax keys (u64 per token)
size_t fwd_sync_words(int) { return 32 + 2 * kMaxS; }

cudaError_t fwd_init_attrs(int max_smem) {
    return cudaFuncSetAttribute(k_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

cudaError_t fwd_blocks_per_sm(size_t smem, int* n) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, k_forward, kGemvThreads, smem);
}

cudaError_t launch_forward(const FwdArgs& a, int grid, size_t smem, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_forward, a);
}

}  // namespace sd
