// sd_dev.cuh -- device building blocks shared by the stand-alone kernels (sd_gemv.cu, sd_attn.cu,
// sd_quant.cu) and the persistent forward kernel (sd_fwd.cu).  Both paths run the same code in the same
// reduction orders, so they produce bit-identical results.
#pragma once
#include "sd_attn.h"
#include "sd_common.cuh"

namespace sd {

// The MMA accumulator is initialised with -8*sum(codes) + kMagic: the result bits are then the fp32
// value 1.5*2^23 + isum (exact for |isum| < 2^22; |isum| <= 32*8*128 here), so one exact FADD
// recovers (float)isum without the quarter-rate I2F conversion.
constexpr int kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float2 h2x2f(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// ---------------------------------------------------------------------------------------------
// Matvec activation fragments in shared memory, for one K slice of nb Q8_0 blocks and S tokens:
//   b[blk*4S + 4s + tt]  = (word tt, word 4+tt) of token s's codes in block blk  (MMA B fragment)
//   zero[4 * 4S]         = zeros read by lanes whose token column g >= S
//   c[blk*4 + t]         = C quad (-8*sum + magic for tokens 2t, 2t+1, repeated for rows g+8)
//   x[blk*4 + t]         = (xd of token 2t, xd of token 2t+1)
// ---------------------------------------------------------------------------------------------
struct ActSmem {
    uint2* b;
    uint2* zero;
    int4* c;
    float2* x;
};

__host__ __device__ inline size_t act_smem_bytes(int nb, int S) {
    return (size_t)nb * 4 * S * 8 + (size_t)4 * 4 * S * 8 + (size_t)nb * 4 * 16 + (size_t)nb * 4 * 8;
}

__device__ inline ActSmem act_smem_at(uint8_t* base, int nb, int S) {
    ActSmem A;
    A.b = reinterpret_cast<uint2*>(base);
    A.zero = reinterpret_cast<uint2*>(base + (size_t)nb * 4 * S * 8);
    A.c = reinterpret_cast<int4*>(base + (size_t)nb * 4 * S * 8 + (size_t)4 * 4 * S * 8);
    A.x = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(A.c) + (size_t)nb * 4 * 16);
    return A;
}

// Stage Q8 planes (global, row stride K) blocks [kb0, kb0 + nb) of tokens < nv into A.  Loads are
// issued in batches of four per thread before any store, so a staging costs about one memory round trip.
// tok_scale (optional, shared memory): per-token factor applied to the block scales (the RMSNorm
// scale when the planes hold Q8_0 of x*w).
__device__ inline void stage_act_from_planes(const ActSmem& A, const Q8Planes& act, int K, int kb0, int nb, int S, int nv,
                                             int tid, int nthr, const float* tok_scale = nullptr) {
    constexpr int U = 4;
    const int n16 = S * nb * 2;
    for (int i0 = tid; i0 < n16; i0 += U * nthr) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * nthr;
            v[u] = make_uint4(0, 0, 0, 0);
            if (i < n16) {
                const int s = i / (nb * 2), rem = i - s * (nb * 2);
                if (s < nv)
                    v[u] = *reinterpret_cast<const uint4*>(act.qs + (size_t)s * K + (size_t)(kb0 + (rem >> 1)) * 32 +
                                                           (rem & 1) * 16);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * nthr;
            if (i < n16) {
                const int s = i / (nb * 2), rem = i - s * (nb * 2);
                uint32_t* base = reinterpret_cast<uint32_t*>(A.b + (size_t)(rem >> 1) * 4 * S + 4 * s) + (rem & 1);
                base[0] = v[u].x;
                base[2] = v[u].y;
                base[4] = v[u].z;
                base[6] = v[u].w;
            }
        }
    }
    for (int i = tid; i < 4 * 4 * S; i += nthr) A.zero[i] = make_uint2(0, 0);
    const int nbK = K >> 5;
    for (int i0 = tid; i0 < nb * 4; i0 += 2 * nthr) {
        int sm[2][2];
        float dv[2][2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = i0 + u * nthr;
            const int b = i >> 2, tt = i & 3;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int s = 2 * tt + h;
                sm[u][h] = 0;
                dv[u][h] = 0.f;
                if (i < nb * 4 && s < nv) {
                    sm[u][h] = act.sum[(size_t)s * nbK + kb0 + b];
                    dv[u][h] = act.d[(size_t)s * nbK + kb0 + b];
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = i0 + u * nthr;
            if (i < nb * 4) {
                const int c0 = kMagicI - 8 * sm[u][0], c1 = kMagicI - 8 * sm[u][1];
                A.c[i] = make_int4(c0, c1, c0, c1);
                float d0 = dv[u][0], d1 = dv[u][1];
                if (tok_scale) {
                    const int tt = i & 3;
                    if (2 * tt < nv) d0 = d0 * tok_scale[2 * tt];
                    if (2 * tt + 1 < nv) d1 = d1 * tok_scale[2 * tt + 1];
                }
                A.x[i] = make_float2(d0, d1);
            }
        }
    }
}

// Write one quantised block (lane j holds code q of element j, every lane holds d and sum) of token s
// into A.  Called by one full warp.  Tokens s < S only; the C quad / scale slots of s are set here.
__device__ inline void stage_act_block(const ActSmem& A, int s, int b, int S, int q, float d, int sum, int lane) {
    // word w (0..7) = codes 4w..4w+3; lane w < 8 gathers its word
    uint32_t word = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int v = __shfl_sync(0xffffffffu, q, (lane & 7) * 4 + k);
        word |= (uint32_t)(v & 0xFF) << (8 * k);
    }
    if (lane < 8) {
        uint32_t* base = reinterpret_cast<uint32_t*>(A.b + (size_t)b * 4 * S + 4 * s);
        const int tt = lane & 3, half = lane >> 2;
        base[tt * 2 + half] = word;
    }
    if (lane == 0) {
        int* cp = reinterpret_cast<int*>(&A.c[b * 4 + (s >> 1)]);
        cp[s & 1] = kMagicI - 8 * sum;
        cp[(s & 1) + 2] = kMagicI - 8 * sum;
        reinterpret_cast<float*>(&A.x[b * 4 + (s >> 1)])[s & 1] = d;
    }
}

// Empty token slot s (s >= nv, s < the pair's 8-token width): C quad magic, scale 0, codes 0.
__device__ inline void stage_act_empty(const ActSmem& A, int s, int b, int S, int lane) {
    if (s < S && lane < 4) A.b[(size_t)b * 4 * S + 4 * s + lane] = make_uint2(0, 0);
    if (lane == 0) {
        int* cp = reinterpret_cast<int*>(&A.c[b * 4 + (s >> 1)]);
        cp[s & 1] = kMagicI;
        cp[(s & 1) + 2] = kMagicI;
        reinterpret_cast<float*>(&A.x[b * 4 + (s >> 1)])[s & 1] = 0.f;
    }
}

// One consumer warp's share of a ring slot: its 1152-byte tile of each of the kRPW row-groups of the
// pair (tile r at slot + r*half_bytes + warp*kTileBytes).  Loaded into registers so that the slot can
// be released before the math.
struct TileRegs {
    uint4 wl[kRPW], wh[kRPW];
    uint2 sl[kRPW], sh[kRPW];
};

__device__ __forceinline__ void load_tiles(const uint8_t* slot, uint32_t half_bytes, int warp, int lane, TileRegs& tr) {
    const int g = lane >> 2;
#pragma unroll
    for (int r = 0; r < kRPW; ++r) {
        const uint8_t* tile = slot + r * half_bytes + warp * kTileBytes;
        tr.wl[r] = *reinterpret_cast<const uint4*>(tile + lane * 16);
        tr.wh[r] = *reinterpret_cast<const uint4*>(tile + 512 + lane * 16);
        tr.sl[r] = *reinterpret_cast<const uint2*>(tile + 1024 + g * 8);
        tr.sh[r] = *reinterpret_cast<const uint2*>(tile + 1088 + g * 8);
    }
}

// int8 MMA over blocks [bbase, bbase+4) of the slice for both row-groups (rg, rg+1) of the pair.
// Accumulates (wd*xd) * isum per block into accL (rows g) / accH (rows g+8), or with BLOCKSUMS writes
// the exact block sums isum[row][kb0 + block] instead.
template <bool BLOCKSUMS>
__device__ __forceinline__ void consume_tiles(const TileRegs& tr, int lane, const ActSmem& A, int S, int bbase,
                                              float2 (&accL)[kRPW], float2 (&accH)[kRPW], int32_t* isum, int rg,
                                              int out_rows, size_t nbK, int kb0) {
    const int g = lane >> 2, t = lane & 3;
    float2 dl[kRPW][2], dh[kRPW][2];
#pragma unroll
    for (int r = 0; r < kRPW; ++r) {
        dl[r][0] = h2x2f(tr.sl[r].x);
        dl[r][1] = h2x2f(tr.sl[r].y);
        dh[r][0] = h2x2f(tr.sh[r].x);
        dh[r][1] = h2x2f(tr.sh[r].y);
    }
    const bool zero_lane = g >= S;  // token column g beyond S reads zeros
    const uint2* bf_p = zero_lane ? A.zero + t : A.b + lane + (size_t)bbase * 4 * S;
    const int4* c_p = A.c + bbase * 4 + t;
    const float2* x_p = A.x + bbase * 4 + t;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const uint2 bf = bf_p[zero_lane ? 0 : blk * 4 * S];
        const int4 cq = c_p[blk * 4];
        const float2 xd = x_p[blk * 4];
#pragma unroll
        for (int r = 0; r < kRPW; ++r) {
            const uint32_t wlo = blk == 0 ? tr.wl[r].x : blk == 1 ? tr.wl[r].y : blk == 2 ? tr.wl[r].z : tr.wl[r].w;
            const uint32_t whi = blk == 0 ? tr.wh[r].x : blk == 1 ? tr.wh[r].y : blk == 2 ? tr.wh[r].z : tr.wh[r].w;
            const uint32_t a0 = wlo & 0x0F0F0F0Fu, a2 = (wlo >> 4) & 0x0F0F0F0Fu;
            const uint32_t a1 = whi & 0x0F0F0F0Fu, a3 = (whi >> 4) & 0x0F0F0F0Fu;
            int d[4];
            mma_u8s8(d, a0, a1, a2, a3, bf.x, bf.y, cq.x, cq.y, cq.z, cq.w);
            if constexpr (BLOCKSUMS) {
                if (t == 0 && (rg + r) * kTileRows < out_rows) {
                    const int r0 = (rg + r) * kTileRows + g;
                    isum[(size_t)r0 * nbK + kb0 + bbase + blk] = d[0] - kMagicI;
                    isum[(size_t)(r0 + 8) * nbK + kb0 + bbase + blk] = d[2] - kMagicI;
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

// Consumer partials of one pair -> red slot [kRPW][kConsumerWarps][128] (row*8 + tok).
__device__ __forceinline__ void write_partials(float* slot_base, int warp, int lane, const float2 (&accL)[kRPW],
                                               const float2 (&accH)[kRPW]) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int r = 0; r < kRPW; ++r) {
        float* rr = slot_base + ((size_t)r * kConsumerWarps + warp) * 128;
        *reinterpret_cast<float2*>(&rr[g * 8 + 2 * t]) = accL[r];
        *reinterpret_cast<float2*>(&rr[(g + 8) * 8 + 2 * t]) = accH[r];
    }
}

// Epilogue warp: sum the partials of consumer warps 0..nw-1 (in order) of one row-group.
// v[k] is element e = lane + 32k: row = e >> 3, token = e & 7.
__device__ __forceinline__ void reduce_partials(const float* rr, int nw, int lane, float (&v)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = 0.f;
    for (int w = 0; w < nw; ++w) {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] += rr[w * 128 + lane + 32 * k];
    }
}

// QKV epilogue for one row-group (see sd_internal.h EPI_QKV).  element (row, tok) lives in lane
// (row*8 + tok) % 32, register (row*8 + tok) / 32; the partner row (row ^ 1) of a RoPE pair is the same
// register of lane ^ 8.
__device__ __forceinline__ void epi_qkv(const float (&v)[4], int rg, int lane, int nv, int pos, float* q_out, __half* k_cache,
                                        __half* v_cache, int q_rows, int kv_rows, int max_seq, int head_dim,
                                        const float* theta_inv, float q_scale) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int e = lane + 32 * k;
        const int row = e >> 3, tok = e & 7;
        const float other = __shfl_xor_sync(0xffffffffu, v[k], 8);
        if ((row & 1) == 0 && tok < nv) {
            const float ve = v[k], vo = other;
            const int gr = rg * kTileRows + row;
            const int tpos = pos + tok;
            if (gr < q_rows + kv_rows) {
                // RoPE on q and k rows (mistral/mistral_model.h:79-122)
                const int i = (gr % head_dim) >> 1;
                const float ang = theta_inv[i] * (float)tpos;
                float sn, cs;
                sincosf(ang, &sn, &cs);
                const float e2 = fmaf(-vo, sn, ve * cs);
                const float o2 = fmaf(ve, sn, vo * cs);
                if (gr < q_rows) {
                    q_out[(size_t)tok * q_rows + gr] = e2 * q_scale;
                    q_out[(size_t)tok * q_rows + gr + 1] = o2 * q_scale;
                } else {
                    const size_t sl = (size_t)(tpos % max_seq) * kv_rows + (gr - q_rows);
                    k_cache[sl] = __float2half_rn(e2);
                    k_cache[sl + 1] = __float2half_rn(o2);
                }
            } else if (gr < q_rows + 2 * kv_rows) {
                const size_t sl = (size_t)(tpos % max_seq) * kv_rows + (gr - q_rows - kv_rows);
                v_cache[sl] = __float2half_rn(ve);
                v_cache[sl + 1] = __float2half_rn(vo);
            }
        }
    }
}

// SiLU(gate)*up + Q8_0 of one 32-unit block for tokens r*4 .. r*4+3 (epilogue warp r of 2).
// ubuf: [4][128] = gate lo, gate hi, up lo, up hi (row*8 + tok).
__device__ __forceinline__ void epi_silu_q8(const float* ubuf, int r, int lane, int unit, int nv, Q8Planes h, int hidden) {
    const int nbh = hidden >> 5;
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
            h.qs[(size_t)tok * hidden + unit * 32 + lane] = (int8_t)q;
            if (lane == 0) {
                h.d[(size_t)tok * nbh + unit] = dq;
                h.sum[(size_t)tok * nbh + unit] = sq;
            }
        }
    }
}

// Canonical RMSNorm statistics, shared by both forward paths so that they agree bit for bit
// (mistral/mistral_model.h:54-77 sums sequentially; this is a fixed parallel order).  A row of dim
// values is cut into 16-value groups -- the row-groups of the matvec that produces the row, so that a
// matvec epilogue can finish its group's statistic.  Group sum: q_j = fma chain over k = 0..3 of
// v[4k + j]^2 (j = 0..3), then (q0 + q1) + (q2 + q3).  Row sum: lane l adds groups l, l + 32, ... in
// order (dim / 16 a multiple of 32), then the warp butterfly.

// Thread-level group sum of v[0..15].
__device__ __forceinline__ float group16_sumsq(const float* v) {
    float q[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        q[j] = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) q[j] = fmaf(v[4 * k + j], v[4 * k + j], q[j]);
    }
    return (q[0] + q[1]) + (q[2] + q[3]);
}

// The same sum in the matvec epilogue layout: lane holds v[k] = (row (lane >> 3) + 4k, token lane & 7)
// of one row-group; every lane returns the sum of its token.
__device__ __forceinline__ float group16_sumsq_epi(const float (&v)[4]) {
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) q = fmaf(v[k], v[k], q);
    q += __shfl_xor_sync(0xffffffffu, q, 8);
    q += __shfl_xor_sync(0xffffffffu, q, 16);
    return q;
}

// Row sum of squares from the group sums (one warp; every lane returns it).  ngroups <= 256; the
// loads are all issued before the (ordered) additions.
__device__ __forceinline__ float row_sumsq(const float* gss, int ngroups, int lane) {
    float g[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] = (lane + 32 * k < ngroups) ? gss[lane + 32 * k] : 0.f;
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
        if (lane + 32 * k < ngroups) t += g[k];
    return warp_sum(t);
}

__device__ __forceinline__ float rms_scale(float ss, int dim, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)dim) + eps));
}

// Value e (0..31) of a Q4_0 embedding block (mistral/dequant.h dequant_q4_0 semantics).
__device__ __forceinline__ float q4_0_value(const uint8_t* blk, int e) {
    const float dd = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
    const uint8_t byte = blk[2 + (e & 15)];
    const int q = (e < 16) ? (byte & 0x0F) : (byte >> 4);
    return dd * ((float)q - 8.0f);
}

// ---------------------------------------------------------------------------------------------
// Attention work item (kv head, chunk) for one group of 4 warps (128 threads); see sd_attn.cu.
// ---------------------------------------------------------------------------------------------
constexpr int kHD = 128;        // head_dim
constexpr int kGQA = 4;         // query heads per kv head
constexpr int kSub = 32;        // positions per sub-block (one per lane)
constexpr int kAttnThreads = 128;

struct AttnSmem {
    float* qs;      // [kMaxS * kGQA][kHD]
    __half* kt;     // [kHD][kSub + 2]
    __half* vt;     // [kSub][kHD]
};

__host__ __device__ constexpr size_t attn_smem_bytes() {
    return (size_t)kMaxS * kGQA * kHD * 4 + (size_t)kHD * (kSub + 2) * 2 + (size_t)kSub * kHD * 2;
}

__device__ inline AttnSmem attn_smem_at(uint8_t* base) {
    AttnSmem s;
    s.qs = reinterpret_cast<float*>(base);
    s.kt = reinterpret_cast<__half*>(base + (size_t)kMaxS * kGQA * kHD * 4);
    s.vt = reinterpret_cast<__half*>(base + (size_t)kMaxS * kGQA * kHD * 4 + (size_t)kHD * (kSub + 2) * 2);
    return s;
}

// K/V sub-block of kSub positions: thread's 4 pieces (position j = i/16, dims 8*(i%16) .. +7) of
// K and V, loaded into registers together.
struct KvRegs {
    uint4 k[4], v[4];
};

__device__ __forceinline__ void attn_load_kv(const AttnArgs& a, int kvh, int sb, int p1, int tid, KvRegs& r) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = tid + u * kAttnThreads;  // < kSub * kHD / 8 = 512
        const int j = i >> 4, d8 = (i & 15) * 8;
        const int p = sb + j;
        r.k[u] = r.v[u] = make_uint4(0, 0, 0, 0);
        if (p < p1) {
            const size_t off = (size_t)(p % a.max_seq) * a.kv_ld + (size_t)kvh * kHD + d8;
            r.k[u] = *reinterpret_cast<const uint4*>(a.k + off);
            r.v[u] = *reinterpret_cast<const uint4*>(a.v + off);
        }
    }
}

__device__ __forceinline__ void attn_store_kv(const AttnSmem& sm, int tid, const KvRegs& r) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = tid + u * kAttnThreads;
        const int j = i >> 4, d8 = (i & 15) * 8;
        const __half* kh = reinterpret_cast<const __half*>(&r.k[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) sm.kt[(d8 + e) * (kSub + 2) + j] = kh[e];
        *reinterpret_cast<uint4*>(&sm.vt[j * kHD + d8]) = r.v[u];
    }
}

// gsync(): a barrier over the 128 threads of the group.  The query rows and the first K/V sub-block are
// loaded together, so an item of one sub-block costs about one memory round trip before its math.
// Tokens are processed TG at a time (a register budget: TG = 4 in the persistent forward, 8 in the
// attention kernel); each token's arithmetic is the same either way.
template <int TG, class Sync>
__device__ void attn_item(const AttnArgs& a, int nv, int pos, int lo_min, int hi_max, int kvh, int c, const AttnSmem& sm,
                          int tid, Sync gsync) {
    const int warp = tid >> 5, lane = tid & 31;
    const int hq = warp;  // warp w computes query head 4*kvh + w
    const int p0 = max(c * a.chunk, lo_min);
    const int p1 = min((c + 1) * a.chunk, hi_max + 1);  // exclusive
    gsync();
    {
        float4 qv[8];  // rows r = s*4 + h, 32 float4 per row: kMaxS * kGQA * 32 = 8 * 128
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + u * kAttnThreads;
            const int r = i >> 5, d4 = (i & 31) * 4;
            const int s = r / kGQA, h = r % kGQA;
            qv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (s < nv) qv[u] = *reinterpret_cast<const float4*>(a.q + (size_t)s * a.q_ld + (size_t)(kvh * kGQA + h) * kHD + d4);
        }
        KvRegs kv;
        attn_load_kv(a, kvh, p0, p1, tid, kv);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + u * kAttnThreads;
            *reinterpret_cast<float4*>(&sm.qs[(i >> 5) * kHD + (i & 31) * 4]) = qv[u];
        }
        attn_store_kv(sm, tid, kv);
    }
    int resident = p0;  // sub-block held in shared memory
    for (int t0 = 0; t0 < nv; t0 += TG) {
        float m[TG], l[TG], acc[TG][4];
#pragma unroll
        for (int j = 0; j < TG; ++j) {
            m[j] = -INFINITY;
            l[j] = 0.f;
            acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        }
        for (int sb = p0; sb < p1; sb += kSub) {
            if (sb != resident) {
                KvRegs kv;
                attn_load_kv(a, kvh, sb, p1, tid, kv);
                gsync();  // every warp is done with the resident sub-block
                attn_store_kv(sm, tid, kv);
                resident = sb;
            }
            gsync();
            float sc[TG];
#pragma unroll
            for (int j = 0; j < TG; ++j) sc[j] = 0.f;
            for (int d = 0; d < kHD; d += 4) {
                const float k0 = __half2float(sm.kt[d * (kSub + 2) + lane]), k1 = __half2float(sm.kt[(d + 1) * (kSub + 2) + lane]);
                const float k2 = __half2float(sm.kt[(d + 2) * (kSub + 2) + lane]), k3 = __half2float(sm.kt[(d + 3) * (kSub + 2) + lane]);
#pragma unroll
                for (int j = 0; j < TG; ++j) {
                    if (t0 + j < nv) {
                        const float4 qv = *reinterpret_cast<const float4*>(&sm.qs[((t0 + j) * kGQA + hq) * kHD + d]);
                        sc[j] = fmaf(qv.x, k0, sc[j]);
                        sc[j] = fmaf(qv.y, k1, sc[j]);
                        sc[j] = fmaf(qv.z, k2, sc[j]);
                        sc[j] = fmaf(qv.w, k3, sc[j]);
                    }
                }
            }
            const int p = sb + lane;
            float pr[TG];
#pragma unroll
            for (int j = 0; j < TG; ++j) {
                pr[j] = 0.f;
                if (t0 + j >= nv) continue;
                const int hi = pos + t0 + j, lo = max(0, hi + 1 - a.max_seq);
                const bool ok = p < p1 && p >= lo && p <= hi;
                const float v = ok ? sc[j] : -INFINITY;
                const float mx = warp_max(v);
                const float mn = fmaxf(m[j], mx);
                // a token with nothing valid yet keeps m = -inf and contributes nothing
                const float e = (mn == -INFINITY || !ok) ? 0.f : expf(v - mn);
                const float corr = (mn == -INFINITY || m[j] == -INFINITY) ? 0.f : expf(m[j] - mn);
                const float es = warp_sum(e);
                l[j] = l[j] * corr + es;
                acc[j][0] *= corr;
                acc[j][1] *= corr;
                acc[j][2] *= corr;
                acc[j][3] *= corr;
                m[j] = mn;
                pr[j] = e;
            }
            for (int jj = 0; jj < kSub; ++jj) {
                const uint2 vraw = *reinterpret_cast<const uint2*>(&sm.vt[jj * kHD + lane * 4]);
                const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.x));
                const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.y));
#pragma unroll
                for (int j = 0; j < TG; ++j) {
                    if (t0 + j < nv) {
                        const float w = __shfl_sync(0xffffffffu, pr[j], jj);
                        acc[j][0] = fmaf(w, f01.x, acc[j][0]);
                        acc[j][1] = fmaf(w, f01.y, acc[j][1]);
                        acc[j][2] = fmaf(w, f23.x, acc[j][2]);
                        acc[j][3] = fmaf(w, f23.y, acc[j][3]);
                    }
                }
            }
        }
        const int h = kvh * kGQA + hq;
#pragma unroll
        for (int j = 0; j < TG; ++j) {
            const int s = t0 + j;
            if (s >= nv) continue;
            const size_t pi = ((size_t)s * a.n_heads + h) * a.max_chunks + c;
            if (lane == 0) a.part_ml[pi] = make_float2(m[j], l[j]);
            *reinterpret_cast<float4*>(a.part_acc + pi * kHD + lane * 4) =
                make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
        }
    }
}

// Merge the chunk partials of (token s, head h) and quantise the 128 outputs to 4 Q8_0 blocks.
// One warp; lane owns dims 4*lane..4*lane+3.  Chunks are taken in groups of 128: a group's
// (max, sum) pairs are loaded lane-parallel in one go and its per-chunk factors broadcast by shuffle;
// the accumulator rows are read in batches of 4 chunks, the next batch's loads in flight while the
// current one is added.  Every sum runs in chunk order (per lane for L), so the result does not depend
// on how the loads are batched.
__device__ inline void attn_combine_row(const AttnArgs& a, int pos, int s, int h, int lane) {
    const int hi = pos + s, lo = max(0, hi + 1 - a.max_seq);
    const int c0 = lo / a.chunk, c1 = hi / a.chunk;
    const size_t base = ((size_t)s * a.n_heads + h) * a.max_chunks;
    auto load_ml = [&](int g0, float2 (&ml)[4]) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = g0 + lane + 32 * u;
            ml[u] = c <= c1 ? a.part_ml[base + c] : make_float2(-INFINITY, 0.f);
        }
    };
    float2 ml0[4];
    load_ml(c0, ml0);
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < 4; ++u) M = fmaxf(M, ml0[u].x);
    for (int g0 = c0 + 128; g0 <= c1; g0 += 128) {
        float2 ml[4];
        load_ml(g0, ml);
#pragma unroll
        for (int u = 0; u < 4; ++u) M = fmaxf(M, ml[u].x);
    }
    M = warp_max(M);
    float L = 0.f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    constexpr int U = 4;
    for (int g0 = c0; g0 <= c1; g0 += 128) {
        float2 ml[4];
        if (g0 == c0) {
#pragma unroll
            for (int u = 0; u < 4; ++u) ml[u] = ml0[u];
        } else {
            load_ml(g0, ml);
        }
        float f[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            f[u] = (ml[u].x == -INFINITY) ? 0.f : expf(ml[u].x - M);
            if (g0 + lane + 32 * u <= c1) L += (ml[u].x == -INFINITY) ? 0.f : ml[u].y * f[u];
        }
        const int gend = min(c1, g0 + 127);
        float4 b0[U], b1[U];
        auto load_batch = [&](int cb, float4 (&dst)[U]) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = cb + u;
                dst[u] = c <= gend ? *reinterpret_cast<const float4*>(a.part_acc + (base + c) * kHD + lane * 4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        auto add_batch = [&](int cb, const float4 (&src)[U]) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int rel = cb + u - g0;  // factor of this chunk: lane rel % 32, slot rel / 32
                const int sl = (rel >> 5) & 3;
                const float fv =
                    __shfl_sync(0xffffffffu, sl == 0 ? f[0] : sl == 1 ? f[1] : sl == 2 ? f[2] : f[3], rel & 31);
                const float fu = cb + u <= gend ? fv : 0.f;
                o[0] = fmaf(src[u].x, fu, o[0]);
                o[1] = fmaf(src[u].y, fu, o[1]);
                o[2] = fmaf(src[u].z, fu, o[2]);
                o[3] = fmaf(src[u].w, fu, o[3]);
            }
        };
        load_batch(g0, b0);
        for (int cb = g0; cb <= gend; cb += 2 * U) {
            if (cb + U <= gend) load_batch(cb + U, b1);
            add_batch(cb, b0);
            if (cb + 2 * U <= gend) load_batch(cb + 2 * U, b0);
            if (cb + U <= gend) add_batch(cb + U, b1);
        }
    }
    L = warp_sum(L);
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

}  // namespace sd
