// sd_dev.cuh -- device building blocks shared by the stand-alone kernels (sd_gemv.cu, sd_attn.cu,
// sd_quant.cu) and the persistent forward kernel (sd_fwd.cu).  Both paths run the same code in the same
// reduction orders, so they produce bit-identical results.
#pragma once
#include "sd_batch.h"
#include "sd_common.cuh"

namespace sd {

// The MMA accumulator is initialised with the bits of kMagic = 1.5*2^23: the result bits are then the fp32
// value kMagic + sum(q*x) (q the 0..15 nibbles; exact, |sum| < 2^16), and one exact FADD of
// -(kMagic + 8*sum(x)) recovers (float)isum = sum((q-8)*x) without the quarter-rate I2F conversion.
constexpr int kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float2 h2x2f(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// ---------------------------------------------------------------------------------------------
// Matvec activation fragments in shared memory, for one K slice of nb Q8_0 blocks.  Every block holds
// all kMaxS token slots (tokens >= the valid count are zero), so a lane's fragment address does not
// depend on S:
//   b[blk*kActStride + 4s + tt] = (word tt, word 4+tt) of token s's codes in block blk  (MMA B fragment)
//   m[blk*4 + t]                = (xd of token 2t, xd of token 2t+1, -(kMagic + 8*sum) of 2t, of 2t+1)
// ---------------------------------------------------------------------------------------------
constexpr int kActStride = 4 * kMaxS;

struct ActSmem {
    uint2* b;
    float4* m;
};

__host__ __device__ inline size_t act_smem_bytes(int nb) { return (size_t)nb * kActStride * 8 + (size_t)nb * 4 * 16; }

__device__ inline ActSmem act_smem_at(uint8_t* base, int nb) {
    ActSmem A;
    A.b = reinterpret_cast<uint2*>(base);
    A.m = reinterpret_cast<float4*>(base + (size_t)nb * kActStride * 8);
    return A;
}

// Offset term of a token's block with code sum `sum` (see kMagicI).
__host__ __device__ inline float act_offset(int sum) { return -(kMagicF + 8.0f * (float)sum); }

// The same fragment layout in global memory for a whole K range (nbK blocks): written by the phase that
// produces the activations so that staging a K slice is three contiguous bulk copies.
//   b: [nbK][kActStride] uint2, m: [nbK][4] float4 (scales before any norm scale, offsets)
__host__ __device__ inline size_t act_image_bytes(int nbK) { return act_smem_bytes(nbK); }

__host__ __device__ inline ActImage act_image_at(void* base, int nbK) {
    ActImage im;
    im.b = reinterpret_cast<uint2*>(base);
    im.m = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(base) + (size_t)nbK * kActStride * 8);
    return im;
}

// Code word w (elements 4w..4w+3, packed little-endian) of token s in block blk.
__device__ __forceinline__ void image_put_word(const ActImage& im, int s, int blk, int w, uint32_t word) {
    reinterpret_cast<uint32_t*>(im.b + (size_t)blk * kActStride + 4 * s + (w & 3))[w >> 2] = word;
}

// Codes of one block held one per lane (lane = element); the whole warp calls this.
__device__ __forceinline__ void image_put_codes_lane(const ActImage& im, int s, int blk, int lane, int code) {
    uint32_t v = (uint32_t)(code & 0xFF) << (8 * (lane & 3));
    v |= __shfl_xor_sync(0xffffffffu, v, 1);
    v |= __shfl_xor_sync(0xffffffffu, v, 2);
    if ((lane & 3) == 0) image_put_word(im, s, blk, lane >> 2, v);
}

// Block scale d and code sum of token s in block blk.
__device__ __forceinline__ void image_put_meta(const ActImage& im, int s, int blk, float d, int sum) {
    float* mp = reinterpret_cast<float*>(im.m + (size_t)blk * 4 + (s >> 1));
    mp[s & 1] = d;
    mp[(s & 1) + 2] = act_offset(sum);
}

// The same writes into a wide image (sd_batch.h) for token m.
__device__ __forceinline__ uint8_t* wimg_seg(const WImg& im, int m, int blk) {
    return im.p + ((size_t)(blk >> 2) * im.NT + (m >> 3)) * kWSeg;
}
__device__ __forceinline__ void wimg_put_word(const WImg& im, int m, int blk, int w, uint32_t word) {
    if (im.tc)
        reinterpret_cast<uint32_t*>(wimg_seg(im, m, blk) + (blk & 3) * 256 + (w >> 2) * 128 + (m & 7) * 16)[w & 3] = word;
    else
        reinterpret_cast<uint32_t*>(wimg_seg(im, m, blk) + (blk & 3) * 256 + (4 * (m & 7) + (w & 3)) * 8)[w >> 2] = word;
}
__device__ __forceinline__ void wimg_put_meta(const WImg& im, int m, int blk, float d, int sum) {
    float* mp = reinterpret_cast<float*>(wimg_seg(im, m, blk) + 1024 + (blk & 3) * 64 + ((m & 7) >> 1) * 16);
    mp[m & 1] = d;
    mp[(m & 1) + 2] = act_offset(sum);
}

// Stage Q8 planes (global, row stride K) blocks [kb0, kb0 + nb) of tokens < nv into A.  Loads are
// issued in batches before any store, so a staging costs about one memory round trip.
// The code slots of tokens >= nv are left as they are: each MMA output column depends only on its own
// token's fragments, and no epilogue reads the columns of tokens >= nv.
// tok_scale (optional, shared memory): per-token factor applied to the block scales (the RMSNorm
// scale when the planes hold Q8_0 of x*w).
__device__ inline void stage_act_from_planes(const ActSmem& A, const Q8Planes& act, int K, int kb0, int nb, int S, int nv,
                                             int tid, int nthr, const float* tok_scale = nullptr) {
    // Codes, three tokens or more: one warp per block at a time, lane l = 4 s + tt building the B-fragment pair
    // (word tt, word 4 + tt) of token s -- one 8-byte shared store per lane, the block's 256 bytes contiguous (no bank
    // conflicts); each warp's loads for up to eight blocks are issued before its stores.  Fewer tokens would leave
    // most lanes idle: 16-byte pieces per thread then (below).
    if (nv >= 3) {
        constexpr int UB = 8;
        const int lane = tid & 31, w = tid >> 5, nw = nthr >> 5;
        const int s = lane >> 2, tt = lane & 3;
        if (s < nv) {
            const uint8_t* src = reinterpret_cast<const uint8_t*>(act.qs) + (size_t)s * K + (size_t)kb0 * 32 + 4 * tt;
            for (int b0 = w; b0 < nb; b0 += UB * nw) {
                uint32_t lo[UB], hi[UB];
#pragma unroll
                for (int u = 0; u < UB; ++u) {
                    const int b = b0 + u * nw;
                    lo[u] = hi[u] = 0;
                    if (b < nb) {
                        lo[u] = *reinterpret_cast<const uint32_t*>(src + (size_t)b * 32);
                        hi[u] = *reinterpret_cast<const uint32_t*>(src + (size_t)b * 32 + 16);
                    }
                }
#pragma unroll
                for (int u = 0; u < UB; ++u) {
                    const int b = b0 + u * nw;
                    if (b < nb) A.b[(size_t)b * kActStride + lane] = make_uint2(lo[u], hi[u]);
                }
            }
        }
    } else {
        constexpr int U = 4;
        const int n16 = nv * nb * 2;  // 16-byte halves of the valid tokens' blocks
        for (int i0 = tid; i0 < n16; i0 += U * nthr) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * nthr;
                v[u] = make_uint4(0, 0, 0, 0);
                if (i < n16) {
                    const int s = i / (nb * 2), rem = i - s * (nb * 2);
                    v[u] = *reinterpret_cast<const uint4*>(act.qs + (size_t)s * K + (size_t)(kb0 + (rem >> 1)) * 32 +
                                                           (rem & 1) * 16);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * nthr;
                if (i < n16) {
                    const int s = i / (nb * 2), rem = i - s * (nb * 2);
                    uint32_t* base = reinterpret_cast<uint32_t*>(A.b + (size_t)(rem >> 1) * kActStride + 4 * s) + (rem & 1);
                    base[0] = v[u].x;
                    base[2] = v[u].y;
                    base[4] = v[u].z;
                    base[6] = v[u].w;
                }
            }
        }
    }
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
                float d0 = dv[u][0], d1 = dv[u][1];
                if (tok_scale) {
                    const int tt = i & 3;
                    if (2 * tt < nv) d0 = d0 * tok_scale[2 * tt];
                    if (2 * tt + 1 < nv) d1 = d1 * tok_scale[2 * tt + 1];
                }
                A.m[i] = make_float4(d0, d1, act_offset(sm[u][0]), act_offset(sm[u][1]));
            }
        }
    }
}

// One consumer warp's share of a ring slot: its 1152-byte tile of each of the kRPW row-groups of the
// pair (tile r at slot + r*half_bytes + warp*kTileBytes).  Loaded into registers so that the slot can
// be released before the math.
struct TileRegs {
    uint4 wl[kRPW], wh[kRPW];
    uint2 sl[kRPW], sh[kRPW];
};

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}

__device__ __forceinline__ void load_tiles(const uint8_t* slot, uint32_t half_bytes, int warp, int lane, TileRegs& tr) {
    const int g = lane >> 2;
    const uint32_t base = smem_u32(slot) + warp * kTileBytes;
#pragma unroll
    for (int r = 0; r < kRPW; ++r) {
        const uint32_t tile = base + r * half_bytes;
        tr.wl[r] = lds128(tile + lane * 16);
        tr.wh[r] = lds128(tile + 512 + lane * 16);
        const uint4 sc = lds128(tile + 1024 + g * 16);
        tr.sl[r] = make_uint2(sc.x, sc.y);
        tr.sh[r] = make_uint2(sc.z, sc.w);
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
    const uint32_t bf_a = smem_u32(A.b) + (bbase * kActStride + lane) * 8;  // token slot g, word pair t
    const uint32_t m_a = smem_u32(A.m) + (bbase * 4 + t) * 16;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const uint2 bf = lds64(bf_a + blk * kActStride * 8);
        const uint4 mu = lds128(m_a + blk * 64);
        const float2 xd = make_float2(__uint_as_float(mu.x), __uint_as_float(mu.y));
        const float2 off = make_float2(__uint_as_float(mu.z), __uint_as_float(mu.w));
#pragma unroll
        for (int r = 0; r < kRPW; ++r) {
            const uint32_t wlo = blk == 0 ? tr.wl[r].x : blk == 1 ? tr.wl[r].y : blk == 2 ? tr.wl[r].z : tr.wl[r].w;
            const uint32_t whi = blk == 0 ? tr.wh[r].x : blk == 1 ? tr.wh[r].y : blk == 2 ? tr.wh[r].z : tr.wh[r].w;
            const uint32_t a0 = wlo & 0x0F0F0F0Fu, a2 = (wlo >> 4) & 0x0F0F0F0Fu;
            const uint32_t a1 = whi & 0x0F0F0F0Fu, a3 = (whi >> 4) & 0x0F0F0F0Fu;
            int d[4];
            mma_u8s8(d, a0, a1, a2, a3, bf.x, bf.y, kMagicI, kMagicI, kMagicI, kMagicI);
            if constexpr (BLOCKSUMS) {
                if (t == 0 && (rg + r) * kTileRows < out_rows) {
                    const int r0 = (rg + r) * kTileRows + g;
                    isum[(size_t)r0 * nbK + kb0 + bbase + blk] = (int)(__int_as_float(d[0]) + off.x);
                    isum[(size_t)(r0 + 8) * nbK + kb0 + bbase + blk] = (int)(__int_as_float(d[2]) + off.x);
                }
            } else {
                const float wdl = (blk & 1) ? dl[r][blk >> 1].y : dl[r][blk >> 1].x;
                const float wdh = (blk & 1) ? dh[r][blk >> 1].y : dh[r][blk >> 1].x;
                const float2 fL = __fadd2_rn(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), off);
                const float2 fH = __fadd2_rn(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), off);
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

// SiLU(gate)*up + Q8_0 of one 32-unit block for the valid tokens r, r + 2, ... (epilogue warp r of 2; the
// epilogue is on the gate|up matvec's critical path, so tokens >= nv are skipped and the two warps alternate).
// ubuf: [4][128] = gate lo, gate hi, up lo, up hi (row*8 + tok).
__device__ __forceinline__ void epi_silu_q8(const float* ubuf, int r, int lane, int unit, int nv, Q8Planes h, int hidden,
                                            const ActImage* img = nullptr) {
    const int nbh = hidden >> 5;
    for (int k = 0; k < 4; ++k) {
        const int tok = r + 2 * k;  // tokens alternate between the two epilogue warps
        if (tok >= nv) break;
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
        if (img) {
            if (tok < nv) {
                image_put_codes_lane(*img, tok, unit, lane, q);
                if (lane == 0) image_put_meta(*img, tok, unit, dq, sq);
            }
        } else if (tok < nv) {
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

// Q4_K sub-block scale / min of index j (0..7) from the 12 packed bytes (mistral/dequant.h:47-55).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* q, int& d, int& m) {
    if (j < 4) {
        d = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Q4_K weight fp16(fp16(q * dsc) - dm) of the reference's fp16 dequant (mistral/dequant.h:63-113): products and
// differences of fp16 values rounded once to fp16 (evaluated in fp32, which holds the exact product of a 4-bit q
// and an fp16, and whose rounding before the fp16 one is harmless for a difference of two fp16 values).
__device__ __forceinline__ float q4k_weight(uint32_t q, float dsc, float dm) {
    const float p = __half2float(__float2half_rn((float)q * dsc));
    return __half2float(__float2half_rn(p - dm));
}

// Value `lane` of 32-value block blk of token `token`'s embedding row: Q4_0 (type 2) or Q4_K (type 12, the
// reference's fp16 dequant, mistral/mistral_model.h:146-156).
__device__ __forceinline__ float embed_value(const uint8_t* embd, int type, int token, int dim, int blk, int lane) {
    if (type == 12) {
        const uint8_t* b = embd + ((size_t)token * (dim >> 8) + (blk >> 3)) * 144;
        const int sb = blk & 7;
        int sc, m;
        q4k_scale_min(sb, b + 4, sc, m);
        const float d = __half2float(__ushort_as_half((unsigned short)(b[0] | (b[1] << 8))));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(b[2] | (b[3] << 8))));
        const float vd = __half2float(__float2half_rn(d * (float)sc));
        const float vm = __half2float(__float2half_rn(dmin * (float)m));
        const uint8_t byte = b[16 + 32 * (sb >> 1) + lane];
        return q4k_weight((sb & 1) ? (byte >> 4) : (byte & 0xF), vd, vm);
    }
    return q4_0_value(embd + ((size_t)token * (dim >> 5) + blk) * 18, lane);
}

// ---------------------------------------------------------------------------------------------
// Attention work item (kv head, chunk) for a group of 8 warps (256 threads), on the tensor cores.
//
// Query rows r = 4*s + h (token s < 8, query head h of the kv head: 32 rows = four 8-row n-tiles).
// The products run transposed, positions x rows: scores S^T = K Q^T and outputs O^T = V^T P^T, with
// mma.m16n8k16 (f16 inputs, f32 accumulate).  K and V are fp16 already; Q (fp32) and the probabilities
// P (fp32) are split into a high and a low fp16 part and both are multiplied, so products keep ~22 bits
// (fp32-class results).  Warp w owns n-tile w & 3 (tokens 2*(w&3), +1) and output dims 64*(w >> 2) .. +63:
// it computes the scores of its rows over each whole 32-position sub-block (the two warps of an n-tile
// compute the same scores and the same online softmax -- mistral/mistral_model.h:362-487 semantics, exp
// of score minus running max -- identically), so each warp holds its state and its 64 output dims in
// registers and the warps meet only to stage K/V.
// ---------------------------------------------------------------------------------------------
constexpr int kHD = 128;        // head_dim
constexpr int kGQA = 4;         // query heads per kv head
constexpr int kSub = 32;        // positions per sub-block
constexpr int kAttnThreads = 256;
constexpr int kQRows = kMaxS * kGQA;  // 32
constexpr int kQStride = kHD + 8;     // halves per Q / K / V row (conflict-free ldmatrix rows)

struct AttnSmem {
    __half* qh;     // [kQRows][kQStride] high part of q
    __half* ql;     // [kQRows][kQStride] low part
    __half* kk;     // [kSub][kQStride]  K sub-block (position-major)
    __half* vv;     // [kSub][kQStride]  V sub-block (position-major; fragments by ldmatrix.trans)
};

__host__ __device__ constexpr size_t attn_smem_bytes() {
    return (size_t)2 * kQRows * kQStride * 2 + (size_t)2 * kSub * kQStride * 2;
}

__device__ inline AttnSmem attn_smem_at(uint8_t* base) {
    AttnSmem s;
    s.qh = reinterpret_cast<__half*>(base);
    s.ql = s.qh + kQRows * kQStride;
    s.kk = s.ql + kQRows * kQStride;
    s.vv = s.kk + kSub * kQStride;
    return s;
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four 8x8 b16 matrices from shared memory; lanes 8i..8i+7 give the row addresses of matrix i.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// Transpose of an 8x8 b16 matrix held one row pair per lane (lane 4g+t: row g, columns 2t, 2t+1).
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// Start moving bytes (16-byte aligned, a multiple of 16) of global memory into L2; no completion.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// (x, y) -> high and low fp16x2 parts: hi = fp16(x), lo = fp16(x - hi).
__device__ __forceinline__ void split_f16x2(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    hi = h2u(h);
    lo = h2u(__floats2half2_rn(x - hf.x, y - hf.y));
}

// Ring slot of position p (0 <= p < 2 * max_seq).
__device__ __forceinline__ int ring_slot(int p, int max_seq) { return p < max_seq ? p : p - max_seq; }

// exp(x) as 2^(x log2 e) on the special-function unit (relative error ~1e-6 for the |x| of a softmax).
__device__ __forceinline__ float exp_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.44269504088896341f));
    return y;
}

// L2 prefetch of the K and V rows of kv head kvh at positions [p0, p1): one 256-byte row per thread per
// round of 128 positions, K by threads 0-127, V by 128-255.
__device__ __forceinline__ void attn_prefetch(const AttnArgs& a, int kvh, int p0, int p1, int tid) {
    for (int p = p0 + (tid & 127); p < p1; p += 128) {
        const size_t off = (size_t)ring_slot(p, a.max_seq) * a.kv_ld + (size_t)kvh * kHD;
        prefetch_l2((tid < 128 ? a.k : a.v) + off, kHD * 2);
    }
}

// Load one 32-position K/V sub-block into registers: this thread's pieces are positions sb + (tid >> 4) and
// +16, dims 8 * (tid & 15) .. +7 of the kv head whose first dim is at column col = kvh * 128 + 8 * (tid & 15).
__device__ __forceinline__ void attn_load_kv(const AttnArgs& a, uint32_t col, int sb, int p1, int tid, uint4 (&kr)[2],
                                             uint4 (&vr)[2]) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int p = sb + (tid >> 4) + 16 * u;
        kr[u] = vr[u] = make_uint4(0, 0, 0, 0);
        if (p < p1) {
            const size_t off = (size_t)ring_slot(p, a.max_seq) * a.kv_ld + col;
            kr[u] = *reinterpret_cast<const uint4*>(a.k + off);
            vr[u] = *reinterpret_cast<const uint4*>(a.v + off);
        }
    }
}

__device__ __forceinline__ void attn_store_kv(const AttnSmem& sm, int tid, const uint4 (&kr)[2], const uint4 (&vr)[2]) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int i = tid + u * kAttnThreads;
        const int j = i >> 4, d8 = (i & 15) * 8;
        *reinterpret_cast<uint4*>(sm.kk + j * kQStride + d8) = kr[u];
        *reinterpret_cast<uint4*>(sm.vv + j * kQStride + d8) = vr[u];
    }
}

// One work item: every query row (4 heads x nv tokens) of kv head kvh over chunk c.  The chunk's K/V rows
// (and those of the next item, nkvh / nc, if nc >= 0) are prefetched into L2 at the start; each sub-block's
// loads are issued before the previous sub-block's math so that their latency overlaps it.
// gsync(): a barrier over the group's 256 threads (tid = 0..255).
template <class Sync>
__device__ void attn_item(const AttnArgs& a, int nv, int pos, int lo_min, int hi_max, int kvh, int c, int nkvh, int nc,
                          const AttnSmem& sm, int tid, Sync gsync) {
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nt = warp & 3, dh = warp >> 2;
    const bool active = 2 * nt < nv;  // this n-tile holds a valid token
    const int p0 = max(c * a.chunk, lo_min);
    const int p1 = min((c + 1) * a.chunk, hi_max + 1);  // exclusive
    const int lo_max = max(0, pos + nv - a.max_seq);      // window start of the last valid token
    attn_prefetch(a, kvh, p0, p1, tid);
    if (nc >= 0) {
        // the next item's first 128 positions (its whole chunk when chunks are that short)
        const int np0 = max(nc * a.chunk, lo_min);
        attn_prefetch(a, nkvh, np0, min(min((nc + 1) * a.chunk, hi_max + 1), np0 + 128), tid);
    }
    uint4 kr[2], vr[2];
    float4 qv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = tid + u * kAttnThreads;  // < 32 rows * 32 float4
        const int r = i >> 5, d4 = (i & 31) * 4;
        const int s = r >> 2, h = r & 3;
        qv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s < nv) qv[u] = *reinterpret_cast<const float4*>(a.q + (size_t)s * a.q_ld + (size_t)(kvh * kGQA + h) * kHD + d4);
    }
    const uint32_t col = (uint32_t)(kvh * kHD + (tid & 15) * 8);
    attn_load_kv(a, col, p0, p1, tid, kr, vr);
    gsync();  // the previous item is done with the shared buffers
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = tid + u * kAttnThreads;
        const int r = i >> 5, d4 = (i & 31) * 4;
        uint32_t h0, l0, h1, l1;
        split_f16x2(qv[u].x, qv[u].y, h0, l0);
        split_f16x2(qv[u].z, qv[u].w, h1, l1);
        *reinterpret_cast<uint2*>(sm.qh + r * kQStride + d4) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(sm.ql + r * kQStride + d4) = make_uint2(l0, l1);
    }
    attn_store_kv(sm, tid, kr, vr);
    // ldmatrix row addresses (lane = 8 * lq + lr gives a row of matrix lq).
    //   K (A of S^T, positions x dims): matrices (pos +0, dims +0), (+8, +0), (+0, +8), (+8, +8).
    //   Q (B of S^T, dims x rows = Q rows): matrices at dims +0, +8 of the k-step (lanes 16-31 repeat 0-15).
    //   V (A of O^T via .trans, dims x positions): matrices (pos +0, dims +0), (+0, +8), (+8, +0), (+8, +8).
    const int lr = lane & 7, lq = lane >> 3;
    const uint32_t k_a = smem_u32(sm.kk + (lr + (lq & 1) * 8) * kQStride + (lq >> 1) * 8);
    const uint32_t qh_a = smem_u32(sm.qh + (nt * 8 + lr) * kQStride + (lq & 1) * 8);
    const uint32_t ql_a = qh_a + (uint32_t)(kQRows * kQStride * 2);
    const uint32_t v_a = smem_u32(sm.vv + (lr + (lq >> 1) * 8) * kQStride + dh * 64 + (lq & 1) * 8);
    // rows 2t, 2t+1 of the n-tile: running max, lane-partial sum (this lane's positions), outputs O^T
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    for (int sb = p0; sb < p1; sb += kSub) {
        const bool more = sb + kSub < p1;
        if (more) attn_load_kv(a, col, sb + kSub, p1, tid, kr, vr);  // lands while this sub-block is computed
        gsync();
        if (active) {
            // ---- S^T: positions sb + 16 mt + (g, g+8) x rows 8 nt + (2t, 2t+1), m-tiles mt = 0, 1 ----
            float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int ks = 0; ks < kHD / 16; ++ks) {
                uint32_t bh0, bh1, bl0, bl1;
                ldsm_x2(qh_a + ks * 32, bh0, bh1);
                ldsm_x2(ql_a + ks * 32, bl0, bl1);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t k0, k1, k2, k3;
                    ldsm_x4(k_a + (uint32_t)(mt * 16 * kQStride * 2) + ks * 32, k0, k1, k2, k3);
                    mma_f16(sc[mt], k0, k1, k2, k3, bh0, bh1);
                    mma_f16(sc[mt], k0, k1, k2, k3, bl0, bl1);
                }
            }
            // positions outside some valid row's window occur only in edge sub-blocks
            if (sb + kSub > p1 || sb + kSub - 1 > pos || sb < lo_max) {
                const int s = 2 * nt + (t >> 1);  // token of rows 2t, 2t+1
                const int hi = pos + s, lo = max(0, hi + 1 - a.max_seq);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int p = sb + mt * 16 + g + (e >> 1) * 8;
                        if (!(s < nv && p < p1 && p >= lo && p <= hi)) sc[mt][e] = -INFINITY;
                    }
            }
            // ---- online softmax over the sub-block: rows 2t (elements 0, 2), 2t+1 (elements 1, 3) ----
            float x0 = fmaxf(fmaxf(sc[0][0], sc[0][2]), fmaxf(sc[1][0], sc[1][2]));
            float x1 = fmaxf(fmaxf(sc[0][1], sc[0][3]), fmaxf(sc[1][1], sc[1][3]));
#pragma unroll
            for (int o2 = 4; o2 < 32; o2 <<= 1) {
                x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, o2));
                x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, o2));
            }
            const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
            // a row with nothing valid yet keeps m = -inf and contributes nothing
            const float c0 = (m0 == -INFINITY) ? 0.f : exp_fast(m0 - n0);
            const float c1 = (m1 == -INFINITY) ? 0.f : exp_fast(m1 - n1);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                sc[mt][0] = sc[mt][0] == -INFINITY ? 0.f : exp_fast(sc[mt][0] - n0);
                sc[mt][1] = sc[mt][1] == -INFINITY ? 0.f : exp_fast(sc[mt][1] - n1);
                sc[mt][2] = sc[mt][2] == -INFINITY ? 0.f : exp_fast(sc[mt][2] - n0);
                sc[mt][3] = sc[mt][3] == -INFINITY ? 0.f : exp_fast(sc[mt][3] - n1);
            }
            m0 = n0;
            m1 = n1;
            l0 = l0 * c0 + ((sc[0][0] + sc[0][2]) + (sc[1][0] + sc[1][2]));
            l1 = l1 * c1 + ((sc[0][1] + sc[0][3]) + (sc[1][1] + sc[1][3]));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                o[i][0] *= c0;
                o[i][1] *= c1;
                o[i][2] *= c0;
                o[i][3] *= c1;
            }
            // ---- O^T (dims 64 dh + 16 i + (g, g+8) x rows 2t, 2t+1) += V^T P^T, k-step = m-tile mt ----
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                // P^T (positions x rows) -> B fragments: b0 from positions g, b1 from g + 8
                uint32_t ph0, pl0, ph1, pl1;
                split_f16x2(sc[mt][0], sc[mt][1], ph0, pl0);
                split_f16x2(sc[mt][2], sc[mt][3], ph1, pl1);
                ph0 = movm_t(ph0);
                pl0 = movm_t(pl0);
                ph1 = movm_t(ph1);
                pl1 = movm_t(pl1);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint32_t v0, v1, v2, v3;
                    ldsm_x4_t(v_a + (uint32_t)(mt * 16 * kQStride * 2) + i * 32, v0, v1, v2, v3);
                    mma_f16(o[i], v0, v1, v2, v3, ph0, ph1);
                    mma_f16(o[i], v0, v1, v2, v3, pl0, pl1);
                }
            }
        }
        if (more) {
            gsync();  // every warp is done with this sub-block's K and V
            attn_store_kv(sm, tid, kr, vr);
        }
    }
    // ---- chunk partials: rows r0, r0 + 1 (token s, heads r0 & 3, +1), this warp's 64 dims ----
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o2);
    }
    const int r0 = nt * 8 + 2 * t;
    const int s = 2 * nt + (t >> 1);
    if (active && s < nv) {
        const size_t pi = ((size_t)s * a.n_heads + kvh * kGQA + (r0 & 3)) * a.max_chunks + c;
        float* acc0 = a.part_acc + pi * kHD + dh * 64;
        float* acc1 = acc0 + (size_t)a.max_chunks * kHD;  // next head, same token and chunk
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = 16 * i + g;
            acc0[d] = o[i][0];
            acc1[d] = o[i][1];
            acc0[d + 8] = o[i][2];
            acc1[d + 8] = o[i][3];
        }
        if (dh == 0 && g == 0) {
            a.part_ml[pi] = make_float2(m0, l0);
            a.part_ml[pi + a.max_chunks] = make_float2(m1, l1);
        }
    }
}

// Merge the chunk partials of (token s, head h) and quantise the 128 outputs to 4 Q8_0 blocks.
// nwc warps share the row (wi = this warp's index among them, lane owns dims 4*lane..4*lane+3):
//   1. every warp reads all (max, sum) pairs lane-parallel (128 chunks per round trip) -> M, in the same
//      round trip as its first eight chunk partials; warp 0: L (lane sums in chunk order, then the butterfly);
//   2. warp wi adds acc_c * exp(m_c - M) over its contiguous share of the chunks, in chunk order, eight
//      chunks' loads in flight at a time;
//   3. the partial vectors meet in obuf ([nwc][128], shared) behind rsync(); warp 0 adds them in warp
//      order, scales by 1/L and quantises.
// The result depends only on nwc, which both forward paths take from combine_warps(max_seq).
constexpr int kCombineWarpsMax = 16;
// Warps per merged row (8 measured 0.6 % faster than 4 on a whole forward at a 1K context; more for long
// rings, whose rows have many chunks).
__host__ __device__ inline int combine_warps(int max_seq) { return max_seq <= 8192 ? 8 : 16; }

template <class Sync>
__device__ void attn_combine_row(const AttnArgs& a, int nwc, int pos, int s, int h, int wi, int lane, float* obuf,
                                 Sync rsync) {
    const int hi = pos + s, lo = max(0, hi + 1 - a.max_seq);
    const int c0 = lo / a.chunk, c1 = hi / a.chunk;
    const size_t base = ((size_t)s * a.n_heads + h) * a.max_chunks;
    constexpr int kMl = 4;  // (max, sum) pairs per lane per round trip
    constexpr int U = 8;    // this warp's chunk partials per round trip
    // this warp's chunk range
    const int nc = c1 - c0 + 1, per = (nc + nwc - 1) / nwc;
    const int ca = c0 + wi * per, cb = min(c1, ca + per - 1);
    // One round trip for the common case: this warp's first U chunk partials (they do not depend on M) and
    // every chunk's (max, sum) pair are loaded together.
    float4 ac[U];
    float mx[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int c = ca + u;
        ac[u] = c <= cb ? *reinterpret_cast<const float4*>(a.part_acc + (base + c) * kHD + lane * 4)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        mx[u] = c <= cb ? a.part_ml[base + c].x : -INFINITY;
    }
    float M = -INFINITY, L = 0.f;
    float2 ml0[kMl];  // the first round's pairs, kept for L
#pragma unroll
    for (int u = 0; u < kMl; ++u) {
        const int c = c0 + lane + 32 * u;
        ml0[u] = c <= c1 ? a.part_ml[base + c] : make_float2(-INFINITY, 0.f);
        M = fmaxf(M, ml0[u].x);
    }
    for (int g0 = c0 + 32 * kMl; g0 <= c1; g0 += 32 * kMl) {
#pragma unroll
        for (int u = 0; u < kMl; ++u) {
            const int c = g0 + lane + 32 * u;
            M = fmaxf(M, c <= c1 ? a.part_ml[base + c].x : -INFINITY);
        }
    }
    M = warp_max(M);
    if (wi == 0) {
        // lane l adds chunks c0 + l + 32k in k order, then the butterfly
#pragma unroll
        for (int u = 0; u < kMl; ++u)
            if (c0 + lane + 32 * u <= c1) L += (ml0[u].x == -INFINITY) ? 0.f : ml0[u].y * expf(ml0[u].x - M);
        for (int g0 = c0 + 32 * kMl; g0 <= c1; g0 += 32 * kMl) {
            float2 ml[kMl];
#pragma unroll
            for (int u = 0; u < kMl; ++u) {
                const int c = g0 + lane + 32 * u;
                ml[u] = c <= c1 ? a.part_ml[base + c] : make_float2(-INFINITY, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kMl; ++u)
                if (g0 + lane + 32 * u <= c1) L += (ml[u].x == -INFINITY) ? 0.f : ml[u].y * expf(ml[u].x - M);
        }
        L = warp_sum(L);
    }
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int cc = ca; cc <= cb; cc += U) {
        if (cc > ca) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = cc + u;
                ac[u] = c <= cb ? *reinterpret_cast<const float4*>(a.part_acc + (base + c) * kHD + lane * 4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
                mx[u] = c <= cb ? a.part_ml[base + c].x : -INFINITY;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (cc + u > cb) break;
            const float f = (mx[u] == -INFINITY) ? 0.f : expf(mx[u] - M);
            o[0] = fmaf(ac[u].x, f, o[0]);
            o[1] = fmaf(ac[u].y, f, o[1]);
            o[2] = fmaf(ac[u].z, f, o[2]);
            o[3] = fmaf(ac[u].w, f, o[3]);
        }
    }
    *reinterpret_cast<float4*>(obuf + wi * kHD + lane * 4) = make_float4(o[0], o[1], o[2], o[3]);
    rsync();
    if (wi != 0) {
        rsync();  // obuf is free again once warp 0 has read it
        return;
    }
    for (int w = 1; w < nwc; ++w) {
        const float4 p = *reinterpret_cast<const float4*>(obuf + w * kHD + lane * 4);
        o[0] += p.x;
        o[1] += p.y;
        o[2] += p.z;
        o[3] += p.w;
    }
    rsync();
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
    if (a.img.b) {
        const int blk = h * (kHD / 32) + (lane >> 3);
        image_put_word(a.img, s, blk, lane & 7, packed);
        if ((lane & 7) == 0) image_put_meta(a.img, s, blk, d, qsum);
        return;
    }
    if (a.wimg.p) {
        const int blk = h * (kHD / 32) + (lane >> 3);
        wimg_put_word(a.wimg, a.tok0 + s, blk, lane & 7, packed);
        if ((lane & 7) == 0) wimg_put_meta(a.wimg, a.tok0 + s, blk, d, qsum);
        return;
    }
    *reinterpret_cast<uint32_t*>(a.out.qs + row_off + lane * 4) = packed;
    if ((lane & 7) == 0) {
        const size_t bi = row_off / 32 + (lane >> 3);
        a.out.d[bi] = d;
        a.out.sum[bi] = qsum;
    }
}

}  // namespace sd
