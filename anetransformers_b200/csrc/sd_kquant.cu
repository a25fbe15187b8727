// sd_kquant.cu -- K-quant matrices (Q6_K, Q4_K super-blocks of 256 values) with fp32 activations: the LM head of
// a GGUF whose output.weight is not Q4_0 (the real Mistral Q4_0 files ship a Q6_K LM head) and the stand-alone
// K-quant matvec.  The reference runs these through its fp32 path (mistral/mistral_model.h:1118-1121 ->
// q4_matvec, :211-242): Q6_K by q6_K_matvec_f32_neon (mistral/dequant.h:349-520), Q4_K by an fp16 dequant
// (dequant_q4_K_block_neon, :63-113) and an fp32 sgemv.
//
// Arithmetic (the CPU oracle does the same, so results agree bit for bit):
//   Q6_K weight n of a super-block: q = (low 4 bits | high 2 bits << 4) - 32, w = (d * sc[n / 16]) * q in fp32
//   (exact: q has 6 bits, d * sc at most 18);
//   Q4_K weight: fp16(fp16(q * fp16(d * sc)) - fp16(dmin * m)), the reference's fp16 arithmetic;
//   y = sum over the row of w * x, value n accumulated by fused multiply-add into lane n % 4 in increasing n,
//   the four lanes added pairwise -- the lane structure of the reference's NEON loop.
// The final RMSNorm before the head runs here too (k_final_norm), with the engine's canonical statistics order.
//
// Layouts in HBM: Q4_K rows stay as in the GGUF (144-byte blocks, 16-byte aligned when a row is); Q6_K blocks are
// padded from 210 to 224 bytes at load (ql 128 | qh 64 | scales 16 | d 2 | pad 14) so every field is reached by
// aligned 16-byte loads.
#include "sd_dev.cuh"
#include "sd_kquant.h"

namespace sd {

namespace {

constexpr int kKqThreads = 128;     // rows per CTA (one thread per row)
constexpr int kKqChunk = 1024;      // activation values staged per round (4 super-blocks)

__global__ void k_repack_q6k(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, size_t n_blocks) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    const uint8_t* s = src + b * kQ6KBytes;
    uint8_t* d = dst + b * kQ6KPadded;
    for (int i = 0; i < kQ6KBytes; ++i) d[i] = s[i];
    for (int i = kQ6KBytes; i < kQ6KPadded; ++i) d[i] = 0;
}

// xn[s] = RMSNorm(x[s]) * w, tokens s < n_valid: one CTA per token.  Statistics in the engine's canonical order
// (16-value group sums, then the groups lane-strided and the warp butterfly); xn = (x * s) * w, the reference's
// order (mistral/mistral_model.h:202-208).
__global__ void __launch_bounds__(256) k_final_norm(const float* __restrict__ x, const float* __restrict__ w,
                                                    float* __restrict__ xn, int dim, float eps, int S,
                                                    const DevCtrl* ctrl) {
    __shared__ float gss[kKqChunk];  // dim / 16 <= 1024
    __shared__ float scale;
    if (ctrl && ctrl->done) return;
    const int nv = ctrl ? min(ctrl->n_valid, S) : S;
    const int s = blockIdx.x;
    if (s >= nv) return;
    const float* xs = x + (size_t)s * dim;
    const int ng = dim >> 4;
    for (int g = threadIdx.x; g < ng; g += blockDim.x) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = xs[g * 16 + i];
        gss[g] = group16_sumsq(v);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        // lane l adds groups l, l + 32, ... in order, then the butterfly
        float t = 0.f;
        for (int g = threadIdx.x; g < ng; g += 32) t += gss[g];
        t = warp_sum(t);
        if (threadIdx.x == 0) scale = rms_scale(t, dim, eps);
    }
    __syncthreads();
    const float sc = scale;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) xn[(size_t)s * dim + i] = (xs[i] * sc) * w[i];
}

template <int NS>
__device__ __forceinline__ void kq_fma16(float (&acc)[NS][4], const float* xs, int n0, const float (&w)[16], int nv) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        if (s >= nv) break;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[s][i & 3] = fmaf(w[i], xs[s * kKqChunk + n0 + i], acc[s][i & 3]);
    }
}

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int i) {
    const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
    return (w >> (8 * (i & 3))) & 0xFF;
}

// One Q6_K super-block (padded layout) of this thread's row against the staged activations at xs + base.
template <int NS>
__device__ __forceinline__ void q6k_block(const uint8_t* blk, const float* xs, int base, float (&acc)[NS][4], int nv) {
    const uint4* p = reinterpret_cast<const uint4*>(blk);
    const uint4 sc4 = __ldg(p + 12);  // scales[16]
    const uint4 dd = __ldg(p + 13);   // d (low half of the first word)
    const float d = __half2float(__ushort_as_half((unsigned short)(dd.x & 0xFFFF)));
    uint4 qh[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) qh[k] = __ldg(p + 8 + k);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {  // values 64 g .. 64 g + 63 in order
        const int qlo = (g & 1) * 4;                 // ql[0..63] for g = 0, 2; ql[64..127] for g = 1, 3
        const int nib = g >> 1;                       // low nibbles for g < 2, high above
        const int hsh = 2 * (g >> 1) + 4 * (g & 1);   // qh shift 0, 4, 2, 6
#pragma unroll
        for (int sb = 0; sb < 4; ++sb) {
            const uint4 ql = __ldg(p + qlo + sb);
            const int8_t scv = (int8_t)byte_of(sc4, 4 * g + sb);
            const float ds = d * (float)scv;
            float w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t lb = byte_of(ql, i);
                const uint32_t lo = nib ? (lb >> 4) : (lb & 0xF);
                const uint32_t hi = (byte_of(qh[sb], i) >> hsh) & 3;
                w[i] = ds * (float)((int)(lo | (hi << 4)) - 32);
            }
            kq_fma16<NS>(acc, xs, base + 64 * g + 16 * sb, w, nv);
        }
    }
}

template <int NS>
__device__ __forceinline__ void q4k_block(const uint8_t* blk, const float* xs, int base, float (&acc)[NS][4], int nv) {
    const uint4* p = reinterpret_cast<const uint4*>(blk);
    const uint4 hd = __ldg(p);  // d, dmin, scales[12]
    uint8_t sc[12];
#pragma unroll
    for (int i = 0; i < 12; ++i) sc[i] = (uint8_t)byte_of(hd, 4 + i);
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
        int s1, m1, s2, m2;
        q4k_scale_min(2 * j, sc, s1, m1);
        q4k_scale_min(2 * j + 1, sc, s2, m2);
        const float vd1 = __half2float(__float2half_rn(d * (float)s1)), vm1 = __half2float(__float2half_rn(dmin * (float)m1));
        const float vd2 = __half2float(__float2half_rn(d * (float)s2)), vm2 = __half2float(__float2half_rn(dmin * (float)m2));
        const uint4 q0 = __ldg(p + 1 + 2 * j), q1 = __ldg(p + 2 + 2 * j);
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // the 32 low nibbles, then the 32 high nibbles
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint4& qq = part ? q1 : q0;
                float w[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t b = byte_of(qq, i);
                    w[i] = half ? q4k_weight(b >> 4, vd2, vm2) : q4k_weight(b & 0xF, vd1, vm1);
                }
                kq_fma16<NS>(acc, xs, base + 64 * j + 32 * half + 16 * part, w, nv);
            }
        }
    }
}

// y[s][row] = W[row] . xn[s], one thread per row, NS tokens (n_valid of them real).
template <int TYPE, int NS>
__global__ void __launch_bounds__(kKqThreads) k_kq_matvec(const uint8_t* __restrict__ W, size_t row_bytes, int rows,
                                                          int in, const float* __restrict__ xn, float* __restrict__ y,
                                                          int ld_y, const DevCtrl* ctrl) {
    __shared__ __align__(16) float xs[NS * kKqChunk];
    if (ctrl && ctrl->done) return;
    const int nv = ctrl ? min(ctrl->n_valid, NS) : NS;
    const int row = blockIdx.x * kKqThreads + threadIdx.x;
    float acc[NS][4];
#pragma unroll
    for (int s = 0; s < NS; ++s) acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0.f;
    constexpr int kBlock = TYPE == kTypeQ6K ? kQ6KPadded : kQ4KBytes;
    const uint8_t* wrow = W + (size_t)(row < rows ? row : 0) * row_bytes;
    for (int c0 = 0; c0 < in; c0 += kKqChunk) {
        const int cn = min(kKqChunk, in - c0);
        __syncthreads();
        for (int i = threadIdx.x; i < NS * kKqChunk / 4; i += kKqThreads) {
            const int s = i / (kKqChunk / 4), k4 = (i % (kKqChunk / 4)) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (s < nv && k4 < cn) v = *reinterpret_cast<const float4*>(xn + (size_t)s * in + c0 + k4);
            *reinterpret_cast<float4*>(xs + s * kKqChunk + k4) = v;
        }
        __syncthreads();
        if (row < rows) {
            for (int b = 0; b < cn / 256; ++b) {
                const uint8_t* blk = wrow + (size_t)((c0 >> 8) + b) * kBlock;
                if constexpr (TYPE == kTypeQ6K) q6k_block<NS>(blk, xs, 256 * b, acc, nv);
                else q4k_block<NS>(blk, xs, 256 * b, acc, nv);
            }
        }
    }
    if (row < rows) {
#pragma unroll
        for (int s = 0; s < NS; ++s)
            if (s < nv) y[(size_t)s * ld_y + row] = (acc[s][0] + acc[s][1]) + (acc[s][2] + acc[s][3]);
    }
}

template <int TYPE>
cudaError_t launch_kq_t(const uint8_t* W, size_t row_bytes, int rows, int in, const float* xn, float* y, int ld_y, int S,
                        const DevCtrl* ctrl, cudaStream_t st) {
    const dim3 grid((rows + kKqThreads - 1) / kKqThreads);
    switch (S) {
        case 1: k_kq_matvec<TYPE, 1><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
        case 2: k_kq_matvec<TYPE, 2><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
        case 3: k_kq_matvec<TYPE, 3><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
        case 4: k_kq_matvec<TYPE, 4><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
        case 5: k_kq_matvec<TYPE, 5><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
        case 6: k_kq_matvec<TYPE, 6><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
        case 7: k_kq_matvec<TYPE, 7><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
        default: k_kq_matvec<TYPE, 8><<<grid, kKqThreads, 0, st>>>(W, row_bytes, rows, in, xn, y, ld_y, ctrl); break;
    }
    return cudaGetLastError();
}

}  // namespace

size_t kq_device_row_bytes(int type, int in) {
    return (size_t)(in / 256) * (type == kTypeQ6K ? kQ6KPadded : kQ4KBytes);
}

cudaError_t launch_repack_q6k(const uint8_t* src, uint8_t* dst, size_t n_blocks, cudaStream_t st) {
    k_repack_q6k<<<(unsigned)((n_blocks + 255) / 256), 256, 0, st>>>(src, dst, n_blocks);
    return cudaGetLastError();
}

cudaError_t launch_final_norm(const float* x, const float* w, float* xn, int dim, float eps, int S, const DevCtrl* ctrl,
                              cudaStream_t st) {
    if (dim % 16 || dim / 16 > kKqChunk) return cudaErrorInvalidValue;
    k_final_norm<<<S, 256, 0, st>>>(x, w, xn, dim, eps, S, ctrl);
    return cudaGetLastError();
}

cudaError_t launch_kq_matvec(int type, const uint8_t* W, int rows, int in, const float* xn, float* y, int ld_y, int S,
                             const DevCtrl* ctrl, cudaStream_t st) {
    if (in % 256 || S < 1 || S > kMaxS) return cudaErrorInvalidValue;
    const size_t rb = kq_device_row_bytes(type, in);
    if (type == kTypeQ6K) return launch_kq_t<kTypeQ6K>(W, rb, rows, in, xn, y, ld_y, S, ctrl, st);
    if (type == kTypeQ4K) return launch_kq_t<kTypeQ4K>(W, rb, rows, in, xn, y, ld_y, S, ctrl, st);
    return cudaErrorInvalidValue;
}

}  // namespace sd
