// sd_common.cuh -- shared device helpers for the sm_100a speculative-decode kernels.
//
// Inline-PTX wrappers for the pieces the kernels are built from: the int8 tensor-core MMA
// (m16n8k32, u8 x s8 -> s32), mbarriers with bounded waits, 1-D bulk async copies (TMA engine,
// global -> shared, no cluster multicast), and programmatic dependent launch (griddepcontrol).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "sd_internal.h"

namespace sd {

// ---------------------------------------------------------------------------------------------
// Device error word (one per context).  Kernels never trap: a wait that runs out sets a code here
// and the kernel returns; the host reads it after the stream synchronises.
// ---------------------------------------------------------------------------------------------
enum : int {
    DEV_ERR_NONE = 0,
    DEV_ERR_FULL_WAIT = 1,     // consumer gave up waiting for a weight stage
    DEV_ERR_EMPTY_WAIT = 2,    // producer gave up waiting for a free ring slot
    DEV_ERR_BAD_ARG = 3,       // a kernel found an argument outside its contract
    DEV_ERR_PEER_WAIT = 4,     // a cross-GPU flag wait gave up
};

// 2^24 polls of try_wait (each poll may itself block for a short hardware-defined window): seconds,
// far beyond any legitimate wait in these kernels.
constexpr uint32_t kSpinLimit = 1u << 24;

__device__ __forceinline__ void set_dev_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Any legitimate wait in these kernels is far below this; a wait that reaches it gives up.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Bounded wait: returns false if the phase did not complete within kWaitLimitNs.  (A try_wait with a
// suspend-time hint measured 1.6 % slower on the whole forward than polling: the waiting warps are the
// ones that resume work first.)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > kWaitLimitNs) return false;
    return true;
}

// Position in an n-slot mbarrier ring without per-step division: slot index and the phase parity of
// the slot's current use.
struct RingPos {
    int slot = 0;
    uint32_t phase = 0;
    __device__ __forceinline__ void advance(int n) {
        if (++slot == n) {
            slot = 0;
            phase ^= 1;
        }
    }
};

// ---------------------------------------------------------------------------------------------
// 1-D bulk copy global -> shared through the TMA engine, completing on an mbarrier (transaction
// bytes).  Both addresses 16-byte aligned, size a multiple of 16.  No multicast.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch.  wait: block until the preceding grid in the stream has completed
// and its memory is visible.  launch_dependents: allow the next grid to be scheduled.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------
// int8 tensor-core MMA: D[16x8] (s32) = A[16x32] (u8, row) * B[32x8] (s8, col) + C.
// Fragment ownership (lane = 4*g + t): a0 = A[g][4t..4t+3], a1 = A[g+8][4t..], a2 = A[g][16+4t..],
// a3 = A[g+8][16+4t..]; b0 = B[4t..4t+3][g], b1 = B[16+4t..][g];
// c0/d0 = (g, 2t), c1 = (g, 2t+1), c2 = (g+8, 2t), c3 = (g+8, 2t+1).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, int c0, int c1, int c2, int c3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Q8_0 quantisation of one 32-value block held one value per lane (lane j = element j), following
// the reference quantizer (mistral/dequant.h:545-599): d = amax/127 (IEEE divide), id = 1/d,
// q = saturate_s8(round_to_nearest_even(x * id)); amax == 0 -> d = 0, q = 0.
// Returns the code; *d_out and *sum_out (sum of the 32 codes) are valid in every lane.
__device__ __forceinline__ int q8_quant_lane(float x, float* d_out, int* sum_out) {
    float amax = warp_max(fabsf(x));
    float d = __fdiv_rn(amax, 127.0f);
    int q = 0;
    if (amax != 0.0f) {
        float id = __fdiv_rn(1.0f, d);
        int r = __float2int_rn(__fmul_rn(x, id));
        q = r > 127 ? 127 : (r < -128 ? -128 : r);
    }
    *d_out = d;
    *sum_out = warp_sum_i(q);
    return q;
}

}  // namespace sd
