/*
 * compat/dequant.h -- drop-in for the reference's mistral/dequant.h entry points on the hot path.
 * Same type names, block layouts and signatures; the bodies run the B200 kernels through
 * libspecdec_b200.so.  Link with -lspecdec_b200.
 *   block_q4_0 / block_q8_0                 mistral/dequant.h:17-21, :537-541 (identical 18 / 36 B layouts;
 *                                           d of block_q4_0 is the fp16 bit pattern)
 *   quantize_f32_to_q8_0                    mistral/dequant.h:545-599
 *   q4_0_q8_0_matvec_sdot_parallel          mistral/dequant.h:1022-1137
 *   q4_0_q8_0_matvec_sdot                   mistral/dequant.h:614-719 (same result contract)
 * The matvec uploads and repacks W on first use per (address, shape) -- weights are immutable mmap'd
 * tensors in the reference -- so later calls only move x and y.
 */
#ifndef SPECDEC_COMPAT_DEQUANT_H
#define SPECDEC_COMPAT_DEQUANT_H
#include "../specdec_b200.h"

#define QK4_0 32
#define QK8_0 32

typedef sd_block_q4_0 block_q4_0;
typedef sd_block_q8_0 block_q8_0;

static inline void quantize_f32_to_q8_0(const float *x, block_q8_0 *out, int n) {
    sd_host_quantize_f32_to_q8_0(x, out, n);
}

static inline void q4_0_q8_0_matvec_sdot_parallel(const void *W_q4, const block_q8_0 *x_q8, float *y, int out_dim,
                                                  int in_dim) {
    sd_host_q4_0_q8_0_matvec(W_q4, x_q8, y, out_dim, in_dim);
}

static inline void q4_0_q8_0_matvec_sdot(const void *W_q4, const block_q8_0 *x_q8, float *y, int out_dim, int in_dim) {
    sd_host_q4_0_q8_0_matvec(W_q4, x_q8, y, out_dim, in_dim);
}

#endif
