// sd_kquant.h -- K-quant (Q6_K, Q4_K) matrices with fp32 activations (sd_kquant.cu).
#pragma once
#include "sd_internal.h"

namespace sd {

// GGML type ids (mistral/gguf_loader.h:39-50)
constexpr int kTypeQ4_0 = 2, kTypeQ4K = 12, kTypeQ6K = 14;
constexpr int kQ4KBytes = 144;   // d, dmin (fp16), scales[12], qs[128]
constexpr int kQ6KBytes = 210;   // ql[128], qh[64], scales[16] (int8), d (fp16)
constexpr int kQ6KPadded = 224;  // device layout of a Q6_K block (16-byte aligned fields)

// Bytes of one row of `in` values in the device layout.
size_t kq_device_row_bytes(int type, int in);
// GGUF Q6_K blocks (device copy) -> the padded device layout.
cudaError_t launch_repack_q6k(const uint8_t* src, uint8_t* dst, size_t n_blocks, cudaStream_t st);
// xn[s] = RMSNorm(x[s]) * w for s < n_valid (ctrl, or all S when null).
cudaError_t launch_final_norm(const float* x, const float* w, float* xn, int dim, float eps, int S, const DevCtrl* ctrl,
                              cudaStream_t st);
// y[s][row] (row stride ld_y) = W[row] . xn[s] for s < n_valid; W in the device layout of `type`.
cudaError_t launch_kq_matvec(int type, const uint8_t* W, int rows, int in, const float* xn, float* y, int ld_y, int S,
                             const DevCtrl* ctrl, cudaStream_t st);

}  // namespace sd
