// sd_batch.h -- internal definitions of the batched (multi-stream) verify path: the wide-token W4A8 GEMM
// (sd_wgemm.cu) and the per-token kernels and engine of sd_batch.cu.
#pragma once
#include "sd_attn.h"

namespace sd {

// ---------------------------------------------------------------------------------------------
// Wide GEMM: Y[m][row] = sum_b (wd[row,b] * xd[m,b]) * isum[row,m,b] over M tokens.
// ---------------------------------------------------------------------------------------------
constexpr int kWgWarps = 8;                       // consumer warps: 2 row halves x 4 token quarters
constexpr int kWgThreads = (kWgWarps + 1) * 32;   // + 1 producer warp
constexpr int kWgRG = 8;                          // row-groups per row tile (128 rows)
constexpr int kWgMaxN8 = 5;                       // n8 tiles per warp at most
constexpr int kWgMaxTT = 4 * kWgMaxN8;            // n8 tiles per token tile at most (160 tokens)
constexpr int kWgWStage = kWgRG * kTileBytes;     // 9216
constexpr int kWgMaxStages = 8;

enum WGemmEpi : int {
    WG_STORE = 0,  // out[kpart][m][row] = partial over the K slice
    WG_SILU = 1,   // gate|up rows interleaved in 64-row units -> SiLU(gate)*up -> Q8_0 wide image
};

struct WGemmArgs {
    const uint8_t* w;   // tile16x4 matrix
    int n_rg, nq;       // row-groups (allocated), quads per row (K / 128)
    const uint8_t* act; // wide image of the input (K = nq * 128)
    int NT, M;          // n8 tiles of the image, tokens
    int n_rt;           // row tiles (kWgRG row-groups each)
    int tt_n8;          // n8 tiles per token tile (<= kWgMaxTT)
    int n_tt;           // token tiles
    int kparts;         // K slices (WG_STORE)
    int nstage;
    int stage_bytes;    // kWgWStage + tt_n8 * kWSeg
    // WG_STORE
    float* out;
    int ld, out_rows;
    size_t part_stride; // floats between the outputs of consecutive K slices
    // WG_SILU
    WImg h;
    int hidden;
    int* err;
};

size_t wgemm_smem_bytes(int tt_n8, int nstage);
cudaError_t wgemm_init_attrs(int max_smem);
cudaError_t launch_wgemm(int epi, const WGemmArgs& a, int grid, size_t smem, cudaStream_t st);

}  // namespace sd
