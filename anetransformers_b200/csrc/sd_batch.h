// sd_batch.h -- internal definitions of the batched (multi-stream) verify path: the wide-token W4A8 GEMM
// (sd_wgemm.cu) and the per-token kernels and engine of sd_batch.cu.
#pragma once
#include "sd_attn.h"

namespace sd {

// ---------------------------------------------------------------------------------------------
// Wide GEMM: Y[m][row] = sum_b (wd[row,b] * xd[m,b]) * isum[row,m,b] over M tokens.
//
// Weights in the "wide" layout (repacked from tile16x4 when a batch is created): per row tile of 128 rows
// (8 row-groups) and quad q, 9216 bytes = [half hh = 0, 1][block bq = 0..3] segments of 1152 bytes:
//   [0, 512)     lane L = 4g + t: 16 bytes = word t of block bq of row 16 r + g, r = 0..3 (row-group 4hh + r)
//   [512, 1024)  the same for rows 16 r + 8 + g
//   [1024, 1152) g = 0..7: 16 bytes = fp16 (wd(row 16r + g), wd(row 16r + 8 + g)) of block bq, r = 0..3
// so the warp that owns a half reads its A words of one block with two conflict-free 16-byte loads and its
// scales with one, and a stage's weights are one contiguous bulk copy.  Row tiles are zero-padded.
// ---------------------------------------------------------------------------------------------
constexpr int kWgWarps = 16;                      // 2 row halves x 8 token groups; warp 0 lane 0 also produces
constexpr int kWgThreads = kWgWarps * 32;
constexpr int kWgRG = 8;                          // row-groups per row tile (128 rows)
constexpr int kWgMaxN8 = 2;                       // n8 tiles per warp at most
constexpr int kWgTokGroups = 8;
constexpr int kWgMaxTT = kWgTokGroups * kWgMaxN8; // n8 tiles per token tile at most (128 tokens)
constexpr int kWgWStage = kWgRG * kTileBytes;     // 9216
constexpr int kWgMaxStages = 8;

inline int wide_row_tiles(int rows) { return (qmat_row_groups(rows) + kWgRG - 1) / kWgRG; }
inline size_t wide_bytes(int rows, int cols) { return (size_t)wide_row_tiles(rows) * (cols / 128) * kWgWStage; }

enum WGemmEpi : int {
    WG_STORE = 0,  // out[kpart][m][row] = partial over the K slice
    WG_SILU = 1,   // gate|up rows interleaved in 64-row units -> SiLU(gate)*up -> Q8_0 wide image
};

struct WGemmArgs {
    const uint8_t* w;   // wide-layout matrix
    int n_rt, nq;       // row tiles, quads per row (K / 128)
    const uint8_t* act; // wide image of the input (K = nq * 128)
    int NT, M;          // n8 tiles of the image, tokens
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
// The same GEMM on tcgen05 (sd_tcgemm.cu): WGemmArgs with tt_n8 even and <= kTcMaxTT, stage_bytes =
// kWgWStage + tt_n8 * kWSeg + 16384, the activation image in the tensor-core arrangement (WImg::tc).
constexpr int kTcMaxTT = 16;      // n8 tiles per token tile (128 tokens)
constexpr int kTcMinTokens = 64;  // forwards of at least this many tokens take the tcgen05 GEMM by default
constexpr int kTcMaxStages = 4;
constexpr int kTcAStage = 4 * 4096;
size_t tcgemm_smem_bytes(int tt_n8, int nstage, int epi);
cudaError_t tcgemm_init_attrs(int max_smem);
cudaError_t launch_tcgemm(int epi, const WGemmArgs& a, int grid, size_t smem, cudaStream_t st);
cudaError_t wgemm_init_attrs(int max_smem);
cudaError_t launch_wgemm(int epi, const WGemmArgs& a, int grid, size_t smem, cudaStream_t st);
// tile16x4 matrix (n_rg row-groups, nq quads) -> wide layout (zero-padded row tiles)
cudaError_t launch_wide_repack(const uint8_t* tiles, int n_rg, int nq, uint8_t* wide, cudaStream_t st);

}  // namespace sd
