// sd_internal.h -- internal (non-ABI) definitions shared by the CUDA sources of libspecdec_b200.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stddef.h>
#include <stdint.h>

namespace sd {

// ---------------------------------------------------------------------------------------------
// Repacked Q4_0 weight layout ("tile16x4") in HBM.
//
// A matrix [rows][cols] of 18-byte Q4_0 blocks is stored as row-groups of 16 rows; each row-group
// as cols/128 tiles ("quads" of 4 consecutive blocks), each tile 1152 bytes:
//   bytes [0, 1024): nibbles.  Half h (rows 8h..8h+7), lane L = 4*g + t (g = row in half, t = word):
//                    16 bytes at h*512 + L*16 = word t (qs[4t..4t+3]) of blocks 4q..4q+3 of row 8h+g.
//   bytes [1024, 1152): fp16 scales, [g][h][blk]: rows g and 8+g side by side, so a lane reads the scales of
//                    both its rows with one 16-byte load.
// Each lane of a warp then reads its int8 MMA A-fragment for 4 blocks with two conflict-free 16-byte
// loads, and one row-group's whole K range is contiguous (cols/128 * 1152 bytes), so a CTA's range of
// row-groups is one contiguous stream for the bulk-copy engine.
// ---------------------------------------------------------------------------------------------
constexpr int kTileRows = 16;
constexpr int kTileBytes = 1152;
constexpr int kConsumerWarps = 16;                       // one tile of each row-group per ring stage
constexpr int kEpiWarps = 2;                             // reduce + epilogue, one row-group each
constexpr int kGemvThreads = (kConsumerWarps + kEpiWarps + 1) * 32;  // + 1 producer warp
constexpr int kRedSlots = 2;                             // row-group pairs in flight to the epilogue
constexpr int kMaxStages = 16;
constexpr int kMaxS = 8;                                 // tokens per forward (n8 MMA tile)
// Tokens per verify: a batch of more than kMaxS tokens runs as consecutive forwards of <= kMaxS tokens
// (every reduction is batch invariant, so the logits equal those of one wide forward).
constexpr int kMaxVerify = 16;
constexpr int kRPW = 2;                                  // row-groups per warp per stage (share B fragments)

// Row-groups are allocated in whole pairs (a zero row-group pads an odd count).
inline int qmat_row_groups(int rows) {
    int n_rg = (rows + kTileRows - 1) / kTileRows;
    return (n_rg + kRPW - 1) / kRPW * kRPW;
}
inline size_t qmat_bytes(int rows, int cols) { return (size_t)qmat_row_groups(rows) * (cols / 128) * kTileBytes; }

// Row placement used while repacking: destination row of source row r is
//   (r / unit) * stride + offset + (r % unit)
struct RowMap {
    int unit, stride, offset;
};

// Activations in the matvec's shared-memory fragment layout, kept in global memory (sd_dev.cuh).
struct ActImage {
    uint2* b;
    float4* m;
};

// ---------------------------------------------------------------------------------------------
// Wide activation image: Q8_0 activations of M tokens over K columns in the GEMM's fragment layout.
// Tokens are grouped in n8 tiles (NT = ceil(M / 8)); for quad q (blocks 4q..4q+3) and n8 tile n the
// segment at ((size_t)q * NT + n) * kWSeg bytes holds
//   [0, 1024)    uint2 b[4][32]: entry 4s + tt of block bq = (word tt, word tt + 4) of token 8n + s's codes
//                (the int8 MMA B fragment of lane 4s + tt)
//   [1024, 1280) float4 m[4][4]: entry t of block bq = (xd(8n+2t), xd(8n+2t+1), off(8n+2t), off(8n+2t+1)),
//                off = -(kMagic + 8 * code sum) (sd_dev.cuh)
// so a CTA's stage (one quad of a range of n8 tiles) is one contiguous bulk copy.
// ---------------------------------------------------------------------------------------------
constexpr int kWSeg = 1280;

//
// Tensor-core arrangement (tc = 1; read by the tcgen05 GEMM): the same segments and meta, but the codes of
// block bq are [kc][8 tokens][16 bytes] at bq * 256 (kc = 0: elements 0..15, kc = 1: elements 16..31), the
// canonical K-major operand layout of tcgen05.mma (8-row x 16-byte core matrices).
struct WImg {
    uint8_t* p;
    int NT;
    int tc = 0;
};

inline size_t wimg_bytes(int M, int K) { return (size_t)(K / 128) * ((M + 7) / 8) * kWSeg; }

// Q8_0 activations on device as planes (codes, fp32 scale, per-block code sum).
struct Q8Planes {
    int8_t* qs;     // [S][n]
    float* d;       // [S][n/32]
    int32_t* sum;   // [S][n/32]
};

// Per-forward control block in device memory.  Kernels read positions / valid-token counts from it
// so a captured CUDA graph replays for any position.
struct DevCtrl {
    int pos;          // position of token 0 of this forward
    int n_valid;      // tokens of this forward that are real (<= S of the launch)
    int done;         // generation finished: every kernel of an iteration returns immediately
    int tokens[kMaxVerify];
};

enum GemvEpi : int {
    EPI_STORE = 0,      // out[tok][row] = y
    EPI_QKV = 1,        // RoPE(q) * 1/sqrt(hd) -> q buffer; RoPE(k), v -> fp16 KV ring
    EPI_SILU_Q8 = 2,    // h = silu(gate) * up, quantised to Q8_0 planes (gate/up row-groups interleaved)
    EPI_BLOCKSUMS = 3,  // raw int32 block dot products of token 0 (parity checks)
};

struct GemvArgs {
    const uint8_t* w;
    int n_rg, nq, K;
    int rg_per_unit, n_units;
    Q8Planes act;
    int S;
    const DevCtrl* ctrl;  // may be null: then all S tokens are valid, pos = 0
    int* err;
    int nstage;           // ring stages (each: chunk tiles of each row-group of a pair)
    int chunk;            // tiles per stage per row-group = consumer warps with tiles: min(16, nq/kparts)
    int kparts;           // K split into kparts slices (EPI_STORE / EPI_BLOCKSUMS only); CTAs
                          // [p*G/kparts, (p+1)*G/kparts) handle slice p and write out + p*part_stride
    size_t part_stride;   // floats between the partial outputs of consecutive K slices
    // EPI_STORE
    float* out;
    int out_ld, out_rows;
    // EPI_QKV
    float* q_out;         // [S][q_rows]
    __half* k_cache;      // layer base: [max_seq][kv_rows]
    __half* v_cache;
    int q_rows, kv_rows, max_seq, head_dim;
    const float* theta_inv;
    float q_scale;
    // EPI_SILU_Q8
    Q8Planes h;
    int hidden;
    // EPI_BLOCKSUMS
    int32_t* isum;        // [rows][K/32]
};

size_t gemv_smem_bytes(int Kp, int S, int chunk, int nstage);
int gemv_pick_stages(int Kp, int S, int chunk, int max_smem);
inline int gemv_chunk(int nq_part) { return nq_part >= kConsumerWarps ? kConsumerWarps : nq_part; }
cudaError_t gemv_init_attrs(int max_smem);
cudaError_t launch_gemv(int epi, const GemvArgs& a, int grid, size_t smem, cudaStream_t st, bool pdl);
cudaError_t launch_sum_parts(const float* parts, float* out, int n, int kparts, size_t stride, cudaStream_t st);

cudaError_t launch_repack(const uint8_t* aos, int rows, int cols, size_t src_row_bytes, RowMap map, uint8_t* dst,
                          cudaStream_t st);
cudaError_t launch_quantize(const float* x, Q8Planes out, int S, int n, cudaStream_t st);
cudaError_t launch_q8_to_blocks(Q8Planes in, void* blocks, int S, int n, cudaStream_t st);
cudaError_t launch_blocks_to_q8(const void* blocks, Q8Planes out, int S, int n, cudaStream_t st);

// Residual add + RMSNorm + Q8_0 quantisation of S tokens (one CTA per token).
//   mode 0: x = embed(tokens) (Q4_0 rows of tok_embd) ; 1: x += y ; 2: x unchanged
// Tensor-parallel exchange over peer memory (CUDA IPC): every rank's o-proj / down-proj partial outputs
// live in its own double-buffered region that the other ranks read over NVLink; flags[src] in each
// rank's region holds the last reduction sequence number rank src has published.
constexpr int kMaxTp = 8;
struct TpXchg {
    int n = 0, rank = 0;                       // n = 0: off
    float* y[kMaxTp] = {};                     // each rank's buffers: [2][buf] floats
    unsigned long long* flags[kMaxTp] = {};    // each rank's flags[kMaxTp]
    const unsigned long long* base = nullptr;  // reductions done before this forward (this rank)
    size_t buf = 0;                            // floats per buffer
    int idx = 0;                               // this reduction's index within the forward
};

struct NormArgs {
    float* x;             // [S][dim] residual stream
    const float* y;       // [S][dim] to add (mode 1)
    const uint8_t* embd;  // embedding rows as in the GGUF (mode 0): Q4_0 (embd_type 2) or Q4_K (12)
    int embd_type;
    const float* w;       // [dim] RMSNorm weight
    Q8Planes out;
    int dim, S;
    float eps;
    const DevCtrl* ctrl;
    const int* tokens;    // host-independent token ids (mode 0); defaults to ctrl->tokens
    float* xn_out;        // optional: normalised fp32 output [S][dim]
    int yparts;           // mode 1: y holds yparts partial slices summed in order (K-split matvec)
    size_t ystride;       // floats between slices
    TpXchg tp;            // mode 1 with tp.n > 1: y of every rank (read over NVLink), summed in rank order
    int* err;             // device error word (a peer wait that runs out)
};
cudaError_t launch_tp_advance(unsigned long long* base, int n, cudaStream_t st);
cudaError_t launch_norm_quant(int mode, const NormArgs& a, cudaStream_t st, bool pdl);

}  // namespace sd
