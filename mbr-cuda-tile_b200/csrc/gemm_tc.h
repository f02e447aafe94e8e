// gemm_tc.h — tcgen05 (5th-gen tensor core) grouped GEMM for sm_100a.
//
// C_g = epi(A_g * B_g^T + bias_g) for a list of groups whose A (and B) operands
// are row blocks of one K-major 2-D tensor each.  A persistent kernel walks a
// host-built tile list; TMA streams 128 x 64 A tiles and BN x 64 B tiles
// (128-byte swizzle) through a shared-memory ring, one thread issues
// tcgen05.mma into a double-buffered TMEM accumulator, and eight epilogue warps
// drain TMEM (tcgen05.ld) through the fused epilogue while the next tile's
// MMAs run.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "ops.h"

namespace mbr {
namespace tc {

struct GemmPlanTC {
    const ops::GemmGroup* groups = nullptr;    // device copy of the groups
    const ops::GemmGroup* h_groups = nullptr;  // host copy (same order)
    int ngroups = 0, maxM = 0, maxN = 0, epi = 0;
    // The A and B operands of every group live in one 2-D row-major tensor each
    // (rows x cols elements, K-major); groups address them through
    // a_row0 / b_row0 / k_col0.
    const void* a_base = nullptr;
    int64_t a_rows = 0, a_cols = 0;
    const void* b_base = nullptr;
    int64_t b_rows = 0, b_cols = 0;
    // Optional output view C[group][row][col] = c_base[group*c_group_stride +
    // row*c_row_stride + col] written by TMA stores / reduce-adds from shared
    // memory (rows beyond c_rows and columns beyond c_cols are clipped); group
    // g's block is its c_group.  c_dtype < 0: the epilogue stores from registers.
    const void* c_base = nullptr;
    int64_t c_rows = 0, c_cols = 0, c_groups = 1, c_row_stride = 0, c_group_stride = 0;
    int c_dtype = -1;
};

// Parameters of the fused QKV epilogue (ops::EPI_QKV): RoPE on q/k with the
// position of each token in its sequence, and scatter into [seq][H][L][64].
struct EpiQKV {
    int mode = 0, NB = 0, T = 0, H = 0;
    const float* cos_t = nullptr;  // [L][32]
    const float* sin_t = nullptr;
    void* q = nullptr;
    void* k = nullptr;
    void* v = nullptr;
};

// Prepared launch: tensor maps and the tile list (built once per workspace).
struct GemmLaunch {
    CUtensorMap tmA, tmB, tmC;
    int c_tma = 0;  // epilogue writes C through tmC
    const int4* tiles = nullptr;  // device, two int4 per tile: (group, m0, n0, k-blocks), (A row, B row, K column, last k-steps)
    int ntiles = 0;
    int bn = 128;
    int cg = 1;  // 2: CTA pairs (cluster of two, cta_group::2 MMAs on 256-row tiles)
    int epi = 0;
    const ops::GemmGroup* groups = nullptr;
    EpiQKV qkv;
    bool ok = false;
};

bool gemm_supported(int epi);
// Appends the plan's tiles to `tiles` (host) and fills `L` except L.tiles,
// which the caller points at the uploaded copy (offset `L_first`).
void gemm_prepare(const GemmPlanTC& p, int dtype, std::vector<int4>& tiles, GemmLaunch& L, size_t& L_first);
void gemm_launch(const GemmLaunch& L, int dtype, int* d_err, cudaStream_t st);

}  // namespace tc
}  // namespace mbr
