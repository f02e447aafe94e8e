// gemm_tc.h — tcgen05 (5th-gen tensor core) grouped GEMM for sm_100a.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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
};

bool gemm_supported(int epi);
void gemm(const GemmPlanTC& p, int dtype, cudaStream_t st);

}  // namespace tc
}  // namespace mbr
