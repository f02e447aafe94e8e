// gemm_tc.cu — tcgen05 grouped GEMM (placeholder until the tensor-core kernel lands).
#include "common.cuh"
#include "gemm_tc.h"

namespace mbr {
namespace tc {

bool gemm_supported(int) { return false; }
void gemm(const GemmPlanTC&, int, cudaStream_t) { throw Error(ERR_UNSUPPORTED, "tcgen05 GEMM not built"); }

}  // namespace tc
}  // namespace mbr
