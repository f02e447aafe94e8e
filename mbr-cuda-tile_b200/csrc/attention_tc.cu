// attention_tc.cu — tcgen05 attention (placeholder until the tensor-core kernel lands).
#include "attention_tc.h"
#include "common.cuh"

namespace mbr {
namespace tc {

bool attention_supported(int) { return false; }
void attention(const void*, const void*, const void*, int64_t, int, int, int, float, const float*, int, int, int,
               void*, int, int*, cudaStream_t) {
    throw Error(ERR_UNSUPPORTED, "tcgen05 attention not built");
}

}  // namespace tc
}  // namespace mbr
