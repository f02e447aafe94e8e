// common.h — host-side error handling and dtype codes shared by every source file.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace mbr {

// Error raised by host code; converted to a status code at the C-ABI.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

enum Status { OK = 0, ERR_INVALID = 1, ERR_CUDA = 2, ERR_IO = 3, ERR_UNSUPPORTED = 4, ERR_OOM = 5, ERR_TIMEOUT = 6 };

#define MBR_CUDA(call)                                                                                   \
    do {                                                                                                 \
        cudaError_t e_ = (call);                                                                         \
        if (e_ != cudaSuccess)                                                                           \
            throw ::mbr::Error(e_ == cudaErrorMemoryAllocation ? ::mbr::ERR_OOM : ::mbr::ERR_CUDA,       \
                               std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " + __FILE__ + \
                                   ":" + std::to_string(__LINE__));                                      \
    } while (0)

#define MBR_CHECK(cond, msg)                                               \
    do {                                                                   \
        if (!(cond)) throw ::mbr::Error(::mbr::ERR_INVALID, std::string(msg)); \
    } while (0)

// Compute dtype codes (match the .csm dtype codes of the reference:
// 0 f32, 1 f16, 3 bf16).
enum DType { DT_F32 = 0, DT_F16 = 1, DT_I64 = 2, DT_BF16 = 3 };

inline size_t dtype_bytes(int dt) { return dt == DT_F32 ? 4 : dt == DT_I64 ? 8 : 2; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

}  // namespace mbr
