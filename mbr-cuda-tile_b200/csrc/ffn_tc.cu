// ffn_tc.cu — fused feed-forward block on tcgen05 (sm_100a); see ffn_tc.h.
//
// One CTA per SM, 320 threads: warp 0 lane 0 issues the TMA loads, warp 1
// lane 0 issues tcgen05.mma (and owns the 512 TMEM columns), warps 2-9 run
// the epilogues.  Per work item (128 rows m0.., hidden chunks [c0, c1)):
//   * X (128 x D, 16-bit) is loaded once as D/64 swizzled 128 x 64 slabs;
//   * chunk c: H_c = X W1[64c..64c+63]^T (M 128, N 64, K D) into TMEM H buffer
//     c % 2 (columns D + 64 (c % 2)); the epilogue warps read it, add b1, apply
//     the reference GELU x Phi(sqrt(2) x) and write P_c (16-bit, 128-byte
//     swizzle, the A-operand layout) into shared-memory P buffer c % 2;
//   * O += P_c W2[:, 64c..64c+63]^T (N = D as N2-wide MMAs) into TMEM columns
//     [0, D), issued one chunk behind H so H_{c+1} overlaps GELU(H_c);
//   * after the item's last chunk the epilogue warps reduce-add O (+ b2 when
//     the item holds chunk 0 of its tile) into the fp32 residual R through
//     32 x 32 TMA boxes staged in the (then idle) P buffers.
// W1 streams through a 6-slab ring of 64 x 64 tiles and W2 through a 2-slab
// ring of N2 x 64 tiles (both L2-resident weights).  Every wait is bounded:
// on timeout the kernel records an error word and unwinds.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "ffn_tc.h"
#include "sm100.cuh"

namespace mbr {
namespace tc {

using namespace sm100;

namespace {

constexpr int FBM = 128;             // rows per tile
constexpr int FHC = 64;              // hidden units per chunk
constexpr int kEpiWarps = 8;         // warps 2-9
constexpr int kFfnThreads = 64 + 32 * kEpiWarps;

template <int D>
struct FfnCfg {
    static constexpr int XS = D / 64;                // X slabs of 128 x 64
    static constexpr int N2 = D == 384 ? 192 : 256;  // output columns per O MMA (N <= 256)
    static constexpr int NS2 = D / N2;               // W2 slabs (O MMAs) per chunk
    static constexpr int NW1 = 6, NW2 = 2;           // ring depths
    static constexpr int X_OFF = 0;
    static constexpr int W1_OFF = XS * 16384;
    static constexpr int W2_OFF = W1_OFF + NW1 * 8192;
    static constexpr int W2_BYTES = N2 * 128;
    static constexpr int P_OFF = W2_OFF + NW2 * W2_BYTES;
    static constexpr int BAR_OFF = P_OFF + 2 * 16384;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;  // + alignment slack
    static constexpr uint32_t TMEM_H = D;              // H buffers at columns D and D + 64
    static_assert(D % 64 == 0 && D % N2 == 0, "D must be a multiple of the slab widths");
    static_assert(D + 2 * FHC <= 512, "TMEM holds O and two hidden chunks");
    static_assert(SMEM <= 232448, "shared memory");
    static_assert(W2_OFF % 1024 == 0 && W2_BYTES % 1024 == 0 && P_OFF % 1024 == 0,
                  "operand tiles 1024-byte aligned for the 128-byte swizzle");
    static_assert(kEpiWarps * 4096 <= 2 * 16384, "O staging fits the P buffers");
};

template <typename T>
struct IsBf16 {
    static constexpr bool value = false;
};
template <>
struct IsBf16<__nv_bfloat16> {
    static constexpr bool value = true;
};

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T, int D>
__global__ void __launch_bounds__(kFfnThreads, 1)
    ffn_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW1,
                  const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmR,
                  const float* __restrict__ b1, const float* __restrict__ b2, const int4* __restrict__ items, int M,
                  int* err) {
    using C = FfnCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bar = (uint64_t*)(smem + C::BAR_OFF);
    uint64_t* x_full = bar;               // X of the item landed
    uint64_t* x_empty = bar + 1;          // the item's last H MMAs completed (X free)
    uint64_t* w1_full = bar + 2;          // [NW1]
    uint64_t* w1_empty = w1_full + C::NW1;
    uint64_t* w2_full = w1_empty + C::NW1;  // [NW2]
    uint64_t* w2_empty = w2_full + C::NW2;
    uint64_t* h_full = w2_empty + C::NW2;   // [2] H chunk computed
    uint64_t* h_free = h_full + 2;          // [2] H chunk read by the 8 epilogue warps
    uint64_t* p_full = h_free + 2;          // [2] P chunk written by the 8 epilogue warps
    uint64_t* p_empty = p_full + 2;         // [2] O MMAs of the P chunk completed
    uint64_t* o_full = p_empty + 2;         // the item's O complete
    uint64_t* o_empty = o_full + 1;         // O read and its staging consumed (8 warps)
    uint32_t* tmem_slot = (uint32_t*)(o_empty + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int4 hdr = items[blockIdx.x];
    const int i0 = hdr.x, nitems = hdr.y - hdr.x;
    if (threadIdx.x == 0) {
        mbar_init(x_full, 1);
        mbar_init(x_empty, 1);
        for (int s = 0; s < C::NW1; ++s) {
            mbar_init(&w1_full[s], 1);
            mbar_init(&w1_empty[s], 1);
        }
        for (int s = 0; s < C::NW2; ++s) {
            mbar_init(&w2_full[s], 1);
            mbar_init(&w2_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&h_full[b], 1);
            mbar_init(&h_free[b], kEpiWarps);
            mbar_init(&p_full[b], kEpiWarps);
            mbar_init(&p_empty[b], 1);
        }
        mbar_init(o_full, 1);
        mbar_init(o_empty, kEpiWarps);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer: loads in the order the MMAs consume them ----
        if (lane == 0) {
            prefetch_tensormap(&tmX);
            prefetch_tensormap(&tmW1);
            prefetch_tensormap(&tmW2);
            uint32_t w1_it = 0, w2_it = 0;
            auto load_w1 = [&](int c) -> bool {  // chunk c: XS slabs of 64 hidden rows x 64 K
                for (int s = 0; s < C::XS; ++s, ++w1_it) {
                    const int slot = w1_it % C::NW1;
                    if (!mbar_wait(&w1_empty[slot], ((w1_it / C::NW1) & 1) ^ 1, err)) return false;
                    mbar_arrive_expect_tx(&w1_full[slot], 8192);
                    tma_load_2d(smem + C::W1_OFF + slot * 8192, &tmW1, 64 * s, FHC * c, &w1_full[slot]);
                }
                return true;
            };
            auto load_w2 = [&](int c) -> bool {  // chunk c: NS2 slabs of N2 output rows x 64 K
                for (int n = 0; n < C::NS2; ++n, ++w2_it) {
                    const int slot = w2_it % C::NW2;
                    if (!mbar_wait(&w2_empty[slot], ((w2_it / C::NW2) & 1) ^ 1, err)) return false;
                    mbar_arrive_expect_tx(&w2_full[slot], C::W2_BYTES);
                    tma_load_2d(smem + C::W2_OFF + slot * C::W2_BYTES, &tmW2, FHC * c, C::N2 * n, &w2_full[slot]);
                }
                return true;
            };
            auto load_x = [&](int k, int m0) -> bool {  // item k's X, once item k-1's H MMAs are done
                if (k > 0 && !mbar_wait(x_empty, (k - 1) & 1, err)) return false;
                mbar_arrive_expect_tx(x_full, C::XS * 16384);
                for (int s = 0; s < C::XS; ++s) tma_load_2d(smem + C::X_OFF + s * 16384, &tmX, 64 * s, m0, x_full);
                return true;
            };
            bool alive = true;
            for (int k = 0; k < nitems && alive; ++k) {
                const int4 it = items[i0 + k];
                if (k == 0) alive = load_x(0, it.x);
                const int n = it.z - it.y;
                for (int j = 0; j < n && alive; ++j) {
                    alive = load_w1(it.y + j);
                    if (alive && j >= 1) alive = load_w2(it.y + j - 1);
                }
                // the next item's X as soon as this item's last H is done, ahead
                // of this item's last W2 chunk
                if (alive && k + 1 < nitems) alive = load_x(k + 1, items[i0 + k + 1].x);
                if (alive) alive = load_w2(it.z - 1);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: H_c, then O += P_{c-1} W2_{c-1}^T ----
        if (lane == 0) {
            constexpr uint32_t idH = idesc_f16(FBM, FHC, IsBf16<T>::value);
            constexpr uint32_t idO = idesc_f16(FBM, C::N2, IsBf16<T>::value);
            // descriptor start addresses advance in 16-byte units: 2 per 16-element K step
            const uint64_t dX = sdesc_sw128(smem_u32(smem + C::X_OFF));
            const uint64_t dW1 = sdesc_sw128(smem_u32(smem + C::W1_OFF));
            const uint64_t dW2 = sdesc_sw128(smem_u32(smem + C::W2_OFF));
            const uint64_t dP = sdesc_sw128(smem_u32(smem + C::P_OFF));
            uint32_t w1_it = 0, w2_it = 0, gc = 0;
            // O (+)= P(g) W2(g)^T; `first`: the item's first chunk (O restarts,
            // after the previous item's O has been read out)
            auto issue_o = [&](int k, uint32_t g, bool first) -> bool {
                const int b = g & 1;
                if (first && k > 0) {
                    if (!mbar_wait(o_empty, (k - 1) & 1, err)) return false;
                    tc_fence_after();
                }
                if (!mbar_wait(&p_full[b], (g >> 1) & 1, err)) return false;
                tc_fence_after();
                for (int n = 0; n < C::NS2; ++n, ++w2_it) {
                    const int slot = w2_it % C::NW2;
                    if (!mbar_wait(&w2_full[slot], (w2_it / C::NW2) & 1, err)) return false;
                    tc_fence_after();
                    const uint64_t a = dP + (uint64_t)(1024 * b);
                    const uint64_t bw = dW2 + (uint64_t)((C::W2_BYTES >> 4) * slot);
#pragma unroll
                    for (int kk = 0; kk < FHC / 16; ++kk)
                        mma_f16(tmem + (uint32_t)(C::N2 * n), a + 2 * kk, bw + 2 * kk, idO, (!first || kk > 0) ? 1u : 0u);
                    mma_commit(&w2_empty[slot]);
                }
                mma_commit(&p_empty[b]);
                return true;
            };
            bool alive = true;
            for (int k = 0; k < nitems && alive; ++k) {
                const int4 it = items[i0 + k];
                if (!(alive = mbar_wait(x_full, k & 1, err))) break;
                tc_fence_after();
                const int n = it.z - it.y;
                for (int j = 0; j < n && alive; ++j, ++gc) {
                    const int b = gc & 1;
                    if (gc >= 2) {  // the epilogue has read H(gc - 2) from this buffer
                        if (!(alive = mbar_wait(&h_free[b], ((gc - 2) >> 1) & 1, err))) break;
                        tc_fence_after();
                    }
                    for (int s = 0; s < C::XS; ++s, ++w1_it) {
                        const int slot = w1_it % C::NW1;
                        if (!(alive = mbar_wait(&w1_full[slot], (w1_it / C::NW1) & 1, err))) break;
                        tc_fence_after();
                        const uint64_t a = dX + (uint64_t)(1024 * s);
                        const uint64_t bw = dW1 + (uint64_t)(512 * slot);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_f16(tmem + C::TMEM_H + 64 * b, a + 2 * kk, bw + 2 * kk, idH, (s | kk) ? 1u : 0u);
                        mma_commit(&w1_empty[slot]);
                    }
                    if (!alive) break;
                    mma_commit(&h_full[b]);
                    if (j == n - 1) mma_commit(x_empty);
                    if (j >= 1) alive = issue_o(k, gc - 1, j == 1);
                }
                if (alive) alive = issue_o(k, gc - 1, n == 1);
                if (alive) mma_commit(o_full);
            }
        }
    } else {
        // ---- epilogue warps: warp (quarter q, column half) ----
        const int q = warp & 3, half = (warp - 2) >> 2;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        const int r = q * 32 + lane;                               // row within the tile
        uint8_t* stg = smem + C::P_OFF + (warp - 2) * 4096;         // O staging (32 rows x 128 B)
        uint32_t gc = 0;
        bool alive = true;
        for (int k = 0; k < nitems && alive; ++k) {
            const int4 it = items[i0 + k];
            const int n = it.z - it.y;
            for (int j = 0; j < n && alive; ++j, ++gc) {
                const int c = it.y + j, b = gc & 1;
                if (!(alive = __all_sync(0xffffffffu, mbar_wait(&h_full[b], (gc >> 1) & 1, err)))) break;
                tc_fence_after();
                uint32_t rr[32];
                tmem_ld32(lane_base + C::TMEM_H + 64 * b + 32 * half, rr);
                tmem_ld_wait(rr);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&h_free[b]);
                float v[32];
                const float4* bb = reinterpret_cast<const float4*>(b1 + FHC * c + 32 * half);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 x = __ldg(bb + i);
                    v[4 * i] = __uint_as_float(rr[4 * i]) + x.x;
                    v[4 * i + 1] = __uint_as_float(rr[4 * i + 1]) + x.y;
                    v[4 * i + 2] = __uint_as_float(rr[4 * i + 2]) + x.z;
                    v[4 * i + 3] = __uint_as_float(rr[4 * i + 3]) + x.w;
                }
                gelu_tail(v);
                // P buffer b is free once the previous item's O staging is
                // consumed (it aliases the P buffers) and O(gc - 2) completed
                if (j == 0 && k > 0 &&
                    !(alive = __all_sync(0xffffffffu, mbar_wait(o_empty, (k - 1) & 1, err))))
                    break;
                if (gc >= 2 &&
                    !(alive = __all_sync(0xffffffffu, mbar_wait(&p_empty[b], ((gc - 2) >> 1) & 1, err))))
                    break;
                uint8_t* prow = smem + C::P_OFF + b * 16384 + r * 128;
#pragma unroll
                for (int u = 0; u < 4; ++u) {  // hidden units 32 half + 8u .. +7: chunk 4 half + u of the row
                    const int chunk = 4 * half + u;
                    *reinterpret_cast<uint4*>(prow + ((chunk ^ (r & 7)) << 4)) =
                        make_uint4(pack2(v[8 * u], v[8 * u + 1], (T*)nullptr),
                                   pack2(v[8 * u + 2], v[8 * u + 3], (T*)nullptr),
                                   pack2(v[8 * u + 4], v[8 * u + 5], (T*)nullptr),
                                   pack2(v[8 * u + 6], v[8 * u + 7], (T*)nullptr));
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[b]);
            }
            if (!alive) break;
            // ---- the item's O: + b2 once per tile, reduce-added into R ----
            if (!(alive = __all_sync(0xffffffffu, mbar_wait(o_full, k & 1, err)))) break;
            tc_fence_after();
            const int yrow = it.x + q * 32;
#pragma unroll 1
            for (int cc = 0; cc < D / 64; ++cc) {
                const int col = half * (D / 2) + 32 * cc;
                uint32_t rr[32];
                tmem_ld32(lane_base + col, rr);
                tmem_ld_wait(rr);
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(rr[i]);
                if (it.w) {
                    const float4* bb = reinterpret_cast<const float4*>(b2 + col);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 x = __ldg(bb + i);
                        v[4 * i] += x.x, v[4 * i + 1] += x.y, v[4 * i + 2] += x.z, v[4 * i + 3] += x.w;
                    }
                }
                if (lane == 0) bulk_wait_read_all();  // the previous box's reduce-add has read the staging
                __syncwarp();
                uint8_t* row = stg + lane * 128;
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8)
                    *reinterpret_cast<float4*>(row + ((c8 ^ (lane & 7)) << 4)) =
                        make_float4(v[4 * c8], v[4 * c8 + 1], v[4 * c8 + 2], v[4 * c8 + 3]);
                fence_async_smem();
                __syncwarp();
                if (lane == 0 && yrow < M) {  // rows past M are clipped by the map; wholly outside boxes skipped
                    tma_reduce_add_3d(&tmR, stg, col, yrow, 0);
                    bulk_commit();
                }
            }
            if (lane == 0) bulk_wait_read_all();
            tc_fence_before();  // O read before the next item's first O MMA
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty);
        }
        if (lane == 0) bulk_wait_all();  // reduce-adds complete before exit
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    if (!fn) throw Error(ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    return fn;
}

// rows x cols row-major operand, box = box_rows x 64 elements, 128-byte swizzle
void map16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows, int dtype) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(m, dtype == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(ERR_CUDA, "ffn: cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

int num_sms() {
    int dev = 0, n = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    return n;
}

template <typename T, int D>
void launch_d(const FfnLaunch& L, int* d_err, cudaStream_t st) {
    using C = FfnCfg<D>;
    auto kern = ffn_tc_kernel<T, D>;
    static bool attr[64] = {};
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < 64, "device index out of range");
    if (!attr[dev]) {
        MBR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr[dev] = true;
    }
    kern<<<L.grid, kFfnThreads, C::SMEM, st>>>(L.tmX, L.tmW1, L.tmW2, L.tmR, L.b1, L.b2, L.items, (int)L.M, d_err);
    MBR_CUDA(cudaGetLastError());
}

}  // namespace

bool ffn_supported(int D, int Hd, int dtype) {
    return (dtype == DT_F16 || dtype == DT_BF16) && (D == 256 || D == 384) && Hd > 0 && Hd % FHC == 0 &&
           Hd <= (1 << 20);
}

void ffn_prepare(const void* x, const void* w1, const float* b1, const void* w2, const float* b2, float* R,
                 int64_t M, int D, int Hd, int dtype, std::vector<int4>& items, FfnLaunch& L, size_t& first) {
    MBR_CHECK(ffn_supported(D, Hd, dtype), "ffn: unsupported shape or dtype");
    MBR_CHECK(M > 0 && M < (1ll << 30), "ffn: row count out of range");
    auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    MBR_CHECK(al16(x) && al16(w1) && al16(w2) && al16(R) && b1 && b2 && al16(b1) && al16(b2),
              "ffn: operands must be 16-byte aligned (biases included)");
    map16(&L.tmX, x, M, D, FBM, dtype);
    map16(&L.tmW1, w1, Hd, D, FHC, dtype);
    map16(&L.tmW2, w2, D, Hd, D == 384 ? 192 : 256, dtype);
    {
        // R [M][D] fp32 as a 3-D map {D, M, 1}: 32 x 32 boxes, 128-byte swizzle
        cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)M, 1};
        cuuint64_t strides[2] = {(cuuint64_t)D * 4, (cuuint64_t)M * D * 4};
        cuuint32_t box[3] = {32, 32, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = encode_fn()(&L.tmR, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, R, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) throw Error(ERR_CUDA, "ffn: cuTensorMapEncodeTiled (R) failed: " + std::to_string((int)r));
    }
    // stream-K work split: the (tile, chunk) units in tile-major order, dealt
    // to the CTAs in equal contiguous shares and cut at tile boundaries
    const int64_t NC = Hd / FHC, ntiles = (M + FBM - 1) / FBM, U = ntiles * NC;
    const int G = (int)std::min<int64_t>(num_sms(), U);
    const int64_t base = U / G, rem = U % G;
    std::vector<int4> body;
    std::vector<int4> hdr((size_t)G);
    for (int k = 0; k < G; ++k) {
        int64_t u = (int64_t)k * base + std::min<int64_t>(k, rem);
        const int64_t u1 = u + base + (k < rem ? 1 : 0);
        hdr[k].x = G + (int)body.size();
        while (u < u1) {
            const int64_t tile = u / NC, c0 = u % NC, c1 = std::min<int64_t>(NC, c0 + (u1 - u));
            body.push_back(make_int4((int)(tile * FBM), (int)c0, (int)c1, c0 == 0 ? 1 : 0));
            u += c1 - c0;
        }
        hdr[k].y = G + (int)body.size();
        hdr[k].z = hdr[k].w = 0;
    }
    first = items.size();
    items.insert(items.end(), hdr.begin(), hdr.end());
    items.insert(items.end(), body.begin(), body.end());
    L.b1 = b1;
    L.b2 = b2;
    L.grid = G;
    L.D = D;
    L.M = M;
    L.ok = true;
}

void ffn_launch(const FfnLaunch& L, int dtype, int* d_err, cudaStream_t st) {
    MBR_CHECK(L.ok && L.items, "ffn launch not prepared");
    if (dtype == DT_BF16) {
        if (L.D == 384) launch_d<__nv_bfloat16, 384>(L, d_err, st);
        else launch_d<__nv_bfloat16, 256>(L, d_err, st);
    } else {
        if (L.D == 384) launch_d<__half, 384>(L, d_err, st);
        else launch_d<__half, 256>(L, d_err, st);
    }
}

}  // namespace tc
}  // namespace mbr
