// attention_tc.cu — tcgen05 flash attention for the time axis (L = T frames,
// 128-key blocks) and the band axis (L <= 64 bands, two sequences packed per
// 128-row tile with a block-diagonal mask), head dim 64, fp16/bf16.
//
// One CTA (8 warps, two CTAs per SM) = one 128-query tile of one (sequence,
// head) [or two packed band sequences]; warps q and q+4 share query rows
// 32q..32q+31 (TMEM lanes), each taking 64 of the 128 keys of a block and 32
// of the 64 output columns.  Per 128-key block j:
//   S = Q K^T          -> TMEM (128 x 128 fp32)
//   P = exp2(S*c - m)  -> shared memory (16-bit, 128-byte swizzled K-major)
//   O += P V           -> TMEM (128 x 64 fp32)
// Thread 0 issues the TMA loads and, after the CTA barrier that publishes
// P(j), the MMAs P.V(j) and S(j+1); K and V blocks are double buffered.
// V keeps the [seq][H][L][64] layout of q and k: its 128-key tile is the
// MN-major B operand of the P.V product.  The epilogue multiplies by the
// sigmoid gate and writes the merged-head row of each token
// (apply_gates_and_merge_heads).  All waits are bounded (error word instead of
// a hang).
#include <cuda.h>

#include <mutex>

#include "attention_tc.h"
#include "common.cuh"
#include "ops.h"
#include "sm100.cuh"

namespace mbr {
namespace tc {

using namespace sm100;

namespace {

constexpr int DH = 64;
constexpr int QT = 128;  // queries per tile
constexpr int KB = 128;  // keys per block
// O and l are rescaled only when a block's row max (log2 units) exceeds the
// running offset by more than this, bounding the probabilities by 2^8.
constexpr float kRescaleLog2 = 8.0f;

// Two CTAs share an SM, so the layout carries no alignment slack: the kernel
// checks that the dynamic window is 1024-byte aligned instead.
struct AttnSmem {
    static constexpr int Q = 0;
    static constexpr int K0 = 16384;  // K and V blocks are double buffered
    static constexpr int K1 = 32768;
    static constexpr int V0 = 49152;
    static constexpr int V1 = 65536;
    static constexpr int P = 81920;  // two 16 KB K-blocks (keys 0-63, 64-127)
    static constexpr int BAR = 114688;
    static constexpr int TOTAL = BAR + 128;
};

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
struct IsBf16 {
    static constexpr bool value = false;
};
template <>
struct IsBf16<__nv_bfloat16> {
    static constexpr bool value = true;
};

// One lane of the (converged) warp returns true.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.b32 %0, 1, 0, P;\n\t}" : "=r"(pred));
    return pred != 0;
}

// Barrier `id` (1..15) over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2^x with the hardware approximation (relative error ~2^-22; the
// probabilities are rounded to 16 bits right after).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T, bool PACK>
__global__ void __launch_bounds__(256, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, int nsh, int H, int L, float scale_log2,
                   const float* __restrict__ gates, int mode, int NB, int Tn, T* __restrict__ merged, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (!smem_aligned_or_flag(smem_raw, err)) return;  // uniform over the CTA
    uint8_t* sm = smem_raw;
    uint64_t* bar = (uint64_t*)(sm + AttnSmem::BAR);
    uint64_t* bar_q = bar + 0;
    uint64_t* bar_k = bar + 1;  // [2]
    uint64_t* bar_v = bar + 3;  // [2]
    uint64_t* bar_s = bar + 5;
    uint64_t* bar_o = bar + 6;
    uint32_t* tmem_slot = (uint32_t*)(bar + 7);

    const int warp = threadIdx.x >> 5;
    const bool leader = threadIdx.x == 0;
    // tile decode
    int sh0, sh1 = 0, q0 = 0, nkv;
    if (PACK) {
        sh0 = blockIdx.x * 2;
        sh1 = min(sh0 + 1, nsh - 1);
        nkv = 1;
    } else {
        sh0 = blockIdx.y;
        q0 = blockIdx.x * QT;
        nkv = (L + KB - 1) / KB;
    }

    if (leader) {
        mbar_init(bar_q, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar_k[i], 1);
            mbar_init(&bar_v[i], 1);
        }
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tO = tmem + 128;

    // ---- leader-thread producer / MMA helpers ----
    auto load_k = [&](int j) {
        uint8_t* dst = sm + ((j & 1) ? AttnSmem::K1 : AttnSmem::K0);
        mbar_arrive_expect_tx(&bar_k[j & 1], 16384);
        if (PACK) {
            tma_load_2d(dst, &tmK, 0, sh0 * L, &bar_k[j & 1]);
            tma_load_2d(dst + 8192, &tmK, 0, sh1 * L, &bar_k[j & 1]);
        } else {
            tma_load_2d(dst, &tmK, 0, sh0 * L + j * KB, &bar_k[j & 1]);
        }
    };
    auto load_v = [&](int j) {
        uint8_t* dst = sm + ((j & 1) ? AttnSmem::V1 : AttnSmem::V0);
        mbar_arrive_expect_tx(&bar_v[j & 1], 16384);
        if (PACK) {
            tma_load_2d(dst, &tmV, 0, sh0 * L, &bar_v[j & 1]);
            tma_load_2d(dst + 8192, &tmV, 0, sh1 * L, &bar_v[j & 1]);
        } else {
            tma_load_2d(dst, &tmV, 0, sh0 * L + j * KB, &bar_v[j & 1]);
        }
    };
    constexpr uint32_t idS = idesc_f16(QT, KB, IsBf16<T>::value);
    constexpr uint32_t idO = idesc_f16(QT, DH, IsBf16<T>::value, /*b_mn_major=*/true);
    const uint32_t sQ = smem_u32(sm + AttnSmem::Q), sPa = smem_u32(sm + AttnSmem::P);
    // descriptor bases; the start-address field (16-byte units) advances by 2
    // per 32 bytes along K and by 1024 per 16 KB P block
    const uint64_t dQ = sdesc_sw128(sQ);
    const uint64_t dK0 = sdesc_sw128(smem_u32(sm + AttnSmem::K0)), dK1 = sdesc_sw128(smem_u32(sm + AttnSmem::K1));
    const uint64_t dV0 = sdesc_sw128_mn(smem_u32(sm + AttnSmem::V0)),
                   dV1 = sdesc_sw128_mn(smem_u32(sm + AttnSmem::V1));
    const uint64_t dP = sdesc_sw128(sPa);
    auto issue_s = [&](int j) {  // S = Q K(j)^T -> tS
        const uint64_t dK = (j & 1) ? dK1 : dK0;
#pragma unroll
        for (int k = 0; k < DH / 16; ++k) mma_f16(tS, dQ + 2 * k, dK + 2 * k, idS, k > 0);
        mma_commit(bar_s);
    };
    auto issue_pv = [&](int j) {  // O (+)= P V(j) -> tO
        const uint64_t dV = (j & 1) ? dV1 : dV0;
#pragma unroll
        for (int k = 0; k < KB / 16; ++k) {
            const uint32_t blk = k >> 2, kk = k & 3;
            // A: P rows (K-major, 64 keys per 16 KB block); B: V keys 16k..16k+15 (MN-major)
            mma_f16(tO, dP + blk * 1024 + 2 * kk, dV + 128 * k, idO, (j | k) != 0);
        }
        mma_commit(bar_o);
    };

    bool ok = true;  // warp-uniform: TMEM loads and stores are warp-collective
    if (leader) {
        prefetch_tensormap(&tmQ);
        prefetch_tensormap(&tmK);
        prefetch_tensormap(&tmV);
        mbar_arrive_expect_tx(bar_q, 16384);
        if (PACK) {
            tma_load_2d(sm + AttnSmem::Q, &tmQ, 0, sh0 * L, bar_q);
            tma_load_2d(sm + AttnSmem::Q + 8192, &tmQ, 0, sh1 * L, bar_q);
        } else {
            tma_load_2d(sm + AttnSmem::Q, &tmQ, 0, sh0 * L + q0, bar_q);
        }
        load_k(0);
        load_v(0);
        if (nkv > 1) {
            load_k(1);
            load_v(1);
        }
        ok = mbar_wait(bar_q, 0, err) && mbar_wait(&bar_k[0], 0, err);
        if (ok) issue_s(0);
    }

    // ---- softmax: warps q and q + 4 share query rows 32q..32q+31 (TMEM lane
    // r = row r); warp half hf = warp / 4 owns key columns [64 hf, 64 hf + 64)
    // of S (= P block hf) and O columns [32 hf, 32 hf + 32).
    // O accumulates in TMEM over the key blocks.  The exponent offset m is the
    // first block's row max and is raised (O and l rescaled in place) only
    // when a later block's max exceeds it by more than kRescaleLog2, so
    // P <= 2^kRescaleLog2 and O / l is the same softmax.
    const int q4 = warp & 3, hf = warp >> 2;
    const int r = q4 * 32 + (threadIdx.x & 31);
    int seg = 0, pos, sh = sh0;
    bool valid;
    if (PACK) {
        seg = r >> 6;
        pos = r & 63;
        sh = seg ? sh1 : sh0;
        valid = pos < L && (seg == 0 || sh0 + 1 < nsh);
    } else {
        pos = q0 + r;
        valid = pos < L;
    }
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    uint8_t* sP = sm + AttnSmem::P;
    // Row-r exchange slots between the two halves: each half writes into the
    // other half's P row r, which that half overwrites only after reading it.
    volatile float* x_mine = (volatile float*)(sP + (hf ^ 1) * 16384 + r * 128);
    volatile float* x_part = (volatile float*)(sP + hf * 16384 + r * 128);
    float m = 0.f, lh = 0.f;  // lh: this half's share of the row sum
    for (int j = 0; j < nkv; ++j) {
        // every thread reaches every barrier below, also after a timeout
        ok = __all_sync(0xffffffffu, ok && mbar_wait(bar_s, j & 1, err));
        tc_fence_after();
        // valid key columns of this row in block j: [kbeg, kend) (warp-uniform)
        int kbeg, kend;
        if (PACK) {
            kbeg = seg * 64;
            kend = kbeg + min(L, 64);
        } else {
            kbeg = 0;
            kend = min(KB, L - j * KB);
        }
        uint32_t sv[2][32];
        float mx = -INFINITY;
        if (ok) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int c0 = hf * 64 + c * 32;
                if (c0 + 32 > kbeg && c0 < kend) tmem_ld32(tS + lane_off + c0, sv[c]);
            }
            tmem_ld_wait();
            float mxp[8];  // 8 independent partial maxima
#pragma unroll
            for (int u = 0; u < 8; ++u) mxp[u] = -INFINITY;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int c0 = hf * 64 + c * 32;
                if (c0 + 32 <= kbeg || c0 >= kend) continue;
                if (c0 >= kbeg && c0 + 32 <= kend) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) mxp[i & 7] = fmaxf(mxp[i & 7], __uint_as_float(sv[c][i]));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c0 + i >= kbeg && c0 + i < kend) mxp[i & 7] = fmaxf(mxp[i & 7], __uint_as_float(sv[c][i]));
                }
            }
            mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                       fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
        }
        // P.V(j-1) finished before S(j) did, so the P rows are free for the exchange
        *x_mine = mx;
        named_barrier_sync(1 + q4, 64);
        const float mx_row = fmaxf(mx, *x_part);  // same value in both halves
        if (ok) {
            const float m_blk = mx_row * scale_log2;  // the scale is positive
            if (j == 0) {
                m = m_blk == -INFINITY ? 0.f : m_blk;
            } else {
                // O holds P.V of blocks < j
                const bool need = m_blk > m + kRescaleLog2;
                if (__any_sync(0xffffffffu, need)) {  // TMEM access is warp-collective
                    const float alpha = need ? fast_exp2(m - m_blk) : 1.0f;
                    if (need) {
                        m = m_blk;
                        lh *= alpha;
                    }
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {  // this half's 32 O columns, 16 at a time
                        uint32_t ov[16];
                        const uint32_t ta = tO + lane_off + hf * 32 + c * 16;
                        tmem_ld16(ta, ov);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                        tmem_st16(ta, ov);
                    }
                    tmem_st_wait();
                }
            }
            // probabilities -> P block hf row r (swizzled K-major); chunks
            // outside the valid range get zeros
            float rsp[8];  // 8 independent partial sums
#pragma unroll
            for (int u = 0; u < 8; ++u) rsp[u] = 0.f;
            uint8_t* prow = sP + hf * 16384 + r * 128;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int c0 = hf * 64 + c * 32;
                if (c0 + 32 <= kbeg || c0 >= kend) {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        *reinterpret_cast<uint4*>(prow + (((4 * c + q) ^ (r & 7)) << 4)) = make_uint4(0, 0, 0, 0);
                    continue;
                }
                float p[32];
                if (c0 >= kbeg && c0 + 32 <= kend) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) p[i] = fast_exp2(fmaf(__uint_as_float(sv[c][i]), scale_log2, -m));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        p[i] = (c0 + i >= kbeg && c0 + i < kend)
                                   ? fast_exp2(fmaf(__uint_as_float(sv[c][i]), scale_log2, -m))
                                   : 0.f;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) rsp[i & 7] += p[i];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint4 u = make_uint4(pack2(p[8 * q], p[8 * q + 1], (T*)nullptr),
                                         pack2(p[8 * q + 2], p[8 * q + 3], (T*)nullptr),
                                         pack2(p[8 * q + 4], p[8 * q + 5], (T*)nullptr),
                                         pack2(p[8 * q + 6], p[8 * q + 7], (T*)nullptr));
                    *reinterpret_cast<uint4*>(prow + (((4 * c + q) ^ (r & 7)) << 4)) = u;
                }
            }
            lh += ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
        }
        fence_proxy_async_smem();  // P visible to the tensor cores
        tc_fence_before();         // S reads / O stores ordered before the next MMAs
        __syncthreads();
        if (warp == 0 && ok) {
            // P.V(j), then S(j+1) behind it, issued by one elected lane of
            // warp 0 (warp-uniform operands).  Buffer reuse: V((j+1)&1) held
            // V(j-1), whose P.V finished before S(j) did; K(j&1) held K(j),
            // consumed by S(j).
            tc_fence_after();
            if (leader && j >= 1 && j + 1 < nkv) load_v(j + 1);
            bool okw = __all_sync(0xffffffffu, mbar_wait(&bar_v[j & 1], (j >> 1) & 1, err));
            if (okw && elect_one()) issue_pv(j);
            __syncwarp();
            if (okw && j + 1 < nkv) {
                okw = __all_sync(0xffffffffu, mbar_wait(&bar_k[(j + 1) & 1], ((j + 1) >> 1) & 1, err));
                if (okw && elect_one()) {
                    issue_s(j + 1);
                    if (j + 2 < nkv) load_k(j + 2);
                }
                __syncwarp();
            }
            ok = okw;
        }
    }
    // S(j+1) is issued after P(j).V(j), so only the last P.V is waited for
    // here (its phase is the only one that can still be open); after it the
    // P rows are free again for the row-sum exchange.
    ok = __all_sync(0xffffffffu, ok && mbar_wait(bar_o, (nkv - 1) & 1, err));
    *x_mine = lh;
    named_barrier_sync(1 + q4, 64);
    const float lo = *x_part;
    const float l = hf == 0 ? lh + lo : lo + lh;
    if (ok) {
        tc_fence_after();
        uint32_t ov[32];
        tmem_ld32(tO + lane_off + hf * 32, ov);
        tmem_ld_wait();
        if (valid) {
            const int hd = sh % H;
            const int64_t s = sh / H;
            int64_t tok;
            if (mode == ops::SEQ_TIME) tok = ((s / NB) * Tn + pos) * NB + (s % NB);
            else tok = s * NB + pos;
            const float g = (gates ? gates[tok * H + hd] : 1.0f) / l;
            uint4* dst = reinterpret_cast<uint4*>(merged + tok * (int64_t)H * DH + hd * DH + hf * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t* o = &ov[q * 8];
                dst[q] = make_uint4(pack2(__uint_as_float(o[0]) * g, __uint_as_float(o[1]) * g, (T*)nullptr),
                                    pack2(__uint_as_float(o[2]) * g, __uint_as_float(o[3]) * g, (T*)nullptr),
                                    pack2(__uint_as_float(o[4]) * g, __uint_as_float(o[5]) * g, (T*)nullptr),
                                    pack2(__uint_as_float(o[6]) * g, __uint_as_float(o[7]) * g, (T*)nullptr));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 256);
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

void make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_cols, int box_rows, int dtype) {
    MBR_CHECK(((uintptr_t)base & 15) == 0 && (cols * 2) % 16 == 0, "attention TMA operand misaligned");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(m, dtype == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

template <typename T, bool PACK>
void launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, int nsh, int H, int L,
            float scale_log2, const float* gates, int mode, int NB, int Tn, void* merged, int* err, cudaStream_t st) {
    auto kern = attn_tc_kernel<T, PACK>;
    static bool attr[64] = {};
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < 64, "device index out of range");
    if (!attr[dev]) {
        MBR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmem::TOTAL));
        attr[dev] = true;
    }
    dim3 grid = PACK ? dim3((unsigned)((nsh + 1) / 2)) : dim3((unsigned)((L + QT - 1) / QT), (unsigned)nsh);
    kern<<<grid, 256, AttnSmem::TOTAL, st>>>(mq, mk, mv, nsh, H, L, scale_log2, gates, mode, NB, Tn, (T*)merged,
                                              err);
    MBR_CUDA(cudaGetLastError());
}

}  // namespace

bool attention_supported(int dim_head) { return dim_head == DH; }

void attention(const void* q, const void* k, const void* v, int64_t nseq, int H, int L, int dh, float scale,
               const float* gates, int mode, int NB, int T, void* merged, int dtype, int* d_err, cudaStream_t st) {
    MBR_CHECK(dh == DH, "tc attention: dim_head must be 64");
    MBR_CHECK(dtype == DT_F16 || dtype == DT_BF16, "tc attention: fp16 or bf16 only");
    const int64_t nsh = nseq * H;
    MBR_CHECK(nsh < (1 << 30) && nsh * L < (1ll << 31), "tc attention: problem too large for 32-bit coordinates");
    const bool pack = L <= 64;
    CUtensorMap mq, mk, mv;
    const int qrows = pack ? 64 : QT;
    make_map(&mq, q, nsh * L, DH, DH, qrows, dtype);
    make_map(&mk, k, nsh * L, DH, DH, pack ? 64 : KB, dtype);
    make_map(&mv, v, nsh * L, DH, DH, pack ? 64 : KB, dtype);
    const float scale_log2 = scale * 1.4426950408889634f;
    if (dtype == DT_BF16) {
        if (pack) launch<__nv_bfloat16, true>(mq, mk, mv, (int)nsh, H, L, scale_log2, gates, mode, NB, T, merged, d_err, st);
        else launch<__nv_bfloat16, false>(mq, mk, mv, (int)nsh, H, L, scale_log2, gates, mode, NB, T, merged, d_err, st);
    } else {
        if (pack) launch<__half, true>(mq, mk, mv, (int)nsh, H, L, scale_log2, gates, mode, NB, T, merged, d_err, st);
        else launch<__half, false>(mq, mk, mv, (int)nsh, H, L, scale_log2, gates, mode, NB, T, merged, d_err, st);
    }
}

}  // namespace tc
}  // namespace mbr
