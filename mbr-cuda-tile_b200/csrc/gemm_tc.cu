// gemm_tc.cu — persistent, warp-specialised tcgen05 grouped GEMM (sm_100a).
//
// Warp roles (320 threads): warp 0 lane 0 issues the TMA loads, warp 1 lane 0
// issues tcgen05.mma (and owns the TMEM allocation), warps 2-9 run the
// epilogue.  Operand tiles are 128 x 64 (A) and BN x 64 (B) 16-bit elements
// with the 128-byte swizzle, so every MMA descriptor addresses a canonical
// K-major layout.  The accumulator is double buffered in TMEM so the epilogue
// of tile i overlaps the MMAs of tile i+1.  Plans with an output view stage
// each warp's 32 x 128-byte slab in shared memory and write it with one TMA
// store (or TMA reduce-add into the fp32 residual stream).  Every wait is
// bounded: on timeout the kernel records an error word and unwinds instead of
// hanging.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "gemm_tc.h"
#include "sm100.cuh"

namespace mbr {
namespace tc {

using namespace sm100;

namespace {

constexpr int BM = 128, BK = 64;

// Epilogue warps: warps 2 .. 2 + EW - 1; warp w drains TMEM lane quarter
// (w % 4), and (w - 2) / 4 numbers it among the EW / 4 warps of its quarter.
// The GELU epilogue, whose math costs more than the tile's MMAs, gets 12
// warps (three per quarter); the others 8.
constexpr int kStageRowBytes = 128;                    // one swizzled 128-byte row per lane
constexpr int kStagingPerWarp = 32 * kStageRowBytes;   // 32 rows x 128 B
__host__ __device__ constexpr int epi_warps(int epi) { return epi == ops::EPI_GELU_T ? 12 : 8; }
__host__ __device__ constexpr int gemm_threads(int epi) { return 64 + 32 * epi_warps(epi); }

// CG = 1: one CTA computes a 128 x BN tile.  CG = 2: a CTA pair (cluster of
// two) computes 256 x BN with cta_group::2 MMAs; each CTA holds its 128 A rows
// and half of the B rows, so a stage is 16 KB + BN*64 bytes per CTA.
// Each epilogue warp owns NSTG staging tiles, so a TMA store can still be
// reading one while the warp fills the other; the operand ring gets what is
// left of the 227 KB (at most 8 stages).  The 128 x 256 single-CTA tile keeps
// one staging tile to keep 4 operand stages, and so do the residual GEMMs
// (long K, a light reduce-add epilogue): their operand ring is the deeper one.
// The GELU epilogue's 12 warps each stage one 32 x 32 box (2 KB) at a time.
template <int BN, int CG, int EPI>
struct TileCfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = (BN / CG) * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EW = epi_warps(EPI);
    static constexpr int NSTG = ((CG == 1 && BN == 256) || EPI == ops::EPI_ADD_F32) ? 1 : 2;
    static constexpr int STG_WARP = EPI == ops::EPI_GELU_T ? kStagingPerWarp / 2 : NSTG * kStagingPerWarp;
    static constexpr int kSmemMax = 232448 - 256 - 1024;  // opt-in maximum less barriers and alignment slack
    static constexpr int STAGES_FIT = (kSmemMax - EW * STG_WARP) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT < 8 ? STAGES_FIT : 8;
    static_assert(STAGES >= 3, "operand ring too shallow");
    static constexpr int STAGING_OFF = STAGES * STAGE_BYTES;  // 1024-aligned
    static constexpr int BAR_OFF = STAGING_OFF + EW * STG_WARP;
    static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;
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

// Applies the epilogue to 32 accumulator columns [n0, n0+32) of one row.
template <typename T, int EPI>
__device__ __forceinline__ void epilogue_chunk(const ops::GemmGroup& g, int row, int n0, const uint32_t (&r)[32]) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    const int nvalid = min(32, g.N - n0);
    if (g.bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < nvalid) v[j] += __ldg(g.bias + n0 + j);
    }
    if constexpr (EPI == ops::EPI_F32 || EPI == ops::EPI_ADD_F32) {
        float* c = (float*)g.C + (int64_t)row * g.ldc + n0;
        if (nvalid == 32 && ((uintptr_t)c & 15) == 0) {
            float4* c4 = reinterpret_cast<float4*>(c);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                if constexpr (EPI == ops::EPI_ADD_F32) {
                    float4 p = c4[j];
                    o.x += p.x, o.y += p.y, o.z += p.z, o.w += p.w;
                }
                c4[j] = o;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nvalid) c[j] = EPI == ops::EPI_ADD_F32 ? c[j] + v[j] : v[j];
        }
    } else if constexpr (EPI == ops::EPI_GLU_F32) {
        float o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = v[2 * i] / (1.0f + __expf(-v[2 * i + 1]));
        float* c = (float*)g.C + (int64_t)row * g.ldc + n0 / 2;
        const int ovalid = nvalid / 2;
        if (ovalid == 16 && ((uintptr_t)c & 15) == 0) {
            float4* c4 = reinterpret_cast<float4*>(c);
#pragma unroll
            for (int j = 0; j < 4; ++j) c4[j] = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < ovalid) c[i] = o[i];
        }
    } else {
        if constexpr (EPI == ops::EPI_GELU_T) {
            gelu_tail(v);
        } else if constexpr (EPI == ops::EPI_TANH_T) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = tanh_fast(v[j]);
        }
        T* c = (T*)g.C + (int64_t)row * g.ldc + n0;
        if (nvalid == 32 && ((uintptr_t)c & 15) == 0) {
            uint4* c4 = reinterpret_cast<uint4*>(c);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                c4[j] = make_uint4(pack2(v[8 * j], v[8 * j + 1], (T*)nullptr), pack2(v[8 * j + 2], v[8 * j + 3], (T*)nullptr),
                                   pack2(v[8 * j + 4], v[8 * j + 5], (T*)nullptr),
                                   pack2(v[8 * j + 6], v[8 * j + 7], (T*)nullptr));
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nvalid) c[j] = from_f32<T>(v[j]);
        }
    }
}

// RoPE (interleaved pairs, src/mbr_cuda_tile.cu:3928-3943) of the 32 columns
// [n0, n0+32) of token `row` of a fused q|k|v projection, in place; v columns
// (section 2) are left alone.  The position is the token's index in its
// sequence: the frame along the time axis, the band along the band axis.
__device__ __forceinline__ void rope_rotate(const EpiQKV& e, int row, int n0, float (&v)[32]) {
    const int DI = e.H * 64;
    const int sec = n0 / DI;
    const int d0 = (n0 - sec * DI) & 63;
    const int pos = e.mode == ops::SEQ_TIME ? (row / e.NB) % e.T : row % e.NB;
    if (sec < 2) {
        // 16 consecutive table entries (64 bytes, 64-byte aligned) per lane as
        // four 16-byte loads: along the band axis every lane has its own
        // position, so scalar loads would cost one L1 wavefront per lane each
        const float4* cs = reinterpret_cast<const float4*>(e.cos_t + pos * 32 + (d0 >> 1));
        const float4* sn = reinterpret_cast<const float4*>(e.sin_t + pos * 32 + (d0 >> 1));
#pragma unroll
        for (int i4 = 0; i4 < 4; ++i4) {
            const float4 c4 = __ldg(cs + i4), s4 = __ldg(sn + i4);
            const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = 4 * i4 + u;
                const float x0 = v[2 * i], x1 = v[2 * i + 1];
                v[2 * i] = x0 * cc[u] - x1 * ss[u];
                v[2 * i + 1] = x0 * ss[u] + x1 * cc[u];
            }
        }
    }
}

// The 16 (cos, sin) pairs [p0, p0 + 16) of one table row (64-byte aligned).
__device__ __forceinline__ void load_rope16(const float* cs, const float* sn, int p0, float4 (&c)[4],
                                            float4 (&s)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        c[i] = __ldg(reinterpret_cast<const float4*>(cs + p0) + i);
        s[i] = __ldg(reinterpret_cast<const float4*>(sn + p0) + i);
    }
}
// Rotates the 16 pairs (v[2i], v[2i+1]) by the angles whose cos / sin are given.
__device__ __forceinline__ void rope_apply16(const float4 (&c)[4], const float4 (&s)[4], float (&v)[32]) {
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
        const float cc[4] = {c[i4].x, c[i4].y, c[i4].z, c[i4].w}, ss[4] = {s[i4].x, s[i4].y, s[i4].z, s[i4].w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = 4 * i4 + u;
            const float x0 = v[2 * i], x1 = v[2 * i + 1];
            v[2 * i] = x0 * cc[u] - x1 * ss[u];
            v[2 * i + 1] = x0 * ss[u] + x1 * cc[u];
        }
    }
}

// QKV epilogue: RoPE, then scatter of the 32 columns [n0, n0+32) of token
// `row` into the per-sequence head-major q / k / v tensors [seq][H][L][64].
template <typename T>
__device__ __forceinline__ void epilogue_qkv(const EpiQKV& e, int row, int n0, const uint32_t (&r)[32]) {
    const int DI = e.H * 64;
    const int sec = n0 / DI, rem = n0 - sec * DI;
    const int h = rem >> 6, d0 = rem & 63;
    int64_t s;
    int pos, L;
    if (e.mode == ops::SEQ_TIME) {
        const int k = row % e.NB;
        const int64_t bt = row / e.NB;
        pos = (int)(bt % e.T);
        s = (bt / e.T) * e.NB + k;
        L = e.T;
    } else {
        s = row / e.NB;
        pos = row % e.NB;
        L = e.NB;
    }
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    rope_rotate(e, row, n0, v);
    T* base = (T*)(sec == 0 ? e.q : sec == 1 ? e.k : e.v);
    uint4* dst = reinterpret_cast<uint4*>(base + ((s * e.H + h) * L + pos) * 64 + d0);
#pragma unroll
    for (int j = 0; j < 4; ++j)
        dst[j] = make_uint4(pack2(v[8 * j], v[8 * j + 1], (T*)nullptr), pack2(v[8 * j + 2], v[8 * j + 3], (T*)nullptr),
                            pack2(v[8 * j + 4], v[8 * j + 5], (T*)nullptr),
                            pack2(v[8 * j + 6], v[8 * j + 7], (T*)nullptr));
}

// Stages 32 accumulator columns of this lane's row through the warp's
// shared-memory tile (128-byte swizzled rows): fp32 outputs fill a whole row,
// 16-bit outputs fill half of it (the other half comes from the next chunk).
template <typename T, int EPI>
__device__ __forceinline__ void stage_chunk(uint8_t* stg, int lane, int half16, const float (&v)[32]) {
    uint8_t* row = stg + lane * kStageRowBytes;
    if constexpr (EPI == ops::EPI_F32 || EPI == ops::EPI_ADD_F32) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
            *reinterpret_cast<float4*>(row + ((c ^ (lane & 7)) << 4)) =
                make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int ch = half16 * 4 + c;
            *reinterpret_cast<uint4*>(row + ((ch ^ (lane & 7)) << 4)) =
                make_uint4(pack2(v[8 * c], v[8 * c + 1], (T*)nullptr), pack2(v[8 * c + 2], v[8 * c + 3], (T*)nullptr),
                           pack2(v[8 * c + 4], v[8 * c + 5], (T*)nullptr),
                           pack2(v[8 * c + 6], v[8 * c + 7], (T*)nullptr));
        }
    }
}

// Stages 32 accumulator columns of this lane's row as one 64-byte row of a
// 32 x 32 box (16-bit outputs, 64-byte swizzle: 16-byte unit u of row r sits at
// unit u ^ ((r >> 1) & 3)).
template <typename T>
__device__ __forceinline__ void stage_chunk64(uint8_t* stg, int lane, const float (&v)[32]) {
    uint8_t* row = stg + lane * 64;
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(row + ((c ^ ((lane >> 1) & 3)) << 4)) =
            make_uint4(pack2(v[8 * c], v[8 * c + 1], (T*)nullptr), pack2(v[8 * c + 2], v[8 * c + 3], (T*)nullptr),
                       pack2(v[8 * c + 4], v[8 * c + 5], (T*)nullptr), pack2(v[8 * c + 6], v[8 * c + 7], (T*)nullptr));
}

// acc + bias and the activation of the epilogue, in place.
template <int EPI>
__device__ __forceinline__ void apply_epi(const ops::GemmGroup& g, int n0, float (&v)[32]) {
    const int nvalid = min(32, g.N - n0);
    if (g.bias) {
        const float* b = g.bias + n0;
        if (nvalid == 32 && ((uintptr_t)b & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 b4 = __ldg(reinterpret_cast<const float4*>(b) + j);
                const float2 s0 = __fadd2_rn(make_float2(v[4 * j], v[4 * j + 1]), make_float2(b4.x, b4.y));
                const float2 s1 = __fadd2_rn(make_float2(v[4 * j + 2], v[4 * j + 3]), make_float2(b4.z, b4.w));
                v[4 * j] = s0.x, v[4 * j + 1] = s0.y, v[4 * j + 2] = s1.x, v[4 * j + 3] = s1.y;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nvalid) v[j] += __ldg(b + j);
        }
    }
    if constexpr (EPI == ops::EPI_GELU_T) {
        gelu_tail(v);
    } else if constexpr (EPI == ops::EPI_TANH_T) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = tanh_fast(v[j]);
    }
}

template <typename T, int BN, int EPI, int CG>
__global__ void __launch_bounds__(gemm_threads(EPI), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, int c_tma, const ops::GemmGroup* __restrict__ groups,
                   const int4* __restrict__ tiles, int ntiles, int* err, const EpiQKV qkv) {
    using Cfg = TileCfg<BN, CG, EPI>;
    // CTA pair: rank 0 issues the MMAs, counts both CTAs' TMA bytes on its full
    // barriers and collects both CTAs' epilogue arrivals on its acc_empty
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0;
    const bool leader = rank == 0;
    const int cta_tile0 = (int)blockIdx.x / CG, cta_tile_step = (int)gridDim.x / CG;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + Cfg::STAGES * Cfg::A_BYTES;
    uint64_t* full = (uint64_t*)(smem + Cfg::BAR_OFF);
    uint64_t* empty = full + Cfg::STAGES;
    uint64_t* acc_full = empty + Cfg::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], Cfg::EW * CG);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        if constexpr (CG == 2) {
            tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if constexpr (CG == 2) cluster_sync();  // the peer's barriers exist before any remote arrive / TMA count
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tensormap(&tmA);
            prefetch_tensormap(&tmB);
            uint32_t it = 0;
            bool alive = true;
            int4 tl = make_int4(0, 0, 0, 0), ta = tl;
            if (cta_tile0 < ntiles) tl = tiles[2 * cta_tile0], ta = tiles[2 * cta_tile0 + 1];
            for (int t = cta_tile0; t < ntiles && alive; t += cta_tile_step) {
                // the next tile's descriptor is in flight while this tile's loads are issued
                int4 tl_n = make_int4(0, 0, 0, 0), ta_n = tl_n;
                if (t + cta_tile_step < ntiles)
                    tl_n = tiles[2 * (t + cta_tile_step)], ta_n = tiles[2 * (t + cta_tile_step) + 1];
                for (int kb = 0; kb < tl.w; ++kb, ++it) {
                    const int s = it % Cfg::STAGES;
                    const uint32_t r = it / Cfg::STAGES;
                    if (!mbar_wait(&empty[s], (r & 1) ^ 1, err)) {
                        alive = false;
                        break;
                    }
                    const int kx = ta.z + kb * BK;
                    if constexpr (CG == 2) {
                        // both CTAs' bytes complete on the leader's full barrier
                        const uint32_t fb = map_to_cta(smem_u32(&full[s]), 0);
                        if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
                        tma_load_2d_pair(sA + s * Cfg::A_BYTES, &tmA, kx, ta.x + (int)rank * BM, fb);
                        tma_load_2d_pair(sB + s * Cfg::B_BYTES, &tmB, kx, ta.y + (int)rank * (BN / 2), fb);
                    } else {
                        mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                        tma_load_2d(sA + s * Cfg::A_BYTES, &tmA, kx, ta.x, &full[s]);
                        tma_load_2d(sB + s * Cfg::B_BYTES, &tmB, kx, ta.y, &full[s]);
                    }
                }
                tl = tl_n;
                ta = ta_n;
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_f16(BM * CG, BN, IsBf16<T>::value);
            uint32_t it = 0;
            int tcount = 0;
            bool alive = true;
            int nkb = 0, klast = 0;  // k-blocks of the tile, k-steps of its last k-block
            if (cta_tile0 < ntiles) nkb = tiles[2 * cta_tile0].w, klast = tiles[2 * cta_tile0 + 1].w;
            for (int t = cta_tile0; t < ntiles && alive; t += cta_tile_step, ++tcount) {
                int nkb_n = 0, klast_n = 0;  // the next tile's, in flight during this one
                if (t + cta_tile_step < ntiles)
                    nkb_n = tiles[2 * (t + cta_tile_step)].w, klast_n = tiles[2 * (t + cta_tile_step) + 1].w;
                const int buf = tcount & 1;
                const uint32_t use = tcount >> 1;
                if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, err)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * BN;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % Cfg::STAGES;
                    const uint32_t r = it / Cfg::STAGES;
                    if (!mbar_wait(&full[s], r & 1, err)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + s * Cfg::B_BYTES);
                    const int ksteps = kb + 1 == nkb ? klast : BK / 16;
                    if constexpr (CG == 2) {
                        for (int k = 0; k < ksteps; ++k)
                            mma_f16_pair(d, sdesc_sw128(a0 + 32 * k), sdesc_sw128(b0 + 32 * k), idesc,
                                         (kb | k) != 0);
                        mma_commit_pair(&empty[s]);  // frees the stage in both CTAs
                    } else {
                        for (int k = 0; k < ksteps; ++k)
                            mma_f16(d, sdesc_sw128(a0 + 32 * k), sdesc_sw128(b0 + 32 * k), idesc, (kb | k) != 0);
                        mma_commit(&empty[s]);
                    }
                }
                if (!alive) break;
                if constexpr (CG == 2) mma_commit_pair(&acc_full[buf]);
                else mma_commit(&acc_full[buf]);
                nkb = nkb_n;
                klast = klast_n;
            }
        }
    } else {
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;  // this warp's number within its quarter
        constexpr int kParts = Cfg::EW / 4;
        constexpr int kChunks = BN / 64;  // 32-column chunks per epilogue warp (8 warps)
        int tcount = 0;
        uint32_t boxes = 0;  // staged boxes this warp has issued (selects its staging tile)
        // this CTA's 128 rows of the tile
        const uint32_t acc_empty_leader = CG == 2 ? map_to_cta(smem_u32(&acc_empty[0]), 0) : 0;
        int4 tl_c = make_int4(0, 0, 0, 0);
        ops::GemmGroup g = {};
        if (cta_tile0 < ntiles) {
            tl_c = tiles[2 * cta_tile0];
            g = groups[tl_c.x];
        }
        for (int t = cta_tile0; t < ntiles; t += cta_tile_step, ++tcount) {
            int4 tl = tl_c;
            tl.y += (int)rank * BM;
            if (t + cta_tile_step < ntiles) tl_c = tiles[2 * (t + cta_tile_step)];  // the next tile's, in flight
            const int buf = tcount & 1;
            const uint32_t use = tcount >> 1;
            if (!mbar_wait(&acc_full[buf], use & 1, err)) break;
            tc_fence_after();
            const int row = tl.y + q * 32 + lane;
            const bool rv = row < g.M;
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + buf * BN + half * (BN / 2);
            constexpr bool kStoresViaTma = EPI == ops::EPI_F32 || EPI == ops::EPI_ADD_F32 || EPI == ops::EPI_T ||
                                           EPI == ops::EPI_GELU_T || EPI == ops::EPI_TANH_T;
            if (EPI == ops::EPI_ROPE_T && c_tma) {
                // RoPE output: warp half `half` takes pair half `half` of every
                // head in the tile (columns 64 h + 32 half .. + 32), so one row
                // of 16 (cos, sin) pairs, loaded once, serves all its chunks.
                // Each 32-column chunk is one 32 x 32 box (64-byte rows, 64-byte
                // swizzle); a warp's staging space holds 2 NSTG boxes in turn.
                constexpr int kHeads = BN / 64;
                constexpr int kSlots = 2 * Cfg::NSTG;
                const int rrow = tl.y + q * 32 + lane;
                const int rpos = qkv.mode == ops::SEQ_TIME ? (rrow / qkv.NB) % qkv.T : rrow % qkv.NB;
                float4 tc[4], ts[4];
                load_rope16(qkv.cos_t + rpos * 32, qkv.sin_t + rpos * 32, half * 16, tc, ts);
                const int DI = qkv.H * 64;
                const int yrow = tl.y + q * 32;
                uint8_t* stg_base = smem + Cfg::STAGING_OFF + (warp - 2) * Cfg::STG_WARP;
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * BN + half * 32;
#pragma unroll 1
                for (int h = 0; h < kHeads; ++h) {
                    const int n0 = tl.z + h * 64 + half * 32;
                    if (n0 >= g.N) break;
                    uint32_t r[32];
                    tmem_ld32(tbase + h * 64, r);
                    tmem_ld_wait(r);
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                    apply_epi<EPI>(g, n0, v);
                    if (n0 / DI < 2) rope_apply16(tc, ts, v);  // q and k sections
                    uint8_t* stg = stg_base + (boxes % kSlots) * (kStagingPerWarp / 2);
                    if (lane == 0) bulk_wait_read_n<kSlots - 1>();  // the store issued from this slot has read it
                    __syncwarp();
                    stage_chunk64<T>(stg, lane, v);
                    fence_async_smem();
                    __syncwarp();
                    if (yrow < g.M) {
                        if (lane == 0) {
                            tma_store_3d(&tmC, stg, n0, c_tma == 2 ? g.c_group : yrow, c_tma == 2 ? yrow : g.c_group);
                            bulk_commit();
                        }
                        ++boxes;
                    }
                }
            } else if (EPI == ops::EPI_GELU_T && c_tma) {
                // GELU output, 12 warps: the three warps of a lane quarter take
                // the tile's 32-column chunks in turn (chunk c to warp c % 3);
                // each chunk is one 32 x 32 box (64-byte rows, 64-byte swizzle)
                // staged in the warp's 2 KB and stored by TMA.
                uint8_t* stg = smem + Cfg::STAGING_OFF + (warp - 2) * Cfg::STG_WARP;
                const int yrow = tl.y + q * 32;
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * BN;
#pragma unroll 1
                for (int c = half; c < BN / 32; c += kParts) {
                    const int n0 = tl.z + c * 32;
                    if (n0 >= g.N) break;
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait(r);
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                    apply_epi<EPI>(g, n0, v);
                    if (lane == 0) bulk_wait_read_all();  // the previous box's store has read the staging
                    __syncwarp();
                    stage_chunk64<T>(stg, lane, v);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0 && yrow < g.M) {
                        tma_store_3d(&tmC, stg, n0, c_tma == 2 ? g.c_group : yrow, c_tma == 2 ? yrow : g.c_group);
                        bulk_commit();
                    }
                }
            } else if (kStoresViaTma && c_tma) {
                // stage through this warp's 32-row tiles (NSTG of them, used in
                // turn); one TMA store (or reduce-add into the fp32 residual)
                // per 128-byte row group.  The TMEM load of the next 32 columns
                // is in flight while the current ones are processed.
                constexpr bool k16 = !(EPI == ops::EPI_F32 || EPI == ops::EPI_ADD_F32);
                uint8_t* stg_base = smem + Cfg::STAGING_OFF + (warp - 2) * Cfg::STG_WARP;
                const int yrow = tl.y + q * 32;
                const int ncol = g.N - (tl.z + half * (BN / 2));
                const int nch = ncol <= 0 ? 0 : (ncol >= 32 * kChunks ? kChunks : (ncol + 31) / 32);
                // the next chunk's TMEM load is issued before this chunk's math
                uint32_t r[32];
                if (nch > 0) tmem_ld32(taddr, r);
#pragma unroll 1
                for (int c = 0; c < nch; ++c) {
                    const int n0 = tl.z + half * (BN / 2) + c * 32;
                    tmem_ld_wait(r);
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                    if (c + 1 < nch) tmem_ld32(taddr + (c + 1) * 32, r);
                    apply_epi<EPI>(g, n0, v);
                    const int h16 = k16 ? (c & 1) : 0;
                    uint8_t* stg = stg_base + (Cfg::NSTG == 2 ? (boxes & 1) : 0) * kStagingPerWarp;
                    if (h16 == 0) {  // a staging tile is free once the store issued from it has read it
                        if (lane == 0) {
                            if constexpr (Cfg::NSTG == 2) bulk_wait_read_1();
                            else bulk_wait_read_all();
                        }
                        __syncwarp();
                    }
                    stage_chunk<T, EPI>(stg, lane, h16, v);
                    const bool flush = !k16 || h16 == 1 || c + 1 == kChunks || n0 + 32 >= g.N;
                    if (flush) {
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0 && yrow < g.M) {  // boxes wholly below the last row are skipped
                            const int x = k16 ? n0 - 32 * h16 : n0;
                            const int y = c_tma == 2 ? g.c_group : yrow;
                            const int z = c_tma == 2 ? yrow : g.c_group;
                            if constexpr (EPI == ops::EPI_ADD_F32) tma_reduce_add_3d(&tmC, stg, x, y, z);
                            else tma_store_3d(&tmC, stg, x, y, z);
                            bulk_commit();
                        }
                        if (yrow < g.M) ++boxes;  // a skipped box leaves its staging tile free for the next one
                    }
                }
            } else {
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * BN;
#pragma unroll 1
                for (int c = half; c < BN / 32; c += kParts) {  // chunk c to warp c % kParts of the quarter
                    const int n0 = tl.z + c * 32;
                    if (n0 >= g.N) break;
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait();
                    if (rv) {
                        if constexpr (EPI == ops::EPI_QKV) {
                            epilogue_qkv<T>(qkv, row, n0, r);
                        } else if constexpr (EPI == ops::EPI_ROPE_T) {
                            float v[32];
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                            apply_epi<EPI>(g, n0, v);
                            rope_rotate(qkv, row, n0, v);
                            uint4* c4 = reinterpret_cast<uint4*>((T*)g.C + (int64_t)row * g.ldc + n0);
#pragma unroll
                            for (int j = 0; j < 4; ++j)  // N is a multiple of 64 (checked on the host)
                                c4[j] = make_uint4(pack2(v[8 * j], v[8 * j + 1], (T*)nullptr),
                                                   pack2(v[8 * j + 2], v[8 * j + 3], (T*)nullptr),
                                                   pack2(v[8 * j + 4], v[8 * j + 5], (T*)nullptr),
                                                   pack2(v[8 * j + 6], v[8 * j + 7], (T*)nullptr));
                        }
                        else {
                            epilogue_chunk<T, EPI>(g, row, n0, r);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (CG == 2) mbar_arrive_cluster(acc_empty_leader + 8u * buf);  // the leader's barrier
                else mbar_arrive(&acc_empty[buf]);
            }
            if (t + cta_tile_step < ntiles) g = groups[tl_c.x];  // loads in flight until the next tile's wait
        }
        if (lane == 0) bulk_wait_all();  // outstanding TMA stores complete before exit
    }
    tc_fence_before();
    if constexpr (CG == 2) cluster_sync();  // no CTA leaves while its peer may still touch its memory
    else __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (CG == 2) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
        else tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

// ---- host: tensor maps ----
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

void make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows, int dtype) {
    MBR_CHECK(((uintptr_t)base & 15) == 0, "TMA base must be 16-byte aligned");
    MBR_CHECK((cols * 2) % 16 == 0, "TMA row pitch must be a multiple of 16 bytes");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(m, dtype == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

// Output map C[group][row][col] for the staged TMA stores: box = one warp's
// 32 rows x 128 bytes, 128-byte swizzle (the layout stage_chunk writes).
// The two outer dimensions are ordered by increasing stride; `swapped` tells
// the kernel that the group dimension comes before the row dimension.
// box_bytes: the inner extent of one store box, 128 (128-byte swizzle,
// 32 rows) or 64 (64-byte swizzle, 32 rows, the RoPE epilogue).
void make_out_map(CUtensorMap* m, const GemmPlanTC& p, bool& swapped, int box_bytes) {
    const int64_t es = p.c_dtype == DT_F32 ? 4 : 2;
    MBR_CHECK(((uintptr_t)p.c_base & 15) == 0, "TMA output base must be 16-byte aligned");
    MBR_CHECK((p.c_row_stride * es) % 16 == 0 && (p.c_group_stride * es) % 16 == 0,
              "TMA output strides must be multiples of 16 bytes");
    swapped = p.c_groups > 1 && p.c_group_stride < p.c_row_stride;
    cuuint64_t dims[3] = {(cuuint64_t)p.c_cols, (cuuint64_t)p.c_rows, (cuuint64_t)p.c_groups};
    cuuint64_t strides[2] = {(cuuint64_t)(p.c_row_stride * es), (cuuint64_t)(p.c_group_stride * es)};
    cuuint32_t box[3] = {(cuuint32_t)(box_bytes / es), 32, 1};
    if (swapped) {
        std::swap(dims[1], dims[2]);
        std::swap(strides[0], strides[1]);
        std::swap(box[1], box[2]);
    }
    cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMapDataType t = p.c_dtype == DT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                            : p.c_dtype == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = encode_fn()(m, t, 3, const_cast<void*>(p.c_base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE,
                             box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(ERR_CUDA, "cuTensorMapEncodeTiled (output) failed: " + std::to_string((int)r));
}

// MBR_GEMM_PAIRS=0 keeps every GEMM on single-CTA tiles (A/B comparisons).
bool pair_tiles_off() {
    static const bool off = [] {
        const char* e = std::getenv("MBR_GEMM_PAIRS");
        return e && e[0] == '0';
    }();
    return off;
}

int num_sms() {
    int dev = 0, n = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    return n;
}

template <typename T, int BN, int EPI, int CG>
void launch_cg(const GemmLaunch& L, int* d_err, cudaStream_t st) {
    auto kern = gemm_tc_kernel<T, BN, EPI, CG>;
    using Cfg = TileCfg<BN, CG, EPI>;
    static bool attr[64] = {};  // per instantiation and device
    static int sms[64] = {};
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < 64, "device index out of range");
    if (!attr[dev]) {
        MBR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
        sms[dev] = num_sms();
        attr[dev] = true;
    }
    // persistent: one CTA (pair) per SM (pair), at most one per tile
    const int grid = CG * std::min(L.ntiles, sms[dev] / CG);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(gemm_threads(EPI));
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CG;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    MBR_CUDA(cudaLaunchKernelEx(&cfg, kern, L.tmA, L.tmB, L.tmC, L.c_tma, L.groups, L.tiles, L.ntiles, d_err, L.qkv));
}

template <typename T, int BN, int EPI>
void launch_one(const GemmLaunch& L, int* d_err, cudaStream_t st) {
    if (L.cg == 2) launch_cg<T, BN, EPI, 2>(L, d_err, st);
    else launch_cg<T, BN, EPI, 1>(L, d_err, st);
}

template <typename T, int BN>
void launch_bn(const GemmLaunch& L, int* d_err, cudaStream_t st) {
    switch (L.epi) {
        case ops::EPI_F32: launch_one<T, BN, ops::EPI_F32>(L, d_err, st); break;
        case ops::EPI_T: launch_one<T, BN, ops::EPI_T>(L, d_err, st); break;
        case ops::EPI_ADD_F32: launch_one<T, BN, ops::EPI_ADD_F32>(L, d_err, st); break;
        case ops::EPI_GELU_T: launch_one<T, BN, ops::EPI_GELU_T>(L, d_err, st); break;
        case ops::EPI_TANH_T: launch_one<T, BN, ops::EPI_TANH_T>(L, d_err, st); break;
        case ops::EPI_GLU_F32: launch_cg<T, BN, ops::EPI_GLU_F32, 1>(L, d_err, st); break;
        case ops::EPI_QKV: launch_cg<T, BN, ops::EPI_QKV, 1>(L, d_err, st); break;
        case ops::EPI_ROPE_T: launch_one<T, BN, ops::EPI_ROPE_T>(L, d_err, st); break;
        default: throw Error(ERR_INVALID, "tc gemm: bad epilogue");
    }
}

template <typename T>
void launch_t(const GemmLaunch& L, int* d_err, cudaStream_t st) {
    if (L.bn == 256) launch_bn<T, 256>(L, d_err, st);
    else if (L.bn == 192) launch_bn<T, 192>(L, d_err, st);
    else launch_bn<T, 128>(L, d_err, st);
}

}  // namespace

bool gemm_supported(int epi) { return epi >= ops::EPI_F32 && epi <= ops::EPI_ROPE_T; }

void gemm_prepare(const GemmPlanTC& p, int dtype, std::vector<int4>& tiles, GemmLaunch& L, size_t& L_first) {
    MBR_CHECK(dtype == DT_F16 || dtype == DT_BF16, "tc gemm needs fp16 or bf16 operands");
    // 16-bit staged stores pair two 32-column chunks per 128-byte box, so a
    // warp's column half (BN / 2) must hold an even number of chunks: BN 192
    // would leave a half-filled box spilling into the neighbouring columns.
    const bool staged16 = p.c_dtype >= 0 && p.c_dtype != DT_F32;
    int bn;
    if (p.epi == ops::EPI_GLU_F32) bn = 128;
    else if (p.maxN % 256 == 0) bn = 256;
    else if (p.maxN % 192 == 0 && !staged16) bn = 192;
    else if (p.maxN % 128 == 0 || p.maxN < 256) bn = 128;
    else bn = 256;
    L.bn = bn;
    L.epi = p.epi;
    if (p.epi == ops::EPI_ROPE_T)
        MBR_CHECK(L.qkv.cos_t && L.qkv.sin_t && L.qkv.H > 0 && p.maxN == 3 * L.qkv.H * 64 && p.c_dtype == dtype,
                  "tc gemm: RoPE epilogue needs head dim 64, the rope tables and a 16-bit output view");
    if (p.epi == ops::EPI_QKV)
        MBR_CHECK(L.qkv.q && L.qkv.k && L.qkv.v && L.qkv.cos_t && L.qkv.H > 0 && p.maxN == 3 * L.qkv.H * 64 &&
                      bn % 64 == 0,
                  "tc gemm: QKV epilogue needs head dim 64 and its q/k/v/rope buffers");
    make_map(&L.tmA, p.a_base, p.a_rows, p.a_cols, BM, dtype);
    // CTA pairs (256-row tiles, cta_group::2) for the large residual GEMMs
    // (out-projection, FFN2): each CTA loads half of the B tile.  For the
    // 16-bit-output GEMMs with K = 384 (QKV, FFN1) the pair's coupled
    // epilogues cost more than the halved B traffic saves, measured on B200.
    L.cg = p.c_dtype >= 0 && p.epi == ops::EPI_ADD_F32 && p.maxM >= 4096 && !pair_tiles_off() ? 2 : 1;
    make_map(&L.tmB, p.b_base, p.b_rows, p.b_cols, bn / L.cg, dtype);
    L_first = tiles.size();
    for (int gi = 0; gi < p.ngroups; ++gi) {
        const ops::GemmGroup& g = p.h_groups[gi];
        MBR_CHECK(g.K % 16 == 0 && g.K > 0, "tc gemm: K must be a positive multiple of 16");
        MBR_CHECK((int64_t)g.a_row0 + g.M <= p.a_rows && (int64_t)g.b_row0 + g.N <= p.b_rows &&
                      (int64_t)g.k_col0 + g.K <= p.a_cols && (int64_t)g.k_col0 + g.K <= p.b_cols,
                  "tc gemm: group outside its operand tensors");
        MBR_CHECK(g.k_col0 % 8 == 0, "tc gemm: K offset must be 16-byte aligned");
        const int kb = (int)ceil_div(g.K, BK);
        const int klast = (g.K - (kb - 1) * BK) / 16;  // k-steps of the last k-block
        // two int4 per tile: {group, m0, n0, k-blocks} and the operand coordinates
        // {A row, B row, first K column, k-steps of the last k-block}
        for (int m0 = 0; m0 < g.M; m0 += BM * L.cg)
            for (int n0 = 0; n0 < g.N; n0 += bn) {
                tiles.push_back(make_int4(gi, m0, n0, kb));
                tiles.push_back(make_int4(g.a_row0 + m0, g.b_row0 + n0, g.k_col0, klast));
            }
    }
    L.ntiles = (int)((tiles.size() - L_first) / 2);
    L.groups = p.groups;
    L.c_tma = 0;
    const bool staged_epi = p.epi == ops::EPI_F32 || p.epi == ops::EPI_ADD_F32 || p.epi == ops::EPI_T ||
                            p.epi == ops::EPI_GELU_T || p.epi == ops::EPI_TANH_T || p.epi == ops::EPI_ROPE_T;
    if (p.c_dtype >= 0 && staged_epi) {
        const bool f32 = p.epi == ops::EPI_F32 || p.epi == ops::EPI_ADD_F32;
        MBR_CHECK(f32 ? p.c_dtype == DT_F32 : p.c_dtype == dtype, "tc gemm: output view dtype mismatch");
        const int64_t es = f32 ? 4 : 2;
        // The staged stores write whole 32-row x 128-byte boxes and rely on the
        // map's bounds for clipping, so every group must cover its output block
        // exactly and agree with its own C / ldc.
        for (int gi = 0; gi < p.ngroups; ++gi) {
            const ops::GemmGroup& g = p.h_groups[gi];
            MBR_CHECK(g.M == p.c_rows && g.N == p.c_cols && g.c_group >= 0 && g.c_group < p.c_groups &&
                          g.ldc == p.c_row_stride &&
                          (const char*)g.C == (const char*)p.c_base + (int64_t)g.c_group * p.c_group_stride * es,
                      "tc gemm: group does not match the output view");
        }
        bool swapped = false;
        make_out_map(&L.tmC, p, swapped,
                     p.epi == ops::EPI_ROPE_T || p.epi == ops::EPI_GELU_T ? 64 : kStageRowBytes);
        L.c_tma = swapped ? 2 : 1;
    }
    L.ok = true;
}

void gemm_launch(const GemmLaunch& L, int dtype, int* d_err, cudaStream_t st) {
    MBR_CHECK(L.ok, "tc gemm launch not prepared");
    if (L.ntiles == 0) return;
    if (dtype == DT_BF16) launch_t<__nv_bfloat16>(L, d_err, st);
    else launch_t<__half>(L, d_err, st);
}

}  // namespace tc
}  // namespace mbr
