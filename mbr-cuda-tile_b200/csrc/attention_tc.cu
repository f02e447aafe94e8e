// attention_tc.cu — tcgen05 flash attention for the time axis (L = T frames,
// 64-key blocks) and the band axis (L <= 64 bands, two sequences packed per
// 128-row tile, each attending only its own key block), head dim 64,
// fp16/bf16.
//
// One CTA (two per SM) = one 128-query tile of one (sequence, head) [or two
// packed band sequences]: warps 0-3 run the softmax (thread r = query row r =
// TMEM lane r), warp 4 issues the TMA loads and warp 5 the MMAs.  Per 64-key
// block j:
//   S(j) = Q K(j)^T       -> TMEM buffer j%2 (128 x 64 fp32)
//   P(j) = exp2(S*c - m)  -> TMEM buffer j%2 (16-bit pairs)
//   O   += P(j) V(j)      -> TMEM (128 x 64 fp32), A operand read from TMEM
// S(j+2) is computed while the softmax works on S(j+1), so the softmax warps
// do not wait for the tensor cores; K and V stream through their own rings.
// V keeps the [seq][H][L][64] layout of q and k: its 64-key tile is the
// MN-major B operand of the P.V product.  The epilogue multiplies by the
// sigmoid gate (loaded at the tile's start) and writes the merged-head row of
// each token (apply_gates_and_merge_heads).  All waits are bounded (error word
// instead of a hang).
//
// Warps whose 32 query rows all lie past the sequence end (the last query
// tile's tail) compute no exponentials.
#include <cuda.h>

#include <algorithm>
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
constexpr int KB = 64;   // keys per block (one 128-byte swizzle atom of P per row)
// The exponent offset of a row is raised (O and l rescaled) only when a
// block's probabilities computed with the current offset sum to more than
// this; every probability then stays below 2^14 (fp16 range) and sums of
// stale-offset probabilities need no separate row max.
constexpr float kRescaleSum = 16384.0f;

// Shared-memory plan: NQ Q tiles in flight (persistent CTAs prefetch the next
// tiles; band tiles have only two key blocks, so they prefetch further), an
// NSK-stage K ring and an NSV-stage V ring.  A K stage is refilled two blocks
// after the S that read it was issued, a V stage four blocks after (its P.V
// completes behind the S two blocks later), so the V ring is the deeper one:
// both give their loads the same lead.  Two CTAs share an SM, so the layout
// carries no alignment slack: the kernel checks that the dynamic window is
// 1024-byte aligned instead.
template <bool PACK>
struct AttnCfg {
    static constexpr int NSK = PACK ? 3 : 4;  // K stages of 64 x 64 (8 KB each)
    static constexpr int NSV = PACK ? 5 : 6;  // V stages
    static constexpr int NQ = PACK ? 3 : 2;   // Q tiles of 128 x 64 (16 KB)
    static constexpr int Q = 0;
    static constexpr int K = NQ * 16384;
    static constexpr int V = K + NSK * 8192;
    static constexpr int BAR = V + NSV * 8192;
    static constexpr int TOTAL = BAR + 256;
    static_assert(2 * (TOTAL + 1024) <= 233472, "two CTAs per SM");
};
// TMEM columns (256 allocated): S double buffer (fp32) at 0 and 64, O at 128.
// Time axis: P double buffer (16-bit pairs, the A operand of P.V) at 192 and
// 224.  Band axis (two key blocks per tile, so the per-tile epilogue weighs
// more): each block's P is written over the first 32 columns of its own S once
// the softmax has read S, and O is double buffered by tile parity at 128 and
// 192, so a tile's output is read while the next tile's blocks already
// accumulate (measured: band 23 % faster per step; the time axis, 13 blocks
// per tile, measured 7 % slower this way and keeps separate P buffers).
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemO = 128, kTmemP = 192;

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


// 2^x with the hardware approximation (relative error ~2^-22; the
// probabilities are rounded to 16 bits right after).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T, bool PACK>
__global__ void __maxnreg__(168)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, int nsh, int H, int L, int n_lo, float scale_log2,
                   const float* __restrict__ gates, int mode, int NB, int Tn, T* __restrict__ merged, int* err) {
    using AttnSmem = AttnCfg<PACK>;
    constexpr int NSK = AttnSmem::NSK, NSV = AttnSmem::NSV, NQ = AttnSmem::NQ;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (!smem_aligned_or_flag(smem_raw, err)) return;  // uniform over the CTA
    uint8_t* sm = smem_raw;
    uint64_t* bar = (uint64_t*)(sm + AttnSmem::BAR);
    uint64_t* bar_q = bar;               // [NQ] Q tile landed
    uint64_t* bar_k = bar + NQ;          // [NSK] K stage landed
    uint64_t* bar_v = bar_k + NSK;       // [NSV] V stage landed
    uint64_t* bar_s = bar_v + NSV;       // [2] S buffer computed
    uint64_t* bar_p = bar_s + 2;         // [2] softmax done with S buffer, P buffer written (4 warps)
    uint64_t* bar_o = bar_p + 2;         // [2] P.V from P buffer complete (last two blocks)
    uint64_t* kv_free = bar_o + 2;       // [NSK] block g's P arrived: its K stage and V(g-2)'s are free
    uint64_t* o_free = kv_free + NSK;    // [2] O buffer read by the softmax's epilogue (4 warps)
    uint32_t* tmem_slot = (uint32_t*)(o_free + 2);
    static_assert((NQ + 2 * NSK + NSV + 8) * 8 + 4 <= 256, "barrier region");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Persistent CTAs: this CTA takes tiles blockIdx.x, + gridDim.x, ...  Time
    // axis: tile = one 128-query tile of sequence-head sh0, 64-key blocks;
    // band axis (PACK): tile = sequence-heads sh0 (rows 0-63) and sh1 (rows
    // 64-127), key block j = the keys of sh_j.  The blocks of all of this
    // CTA's tiles form one stream g = local tile * nkv + j for the pipelines.
    const int qtiles = PACK ? 1 : (L + QT - 1) / QT;
    const int ntiles = PACK ? (nsh + 1) / 2 : nsh * qtiles;
    const int nkv = PACK ? 2 : (L + KB - 1) / KB;
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = my_tiles * nkv;
    auto tile_of = [&](int tl, int& sh0, int& sh1, int& q0) {
        const int t = (int)blockIdx.x + tl * (int)gridDim.x;
        if (PACK) {
            sh0 = 2 * t;
            sh1 = min(sh0 + 1, nsh - 1);
            q0 = 0;
        } else {
            sh0 = t / qtiles;
            sh1 = sh0;
            q0 = (t - sh0 * qtiles) * QT;
        }
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < NQ; ++i) mbar_init(&bar_q[i], 1);
        for (int i = 0; i < NSK; ++i) {
            mbar_init(&bar_k[i], 1);
            mbar_init(&kv_free[i], 1);
        }
        for (int i = 0; i < NSV; ++i) mbar_init(&bar_v[i], 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar_s[i], 1);
            mbar_init(&bar_p[i], 4);
            mbar_init(&bar_o[i], 1);
            mbar_init(&o_free[i], 4);
        }
        fence_barrier_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tO = tmem + kTmemO;

    if (warp >= 4) {
        // ---- warp 4: TMA producer; warp 5: MMA issuer.  One elected lane
        // issues, all lanes wait. ----
        auto wait_all = [&](uint64_t* b, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(b, parity, err));
        };
        // TMA coordinates (d, head, position, sequence % n_lo, sequence / n_lo)
        // of sequence-head sh
        auto seq_coords = [&](int sh, int& h, int& slo, int& shi) {
            const int s = sh / H;
            h = sh - s * H;
            shi = s / n_lo;
            slo = s - shi * n_lo;
        };
        // Position in the block stream without per-block divisions: block g is
        // key block j of local tile tl, starting at key position p of the
        // sequence-head with coordinates (h, slo, shi).
        struct Cursor {
            int g, tl, j, h, p, slo, shi;
        };
        auto set_block = [&](Cursor& c) {
            int sh0, sh1, q0;
            tile_of(c.tl, sh0, sh1, q0);
            seq_coords(PACK && c.j ? sh1 : sh0, c.h, c.slo, c.shi);
            c.p = PACK ? 0 : c.j * KB;
        };
        auto cursor_at = [&](int g) {  // called a few times before the loop only
            Cursor c;
            c.g = g;
            c.tl = g / nkv;
            c.j = g - c.tl * nkv;
            if (c.tl < my_tiles) set_block(c);
            return c;
        };
        auto advance = [&](Cursor& c) {
            ++c.g;
            if (++c.j == nkv) {
                c.j = 0;
                ++c.tl;
                if (c.tl < my_tiles) set_block(c);
            } else if (PACK) {
                set_block(c);
            } else {
                c.p += KB;
            }
        };
        auto load_q = [&](int tl) {
            int sh0, sh1, q0, h, slo, shi;
            tile_of(tl, sh0, sh1, q0);
            const int qb = tl % NQ;
            uint8_t* dst = sm + AttnSmem::Q + qb * 16384;
            mbar_arrive_expect_tx(&bar_q[qb], 16384);
            seq_coords(sh0, h, slo, shi);
            tma_load_5d(dst, &tmQ, 0, h, q0, slo, shi, &bar_q[qb]);
            if (PACK) {
                seq_coords(sh1, h, slo, shi);
                tma_load_5d(dst + 8192, &tmQ, 0, h, 0, slo, shi, &bar_q[qb]);
            }
        };
        auto load_k = [&](const Cursor& c) {
            const int st = c.g % NSK;
            mbar_arrive_expect_tx(&bar_k[st], 8192);
            tma_load_5d(sm + AttnSmem::K + st * 8192, &tmK, 0, c.h, c.p, c.slo, c.shi, &bar_k[st]);
        };
        auto load_v = [&](const Cursor& c) {
            const int st = c.g % NSV;
            mbar_arrive_expect_tx(&bar_v[st], 8192);
            tma_load_5d(sm + AttnSmem::V + st * 8192, &tmV, 0, c.h, c.p, c.slo, c.shi, &bar_v[st]);
        };
        constexpr uint32_t idS = idesc_f16(QT, KB, IsBf16<T>::value);
        constexpr uint32_t idO = idesc_f16(QT, DH, IsBf16<T>::value, /*b_mn_major=*/true);
        // descriptor bases; the start-address field (16-byte units) advances
        // by 2 per 32 bytes along K, by 512 per 8 KB stage, 1024 per 16 KB
        const uint64_t dQ = sdesc_sw128(smem_u32(sm + AttnSmem::Q));
        const uint64_t dK = sdesc_sw128(smem_u32(sm + AttnSmem::K));
        const uint64_t dV = sdesc_sw128_mn(smem_u32(sm + AttnSmem::V));
        auto issue_s = [&](const Cursor& c) {  // S buffer (g & 1) = Q(tile) K(g)^T
            const uint64_t q = dQ + (uint64_t)(1024 * (c.tl % NQ));
            const uint64_t k0 = dK + (uint64_t)(512 * (c.g % NSK));
            const uint32_t d = tmem + (uint32_t)(64 * (c.g & 1));
#pragma unroll
            for (int k = 0; k < DH / 16; ++k) mma_f16(d, q + 2 * k, k0 + 2 * k, idS, k > 0);
            mma_commit(&bar_s[c.g & 1]);
        };
        auto issue_pv = [&](const Cursor& c) {  // O(tile % 2) (+)= P(g) V(g), P read from TMEM; O restarts per tile
            const uint32_t a0 = PACK ? tmem + 64 * (c.g & 1) : tmem + kTmemP + 32 * (c.g & 1);
            const uint32_t d = PACK ? tO + 64 * (c.tl & 1) : tO;
            const uint64_t b0 = dV + (uint64_t)(512 * (c.g % NSV));
#pragma unroll
            for (int k = 0; k < KB / 16; ++k)  // A: keys 16k.. = 8 packed columns; B: V keys 16k.. (MN-major, 2 KB)
                mma_f16_ts(d, a0 + 8 * k, b0 + 128 * k, idO, c.j != 0 || k > 0);
            // P.V(g) completes ahead of S(g+2), issued right behind it, whose
            // commit the softmax waits for instead; only the last two blocks,
            // which no S follows, commit their own barrier (one commit each)
            if (c.g + 2 >= total) mma_commit(&bar_o[c.g & 1]);
        };

        if (warp == 4) {
            // Loads.  Stages are handed back by the MMA warp's plain arrive on
            // kv_free[g % NSK] once it has seen P(g): S(g) has completed, so K
            // stage g is free, and so has P.V(g-2), issued before S(g), so V
            // stage g-2 is free.  The MMA warp runs at most NSK - 2 blocks
            // ahead of these loads (S(g+2) needs K(g+2)), so the ring's parity
            // waits are exact.
            Cursor ck = cursor_at(min(NSK, total));  // next K load
            Cursor cv = cursor_at(min(NSV, total));  // next V load
            if (lane == 0) {
                prefetch_tensormap(&tmQ);
                prefetch_tensormap(&tmK);
                prefetch_tensormap(&tmV);
                for (int tl = 0; tl < NQ && tl < my_tiles; ++tl) load_q(tl);
                Cursor c = cursor_at(0);
                for (int g = 0; g < NSV && g < total; ++g, advance(c)) {
                    if (g < NSK) load_k(c);
                    load_v(c);
                }
            }
            __syncwarp();
            bool ok = true;
            for (Cursor cf = cursor_at(0); cf.g < total && ok; advance(cf)) {
                const int g = cf.g;
                ok = wait_all(&kv_free[g % NSK], (g / NSK) & 1);
                if (!ok) break;
                if (ck.g < total) {
                    if (lane == 0) load_k(ck);
                    advance(ck);
                }
                if (g >= 2 && cv.g < total) {
                    if (lane == 0) load_v(cv);
                    advance(cv);
                }
                // after a tile's last block (its last S has completed) its Q buffer -> Q(tile + NQ)
                if (lane == 0 && cf.j == nkv - 1 && cf.tl + NQ < my_tiles) load_q(cf.tl + NQ);
                __syncwarp();
            }
        } else {
            // S(g) needs its tile's Q (at the tile's first block), K(g) and, for
            // the P.V(g) issued later, V(g)
            auto s_ready = [&](const Cursor& c) -> bool {
                if (c.j == 0 && !wait_all(&bar_q[c.tl % NQ], (c.tl / NQ) & 1)) return false;
                return wait_all(&bar_k[c.g % NSK], (c.g / NSK) & 1) && wait_all(&bar_v[c.g % NSV], (c.g / NSV) & 1);
            };
            Cursor cs = cursor_at(0);  // next S to issue
            Cursor cp = cs;            // next P.V
            // S(0), S(1) go ahead; afterwards S(g+2) is issued once the softmax
            // has consumed S(g) (its buffer), right behind P(g).V(g).
            bool ok = true;
            for (int g = 0; g < 2 && g < total && ok; ++g, advance(cs)) {
                ok = s_ready(cs);
                if (ok) {
                    tc_fence_after();
                    if (elect_one()) issue_s(cs);
                    __syncwarp();
                }
            }
            for (; cp.g < total && ok; advance(cp)) {
                const int g = cp.g;
                ok = wait_all(&bar_p[g & 1], (g >> 1) & 1);
                if (!ok) break;
                if (lane == 0) mbar_arrive(&kv_free[g % NSK]);  // the producer may refill
                // a tile's first P.V overwrites the O buffer of the tile two
                // before, once the softmax's epilogue has read it
                if (PACK && cp.j == 0 && cp.tl >= 2) ok = wait_all(&o_free[cp.tl & 1], ((cp.tl >> 1) - 1) & 1);
                if (!ok) break;
                tc_fence_after();
                if (elect_one()) issue_pv(cp);  // V(g) landed: s_ready(g) waited for it
                __syncwarp();
                // S(g+2) into the buffer S(g) held, behind P.V(g): its completion
                // (bar_s) also tells the softmax that P buffer g%2 is free again
                // and that P.V(g) is complete
                if (cs.g < total) {
                    ok = s_ready(cs);
                    if (!ok) break;
                    tc_fence_after();
                    if (elect_one()) issue_s(cs);
                    __syncwarp();
                    advance(cs);
                }
            }
        }
    } else {
        // ---- softmax warps: thread r owns query row r (TMEM lane r) ----
        // O accumulates in TMEM over a tile's key blocks.  The exponent offset
        // m is the first block's row max and is raised (O and l rescaled in
        // place) only when a later block's probabilities sum to more than
        // kRescaleSum, so P < 2^14 and O / l is the same softmax.
        const int r = threadIdx.x;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        // P.V(x) is complete: through S(x+2), issued right behind it, or the
        // block's own commit when no S follows (the last two blocks)
        auto wait_pv = [&](int x) -> bool {
            const bool ok1 = x + 2 < total ? mbar_wait(&bar_s[x & 1], ((x + 2) >> 1) & 1, err)
                                           : mbar_wait(&bar_o[x & 1], 0, err);
            return __all_sync(0xffffffffu, ok1);
        };
        // A tile's output (band axis: after the next tile's first block, when
        // its last P.V has long completed): O of tile parity pd_par is read,
        // normalised, gated and stored, and the buffer handed back.
        bool pd_have = false, pd_valid = false;
        int64_t pd_tok = 0;
        float pd_gs = 0.f;
        int pd_hd = 0, pd_glast = 0, pd_par = 0;
        auto flush = [&]() -> bool {
            if (!wait_pv(pd_glast)) return false;
            tc_fence_after();
            const uint32_t tOp = tO + 64 * pd_par + lane_off;  // pd_par is 0 on the time axis
            uint32_t ov[DH / 32][32];
#pragma unroll
            for (int c = 0; c < DH / 32; ++c) tmem_ld32(tOp + c * 32, ov[c]);
            tmem_ld_wait();
            if (pd_valid) {
                uint4* dst = reinterpret_cast<uint4*>(merged + pd_tok * (int64_t)H * DH + pd_hd * DH);
#pragma unroll
                for (int q = 0; q < DH / 8; ++q) {
                    const uint32_t* o = &ov[q >> 2][(q & 3) * 8];
                    dst[q] = make_uint4(pack2(__uint_as_float(o[0]) * pd_gs, __uint_as_float(o[1]) * pd_gs, (T*)nullptr),
                                        pack2(__uint_as_float(o[2]) * pd_gs, __uint_as_float(o[3]) * pd_gs, (T*)nullptr),
                                        pack2(__uint_as_float(o[4]) * pd_gs, __uint_as_float(o[5]) * pd_gs, (T*)nullptr),
                                        pack2(__uint_as_float(o[6]) * pd_gs, __uint_as_float(o[7]) * pd_gs, (T*)nullptr));
                }
            }
            tc_fence_before();  // O read before the tile two ahead overwrites the buffer
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[pd_par]);
            pd_have = false;
            return true;
        };
        bool ok = true;  // warp-uniform: TMEM loads and stores are warp-collective
        for (int tl = 0; tl < my_tiles && ok; ++tl) {
        const uint32_t tOc = PACK ? tO + 64 * (tl & 1) : tO;  // this tile's O buffer
        int sh0, sh1, q0;
        tile_of(tl, sh0, sh1, q0);
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
        // this row's token and gate, loaded now so the load is long done by the epilogue
        int64_t tok = 0;
        float gate = 1.0f;
        if (valid) {
            const int64_t s = sh / H;
            tok = mode == ops::SEQ_TIME ? ((s / NB) * Tn + pos) * NB + (s % NB) : s * NB + pos;
            if (gates) gate = __ldg(gates + tok * H + sh % H);
        }
        float m = 0.f, l = 0.f;
        // a warp with no valid query row (the tail of the last query tile)
        // computes no exponentials: its P rows are written as zeros
        const bool wact = __any_sync(0xffffffffu, valid);
        for (int j = 0; j < nkv; ++j) {
            const int g = tl * nkv + j;
            const int b = g & 1;
            ok = __all_sync(0xffffffffu, ok && mbar_wait(&bar_s[b], (g >> 1) & 1, err));
            if (!ok) break;
            tc_fence_after();
            // valid key columns of this row in block j: [0, kend) (warp-uniform)
            const int kend = !wact ? 0 : PACK ? (j == seg ? min(L, KB) : 0) : min(KB, L - j * KB);
            uint32_t sv[2][32];
#pragma unroll
            for (int c = 0; c < 2; ++c)
                if (c * 32 < kend) tmem_ld32(tmem + lane_off + 64 * b + 32 * c, sv[c]);
            tmem_ld_wait();
            // P buffer b (or, band axis, the S(g) just read) is free: P.V(g-2),
            // its last reader, was issued before S(g), whose completion was
            // just observed
            const uint32_t tP = PACK ? tmem + lane_off + 64 * b : tmem + lane_off + kTmemP + 32 * b;
            // exponentials with offset mo -> P buffer b in TMEM as 16-bit pairs
            // (masked keys get zeros); returns the row sum of this block
            auto emit = [&](float mo) {
                float rsp[8];  // independent partial sums
#pragma unroll
                for (int u = 0; u < 8; ++u) rsp[u] = 0.f;
                uint32_t pk[32];
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    if (c * 32 >= kend) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) pk[16 * c + i] = 0u;
                        continue;
                    }
                    float p[32];
                    if (c * 32 + 32 <= kend) {  // whole chunk valid: no per-element masking
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            p[i] = fast_exp2(fmaf(__uint_as_float(sv[c][i]), scale_log2, -mo));
                            rsp[i & 7] += p[i];
                        }
                    } else {
                        const int nv = kend - c * 32;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            p[i] = i < nv ? fast_exp2(fmaf(__uint_as_float(sv[c][i]), scale_log2, -mo)) : 0.f;
                            rsp[i & 7] += p[i];
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) pk[16 * c + i] = pack2(p[2 * i], p[2 * i + 1], (T*)nullptr);
                }
                tmem_st32(tP, pk);
                return ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
            };
            // row max of the valid scores of this block (log2 units)
            auto row_max = [&]() {
                float mxp[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) mxp[u] = -INFINITY;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    if (c * 32 >= kend) continue;
                    const int nv = kend - c * 32;
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (nv >= 32 || i < nv) mxp[i & 7] = fmaxf(mxp[i & 7], __uint_as_float(sv[c][i]));
                }
                const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                       fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
                return mx * scale_log2;  // the scale is positive
            };
            float rs;
            if (j == 0) {
                // first block: the offset is this block's row max
                const float mb = row_max();
                m = mb == -INFINITY ? 0.f : mb;
                rs = emit(m);
            } else {
                // later blocks reuse the offset; a row whose probabilities grow
                // too large raises it to the block max (rare): O and l are
                // rescaled and the row of P is recomputed
                rs = emit(m);
                const bool need = !(rs <= kRescaleSum);  // also catches inf / nan
                if (__any_sync(0xffffffffu, need)) {
                    // O must hold exactly P.V of blocks < j: wait for P.V(g-1)
                    ok = wait_pv(g - 1);
                    if (!ok) break;
                    tc_fence_after();
                    const float m_new = need ? fmaxf(m, row_max()) : m;
                    const float alpha = fast_exp2(m - m_new);
                    m = m_new;
                    l *= alpha;
#pragma unroll 1
                    for (int c = 0; c < DH / 16; ++c) {  // 16 columns at a time: S is still live
                        uint32_t ov[16];
                        tmem_ld16(tOc + lane_off + c * 16, ov);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                        tmem_st16(tOc + lane_off + c * 16, ov);
                    }
                    tmem_st_wait();
                    rs = emit(m);
                }
            }
            l += rs;
            tmem_st_wait();    // P stores complete
            tc_fence_before();  // S reads / P and O stores ordered before the next MMAs
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_p[b]);
            if (PACK && j == 0 && pd_have) {  // the previous tile's output
                ok = flush();
                if (!ok) break;
            }
        }
        // this tile's output: on the band axis after the next tile's first block
        pd_have = ok;
        pd_valid = valid;
        pd_tok = tok;
        pd_gs = gate / l;
        pd_hd = sh % H;
        pd_glast = tl * nkv + nkv - 1;
        pd_par = PACK ? tl & 1 : 0;
        if (!PACK && ok) ok = flush();
        }  // tiles
        if (ok && pd_have) flush();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
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

// 5-D view (d, head, position, sequence % n_lo, sequence / n_lo) of q, k or v;
// the box is one head's 64 columns of `box_pos` consecutive positions.
void make_map(CUtensorMap* m, const void* base, const AttnLayout& lay, int H, int L, int box_pos, int dtype) {
    MBR_CHECK(((uintptr_t)base & 15) == 0, "attention TMA operand misaligned");
    const int64_t es = 2;
    cuuint64_t dims[5] = {(cuuint64_t)DH, (cuuint64_t)H, (cuuint64_t)L, (cuuint64_t)lay.n_lo, (cuuint64_t)lay.n_hi};
    cuuint64_t strides[4] = {(cuuint64_t)(lay.head * es), (cuuint64_t)(lay.pos * es), (cuuint64_t)(lay.lo * es),
                             (cuuint64_t)((lay.n_hi > 1 ? lay.hi : lay.lo * lay.n_lo) * es)};  // unused if n_hi == 1
    for (int i = 0; i < 4; ++i)
        MBR_CHECK(strides[i] % 16 == 0 && strides[i] < (1ull << 40), "attention TMA strides must be 16-byte multiples");
    cuuint32_t box[5] = {(cuuint32_t)DH, 1, (cuuint32_t)box_pos, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = encode_fn()(m, dtype == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             5, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

template <typename T, bool PACK>
void launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, int nsh, int H, int L, int n_lo,
            float scale_log2, const float* gates, int mode, int NB, int Tn, void* merged, int* err, cudaStream_t st) {
    auto kern = attn_tc_kernel<T, PACK>;
    using AttnSmem = AttnCfg<PACK>;
    static bool attr[64] = {};
    static int sms[64] = {};
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < 64, "device index out of range");
    if (!attr[dev]) {
        MBR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmem::TOTAL));
        MBR_CUDA(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
        attr[dev] = true;
    }
    // persistent: two CTAs per SM walk the tiles
    const int64_t ntiles = PACK ? ((int64_t)nsh + 1) / 2 : (int64_t)nsh * ((L + QT - 1) / QT);
    MBR_CHECK(ntiles < (1ll << 30), "tc attention: too many tiles");
    const int grid = (int)std::min<int64_t>(ntiles, 2 * (int64_t)sms[dev]);
    if (grid == 0) return;
    kern<<<grid, 192, AttnSmem::TOTAL, st>>>(mq, mk, mv, nsh, H, L, n_lo, scale_log2, gates, mode, NB, Tn,
                                              (T*)merged, err);
    MBR_CUDA(cudaGetLastError());
}

}  // namespace

bool attention_supported(int dim_head) { return dim_head == DH; }

AttnLayout head_major_layout(int64_t nseq, int H, int L, int dh) {
    AttnLayout lay;
    lay.head = (int64_t)L * dh;
    lay.pos = dh;
    lay.lo = (int64_t)H * L * dh;
    lay.hi = 0;
    lay.n_lo = (int)nseq;
    lay.n_hi = 1;
    return lay;
}

void attention(const void* q, const void* k, const void* v, const AttnLayout& lay, int64_t nseq, int H, int L,
               int dh, float scale, const float* gates, int mode, int NB, int T, void* merged, int dtype, int* d_err,
               cudaStream_t st) {
    MBR_CHECK(dh == DH, "tc attention: dim_head must be 64");
    MBR_CHECK(dtype == DT_F16 || dtype == DT_BF16, "tc attention: fp16 or bf16 only");
    const int64_t nsh = nseq * H;
    MBR_CHECK(nsh < (1 << 30) && L > 0 && lay.n_lo > 0 && lay.n_hi > 0 && (int64_t)lay.n_lo * lay.n_hi == nseq,
              "tc attention: bad problem or layout");
    const bool pack = L <= 64;
    CUtensorMap mq, mk, mv;
    make_map(&mq, q, lay, H, L, pack ? 64 : QT, dtype);
    make_map(&mk, k, lay, H, L, KB, dtype);
    make_map(&mv, v, lay, H, L, KB, dtype);
    const float scale_log2 = scale * 1.4426950408889634f;
    const int n = (int)nsh;
    if (dtype == DT_BF16) {
        if (pack) launch<__nv_bfloat16, true>(mq, mk, mv, n, H, L, lay.n_lo, scale_log2, gates, mode, NB, T, merged, d_err, st);
        else launch<__nv_bfloat16, false>(mq, mk, mv, n, H, L, lay.n_lo, scale_log2, gates, mode, NB, T, merged, d_err, st);
    } else {
        if (pack) launch<__half, true>(mq, mk, mv, n, H, L, lay.n_lo, scale_log2, gates, mode, NB, T, merged, d_err, st);
        else launch<__half, false>(mq, mk, mv, n, H, L, lay.n_lo, scale_log2, gates, mode, NB, T, merged, d_err, st);
    }
}

}  // namespace tc
}  // namespace mbr
