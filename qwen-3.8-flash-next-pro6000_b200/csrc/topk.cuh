// Softmax + top-k + renormalise of one router row by one warp: shared by the router kernel and the MoE kernel's
// fused-router mode, so that both select and weight experts with the same arithmetic.
//   p[e]   = softmax_e(logits)             fp32, max-subtracted
//   ids    = the k largest logits, lower expert id first among equal values (NaN ranks as -1e30, -0 as +0)
//   w      = p[ids] / sum(p[ids]) when renormalising (sum > 0), else p[ids]
// Selection semantics follow serve/qwenfast/qf_router.cu:3-6, 103-157. The logits are bf16 values (held as bf16,
// or as their exact fp32 copies).
#pragma once
#include "qf_common.cuh"

namespace qf {

__device__ __forceinline__ float load_logit(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float load_logit(const __nv_bfloat16* p) {
    return __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(p)) << 16);
}

// Ranking of one logit, larger is better: bits 10..26 the order-preserving key of the value (top 17 bits of the
// monotone uint32 image of the float; NaN ranks as -1e30, -0 as +0), bits 0..9 1023 - expert id, so that among
// equal values the lower id wins and one unsigned max picks the winner. The logits are bf16 values (fp32 copies), so
// 17 bits order them exactly: a bf16 value's image has its low 16 bits all equal, and the image of -1e30 (not a
// bf16 value) falls strictly between those of its two bf16 neighbours. 0 means "no candidate".
constexpr float RANK_NAN_AS = -1e30f;
__device__ __forceinline__ uint32_t image17(float v) {
    const float r = (v == v) ? v : RANK_NAN_AS;
    uint32_t u = __float_as_uint(r);
    if (u == 0x80000000u) u = 0u;
    return ((u & 0x80000000u) ? ~u : (u | 0x80000000u)) >> 15;
}
__device__ __forceinline__ uint32_t rank_of(float v, int e) { return (image17(v) << 10) | (uint32_t)(1023 - e); }
// the logit a rank was made from (NaN for the NaN stand-in)
__device__ __forceinline__ float logit_of(uint32_t rank) {
    const uint32_t k17 = rank >> 10;
    if (k17 == image17(RANK_NAN_AS)) return __uint_as_float(0x7fc00000u);
    const uint32_t img = (k17 << 15) | ((k17 & 1u) ? 0x7fffu : 0u);
    return __uint_as_float((img & 0x80000000u) ? (img & 0x7fffffffu) : ~img);
}

// softmax + top-k of one token row (E logits, fp32 copies of the bf16 values) by one warp. Each round takes the
// warp-wide largest rank (a lane-local max tree, then one redux) and clears it; lane k keeps round k's winner. The
// probabilities are formed afterwards, all lanes at once: p_k = exp(logit_k - max) / sum, the same operands as a
// softmax over the row, and the renormalising sum runs over p_0, p_1, ... in selection order.
// Element i of a lane is expert lane * PL + i when FULL (a row of exactly 32 * PL experts, PL a multiple of 8), else
// expert i * 32 + lane (elements past E hold -inf). The ranking carries the id, so the selection does not depend on
// which lane holds which expert; FULL fixes the softmax summation order, shared by every caller that loads a full row.
template <int PL, bool FULL>
__device__ __forceinline__ void topk_select(const float (&v)[PL], int E, int topk, int renorm, float* __restrict__ wout,
                                            int* __restrict__ iout) {
    const int lane = threadIdx.x & 31;
    uint32_t rk[PL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PL; ++i) mx = fmaxf(mx, v[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        if constexpr (FULL) {
            rk[i] = rank_of(v[i], lane * PL + i);
        } else {
            const int e = i * 32 + lane;
            rk[i] = e < E ? rank_of(v[i], e) : 0u;
        }
        sum += __expf(v[i] - mx);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);

    uint32_t mine = 0u;
    for (int k = 0; k < topk; ++k) {
        uint32_t t[PL];
#pragma unroll
        for (int i = 0; i < PL; ++i) t[i] = rk[i];
#pragma unroll
        for (int w = 1; w < PL; w <<= 1) {
#pragma unroll
            for (int i = 0; i + w < PL; i += 2 * w) t[i] = max(t[i], t[i + w]);
        }
        const uint32_t win = __reduce_max_sync(0xffffffffu, t[0]);
#pragma unroll
        for (int i = 0; i < PL; ++i) rk[i] = rk[i] == win ? 0u : rk[i];
        mine = lane == k ? win : mine;
    }
    float p = 0.f;
    int id = -1;
    if (lane < topk && mine != 0u) {
        id = 1023 - (int)(mine & 1023u);
        p = __expf(logit_of(mine) - mx) / sum;
    }
    float routed = 0.f;
    for (int k = 0; k < topk; ++k) routed += __shfl_sync(0xffffffffu, p, k);
    if (lane < topk) {
        const float norm = routed > 0.f ? routed : 1.f;
        wout[lane] = renorm ? p / norm : p;
        iout[lane] = id;
    }
}

// one warp: the top-k of one row in memory (fp32 or bf16 logits)
template <int PL, typename T>
__device__ void topk_row(const T* __restrict__ row, int E, int topk, int renorm, float* __restrict__ wout,
                         int* __restrict__ iout) {
    const int lane = threadIdx.x & 31;
    float v[PL];
    constexpr int PER16 = 16 / (int)sizeof(T);
    if constexpr (PL % 8 == 0) {
        if (E == 32 * PL && (reinterpret_cast<uintptr_t>(row) & 15u) == 0u) {
            // a full row: 16-byte words, lane l holding experts l * PL .. l * PL + PL - 1
#pragma unroll
            for (int c = 0; c < PL / PER16; ++c) {
                const uint4 w = __ldcg(reinterpret_cast<const uint4*>(row + lane * PL) + c);
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if constexpr (sizeof(T) == 2) {
                        v[PER16 * c + 2 * j] = __uint_as_float(ww[j] << 16);
                        v[PER16 * c + 2 * j + 1] = __uint_as_float(ww[j] & 0xFFFF0000u);
                    } else {
                        v[PER16 * c + j] = __uint_as_float(ww[j]);
                    }
                }
            }
            topk_select<PL, true>(v, 32 * PL, topk, renorm, wout, iout);
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        const int e = i * 32 + lane;
        v[i] = e < E ? load_logit(row + e) : -INFINITY;
    }
    topk_select<PL, false>(v, E, topk, renorm, wout, iout);
}

// one warp: the row's top-k into wout[0..topk) / iout[0..topk) (lanes 0..topk-1 write); E <= 1024
template <typename T>
__device__ __forceinline__ void topk_row_any(const T* __restrict__ row, int E, int topk, int renorm,
                                             float* __restrict__ wout, int* __restrict__ iout) {
    const int pl = (E + 31) / 32;
    if (pl <= 1) topk_row<1>(row, E, topk, renorm, wout, iout);
    else if (pl <= 2) topk_row<2>(row, E, topk, renorm, wout, iout);
    else if (pl <= 4) topk_row<4>(row, E, topk, renorm, wout, iout);
    else if (pl <= 8) topk_row<8>(row, E, topk, renorm, wout, iout);
    else if (pl <= 16) topk_row<16>(row, E, topk, renorm, wout, iout);
    else topk_row<32>(row, E, topk, renorm, wout, iout);
}

}  // namespace qf
