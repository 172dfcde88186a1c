// Routing pieces shared by the stand-alone routing kernels (moe.cu) and the fused one-token MoE layer
// (moe_decode.cu): the float32 router dot product of one (token, expert) on one warp, the softmax / sigmoid scores
// and the k-round warp argmax. Both files compile these same functions, so the fused layer picks bit-identical
// logits, experts and weights to lq_moe_route.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/lq.h"

namespace lq {

__device__ __forceinline__ void unpack8(uint4 u, int dt, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (dt == LQ_BF16) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        } else {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            const float2 v = __half22float2(h);
            f[2 * i] = v.x;
            f[2 * i + 1] = v.y;
        }
    }
}


// float(x_row) . float(w_row) over D values (D % 8 == 0, 16-byte aligned rows) on one warp: lane l sums the 16-byte
// pieces l, l + 32, ... in order with fmaf, then a butterfly of shuffles adds the lanes (every lane gets the sum).
// The one summation order of every router logit in the library (locals/moe.py:134-139 computes the same float32
// product).
__device__ __forceinline__ float router_dot(const uint16_t* xrow, int x_dt, const uint16_t* wrow, int w_dt, int D,
                                            int lane) {
    const uint4* xr = reinterpret_cast<const uint4*>(xrow);
    const uint4* wr = reinterpret_cast<const uint4*>(wrow);
    float acc = 0.0f;
#pragma unroll 4
    for (int i = lane; i < D / 8; i += 32) {
        float xf[8], wf[8];
        unpack8(xr[i], x_dt, xf);
        unpack8(wr[i], w_dt, wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(xf[j], wf[j], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

constexpr int TOPK_MAX_PER_LANE = 32;  // E <= 1024

// An order-preserving 32-bit key of a float that is not NaN (x < y <=> key(x) < key(y); -0.0 never occurs here).
__device__ __forceinline__ uint32_t topk_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float topk_unkey(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// k rounds of a warp argmax over E scores held PER per lane (expert lane + 32 j, j < per), ties to the lower index,
// then renormalisation; lane r < k writes index and weight r. NaN scores rank below every number (-2), an expert
// already taken at -3. Each round is one warp max (redux.sync) of the scores' order-preserving keys and one warp min
// of the indices holding it; the register arrays are indexed by compile-time j only.
template <int PER>
__device__ __forceinline__ void topk_select(const float (&sc)[PER], int per, int E, int k, int lane, uint32_t* inds,
                                            float* weights) {
    const uint32_t taken = topk_key(-3.0f);
    uint32_t key[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int e = lane + 32 * j;
        key[j] = (j < per && e < E) ? topk_key(isnan(sc[j]) ? -2.0f : sc[j]) : 0u;  // 0: below every score
    }
    float picked_sum = 0.0f, my_pick = 0.0f;
    uint32_t my_which = 0;
    for (int r = 0; r < k; ++r) {
        uint32_t best = taken;  // strict: a taken expert never wins, the lower index of this lane wins ties
        uint32_t best_e = uint32_t(E);
#pragma unroll
        for (int j = 0; j < PER; ++j)
            if (key[j] > best) {
                best = key[j];
                best_e = uint32_t(lane + 32 * j);
            }
        const uint32_t m = __reduce_max_sync(0xffffffffu, best);
        const uint32_t win = __reduce_min_sync(0xffffffffu, best == m ? best_e : 0xffffffffu);
#pragma unroll
        for (int j = 0; j < PER; ++j)
            if (uint32_t(lane + 32 * j) == win) key[j] = taken;
        const float v = topk_unkey(m);
        const float pick = v < -1.5f ? 0.0f : v;
        if (lane == r) {
            my_pick = pick;
            my_which = win < uint32_t(E) ? win : uint32_t(E - 1);
        }
        picked_sum += pick;
    }
    if (lane < k) {
        inds[lane] = my_which;
        weights[lane] = my_pick / picked_sum;
    }
}

// softmax (mode 0) or sigmoid (mode 1, NaN -> 0) of the E logits fetched by get(e), then the top k
template <int PER, typename Get>
__device__ __forceinline__ void score_and_select_t(Get get, int E, int k, int mode, int lane, uint32_t* inds,
                                                   float* weights) {
    const int per = (E + 31) / 32;
    float sc[PER];
    if (mode == 0) {
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int e = lane + 32 * j;
            sc[j] = (j < per && e < E) ? get(e) : -INFINITY;
            mx = fmaxf(mx, sc[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float tot = 0.0f;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int e = lane + 32 * j;
            sc[j] = (j < per && e < E) ? expf(sc[j] - mx) : 0.0f;
            tot += sc[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int e = lane + 32 * j;
            sc[j] = (j < per && e < E) ? sc[j] / tot : -1.0f;
        }
    } else {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int e = lane + 32 * j;
            const float v = (j < per && e < E) ? 1.0f / (1.0f + expf(-get(e))) : -1.0f;
            sc[j] = (j < per && e < E) ? (isnan(v) ? 0.0f : v) : -1.0f;
        }
    }
    topk_select<PER>(sc, per, E, k, lane, inds, weights);
}

// score_and_select_t with the per-lane count as a compile-time bound (E <= 1024)
template <typename Get>
__device__ __forceinline__ void score_and_select(Get get, int E, int k, int mode, int lane, uint32_t* inds,
                                                 float* weights) {
    const int per = (E + 31) / 32;
    if (per <= 1)
        score_and_select_t<1>(get, E, k, mode, lane, inds, weights);
    else if (per <= 2)
        score_and_select_t<2>(get, E, k, mode, lane, inds, weights);
    else if (per <= 4)
        score_and_select_t<4>(get, E, k, mode, lane, inds, weights);
    else if (per <= 8)
        score_and_select_t<8>(get, E, k, mode, lane, inds, weights);
    else if (per <= 16)
        score_and_select_t<16>(get, E, k, mode, lane, inds, weights);
    else
        score_and_select_t<TOPK_MAX_PER_LANE>(get, E, k, mode, lane, inds, weights);
}

}  // namespace lq
