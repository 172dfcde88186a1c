// Routed mixture-of-experts helpers: router logits, top-k routing, the expert grouping (counting
// sort + pair-order gather) and the weighted combine. The expert projections themselves run on the
// qmv kernel family in grouped mode (qmv.cu).
//
//  router_logits : float32 logits = float(x) . float(w)^T, one warp per (token, expert), 16-byte loads
//                  (locals/moe.py:86-139: "exactly as x.astype(f32) @ W.astype(f32).T").
//  route_topk    : one warp per token; softmax (or sigmoid, locals/moe.py:36-82) over E experts held
//                  E/32 per lane, k rounds of a warp argmax with ties to the lower index, renormalise.
//  group         : one CTA; per-expert counts in shared memory, segments of used experts in ascending
//                  expert order, a stable order (pair ids ascending within an expert) and its inverse
//                  (locals/moe_kernel.py:28-66 with a deterministic order).
//  gather_rows   : xs[j] = x[order[j] / k], the tokens laid out in pair order for the grouped kernel.
//  combine       : y[t] = sum_r w[t, r] * ys[pos[t*k + r]] in float32, slots in order (locals/moe.py:339-348).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lq_host.h"
#include "lq_status.cuh"

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

// grid: T * ceil(E / 4) blocks of 128 threads (4 warps = 4 experts of one token)
__global__ void router_logits_kernel(const void* x, int x_dt, const void* w, int w_dt, float* logits, int T, int E,
                                     int D) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int eb = (E + 3) / 4;
    const int t = blockIdx.x / eb;
    const int e = (blockIdx.x % eb) * 4 + warp;
    if (t >= T || e >= E) return;
    const uint4* xr = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + size_t(t) * D);
    const uint4* wr = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w) + size_t(e) * D);
    float acc = 0.0f;
    for (int i = lane; i < D / 8; i += 32) {
        float xf[8], wf[8];
        unpack8(xr[i], x_dt, xf);
        unpack8(wr[i], w_dt, wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(xf[j], wf[j], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) logits[size_t(t) * E + e] = acc;
}

constexpr int TOPK_MAX_PER_LANE = 32;  // E <= 1024

// one warp per token; 4 tokens per block
__global__ void route_topk_kernel(const float* logits, int T, int E, int k, int mode, uint32_t* inds,
                                  float* weights) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 4 + warp;
    if (t >= T) return;
    const float* l = logits + size_t(t) * E;
    const int per = (E + 31) / 32;
    float sc[TOPK_MAX_PER_LANE];
    if (mode == 0) {
        float mx = -INFINITY;
        for (int j = 0; j < per; ++j) {
            const int e = lane + 32 * j;
            sc[j] = e < E ? l[e] : -INFINITY;
            mx = fmaxf(mx, sc[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float tot = 0.0f;
        for (int j = 0; j < per; ++j) {
            const int e = lane + 32 * j;
            sc[j] = e < E ? expf(sc[j] - mx) : 0.0f;
            tot += sc[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
        for (int j = 0; j < per; ++j) {
            const int e = lane + 32 * j;
            sc[j] = e < E ? sc[j] / tot : -1.0f;
        }
    } else {
        for (int j = 0; j < per; ++j) {
            const int e = lane + 32 * j;
            const float v = e < E ? 1.0f / (1.0f + expf(-l[e])) : -1.0f;
            sc[j] = e < E ? (isnan(v) ? 0.0f : v) : -1.0f;
        }
    }
    // NaN scores (softmax of NaN logits) rank below every number; the result still names k distinct experts
    for (int j = 0; j < per; ++j)
        if (isnan(sc[j])) sc[j] = -2.0f;
    float picked_sum = 0.0f;
    float picked[32];
    uint32_t which[32];
    for (int r = 0; r < k; ++r) {
        float best = -3.0f;
        int best_e = E;
        for (int j = 0; j < per; ++j) {
            const int e = lane + 32 * j;
            if (e < E && sc[j] > best) {  // strict: the lower index of this lane wins ties
                best = sc[j];
                best_e = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
            if (ob > best || (ob == best && oe < best_e)) {
                best = ob;
                best_e = oe;
            }
        }
        if (best_e < E && (best_e & 31) == lane) sc[best_e >> 5] = -3.0f;
        picked[r] = best < -1.5f ? 0.0f : best;
        which[r] = uint32_t(best_e < E ? best_e : E - 1);
        picked_sum += picked[r];
    }
    if (lane == 0) {
        for (int r = 0; r < k; ++r) {
            inds[size_t(t) * k + r] = which[r];
            weights[size_t(t) * k + r] = picked[r] / picked_sum;
        }
    }
}

// One CTA of 1024 threads. order/starts/experts/nseg as lq_moe_group; pos = inverse of order (optional).
__global__ void group_kernel(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts,
                             int32_t* nseg, int32_t* pos) {
    extern __shared__ int32_t sh[];
    int32_t* cnt = sh;       // E
    int32_t* base = sh + E;  // E
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const uint32_t e = inds[p];
        if (e < uint32_t(E))
            atomicAdd(&cnt[e], 1);
        else
            record_status(LQ_DEV_BOUNDS);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int at = 0, s = 0;
        for (int e = 0; e < E; ++e) {
            base[e] = at;
            if (cnt[e] > 0) {
                starts[s] = at;
                experts[s] = e;
                ++s;
            }
            at += cnt[e];
        }
        starts[s] = at;
        nseg[0] = s;
    }
    __syncthreads();
    // stable placement: rank of p among the pairs of its expert = pairs q < p with the same expert
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const uint32_t e = inds[p];
        if (e >= uint32_t(E)) continue;
        int rank = 0;
        for (int q = 0; q < p; ++q) rank += (inds[q] == e) ? 1 : 0;
        const int j = base[e] + rank;
        order[j] = p;
        if (pos) pos[p] = j;
    }
}

// xs[j] = x[order[j] / k]: one warp per row, 16-byte copies
__global__ void gather_rows_kernel(const uint16_t* x, const int32_t* order, int P, int k, int D, uint16_t* xs) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= P) return;
    const int tok = order[warp] / k;
    const uint4* src = reinterpret_cast<const uint4*>(x + size_t(tok) * D);
    uint4* dst = reinterpret_cast<uint4*>(xs + size_t(warp) * D);
    for (int i = lane; i < D / 8; i += 32) dst[i] = src[i];
}

// y[t, d] = sum_r w[t, r] * ys[row(t, r), d]; row = pos[t*k + r] if pos, else t*k + r
__global__ void combine_kernel(const uint16_t* ys, const float* w, const int32_t* pos, uint16_t* y, int T, int k, int D,
                               int dt) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(T) * D) return;
    const int t = int(i / D), d = int(i % D);
    float acc = 0.0f;
    for (int r = 0; r < k; ++r) {
        const int slot = t * k + r;
        const int row = pos ? pos[slot] : slot;
        const uint16_t h = ys[size_t(row) * D + d];
        float v;
        if (dt == LQ_BF16) {
            v = __uint_as_float(uint32_t(h) << 16);
        } else {
            v = __half2float(*reinterpret_cast<const __half*>(&h));
        }
        acc = fmaf(v, w[slot], acc);
    }
    if (dt == LQ_BF16) {
        __nv_bfloat16 b = __float2bfloat16_rn(acc);
        y[i] = *reinterpret_cast<uint16_t*>(&b);
    } else {
        __half hh = __float2half_rn(acc);
        y[i] = *reinterpret_cast<uint16_t*>(&hh);
    }
}

int router_logits_run(const void* x, int x_dt, const void* w, int w_dt, float* logits, int T, int E, int D,
                      cudaStream_t st) {
    const int blocks = T * ((E + 3) / 4);
    router_logits_kernel<<<blocks, 128, 0, st>>>(x, x_dt, w, w_dt, logits, T, E, D);
    return cuda_status(cudaGetLastError());
}

int route_topk_run(const float* logits, int T, int E, int k, int mode, uint32_t* inds, float* weights,
                   cudaStream_t st) {
    route_topk_kernel<<<(T + 3) / 4, 128, 0, st>>>(logits, T, E, k, mode, inds, weights);
    return cuda_status(cudaGetLastError());
}

int group_run(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts, int32_t* nseg,
              int32_t* pos, cudaStream_t st) {
    group_kernel<<<1, 1024, size_t(2) * E * sizeof(int32_t), st>>>(inds, P, E, order, starts, experts, nseg, pos);
    return cuda_status(cudaGetLastError());
}

int gather_rows_run(const void* x, const int32_t* order, int P, int k, int D, void* xs, cudaStream_t st) {
    const int threads = 256;
    const int blocks = (P * 32 + threads - 1) / threads;
    gather_rows_kernel<<<blocks, threads, 0, st>>>(reinterpret_cast<const uint16_t*>(x), order, P, k, D,
                                                   reinterpret_cast<uint16_t*>(xs));
    return cuda_status(cudaGetLastError());
}

int combine_run(const void* ys, const float* w, const int32_t* pos, void* y, int T, int k, int D, int dt,
                cudaStream_t st) {
    const size_t n = size_t(T) * D;
    const int threads = 256;
    combine_kernel<<<unsigned((n + threads - 1) / threads), threads, 0, st>>>(
        reinterpret_cast<const uint16_t*>(ys), w, pos, reinterpret_cast<uint16_t*>(y), T, k, D, dt);
    return cuda_status(cudaGetLastError());
}

}  // namespace lq
