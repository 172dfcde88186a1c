// MLX affine format on the GPU: quantize (mx.quantize) and dequantize (mx.dequantize).
//
// quantize: one thread per group of 64 values. Per group (the affine algorithm of MLX 0.32.3, which
// the reference calls in its tests, e.g. tests/test_kernel_patching.py:163): scale = (max - min) /
// (2^bits - 1) (at least 1e-7), negated unless |min| > |max|, the larger-magnitude edge made exact
// (q0 = rint(edge / scale); if q0 != 0: scale = edge / q0, bias = edge; else bias = 0), codes =
// clip(rint((w - bias) / scale), 0, 2^bits - 1) from the float32 scale and bias, which are then
// rounded to the scales' dtype. Codes packed low bits first (locals/kernels.py:31-35,63-64).
//
// dequantize: one thread per packed word; w = scale * q + bias in float32, rounded to the dtype.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lq_host.h"

namespace lq {

__device__ __forceinline__ float load_any(const void* p, size_t i, int dt) {
    if (dt == LQ_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == LQ_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void store_any(void* p, size_t i, float v, int dt) {
    if (dt == LQ_F32)
        reinterpret_cast<float*>(p)[i] = v;
    else if (dt == LQ_BF16)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

__global__ void quantize_kernel(const void* w, int w_dt, int64_t n_groups, int K, int bits, int group,
                                uint32_t* wq, void* scales, void* biases, int sb_dt) {
    const int64_t gi = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gi >= n_groups) return;
    const int ng_row = K / group;
    const int64_t row = gi / ng_row, gcol = gi % ng_row;
    const size_t base = size_t(row) * K + size_t(gcol) * group;
    float w_min = INFINITY, w_max = -INFINITY;
    for (int j = 0; j < group; ++j) {
        const float v = load_any(w, base + j, w_dt);
        w_max = fmaxf(w_max, v);
        w_min = fminf(w_min, v);
    }
    const float n_bins = float((1 << bits) - 1);
    const bool mask = fabsf(w_min) > fabsf(w_max);
    float scale = fmaxf(__fdiv_rn(w_max - w_min, n_bins), 1e-7f);
    scale = mask ? scale : -scale;
    const float edge = mask ? w_min : w_max;
    const float q0 = rintf(__fdiv_rn(edge, scale));
    float bias = 0.0f;
    if (q0 != 0.0f) {
        scale = __fdiv_rn(edge, q0);
        bias = edge;
    }
    const int per_word = 32 / bits;
    const size_t words_row = size_t(K) / per_word;
    for (int j0 = 0; j0 < group; j0 += per_word) {
        uint32_t word = 0;
        for (int k = 0; k < per_word; ++k) {
            float q = rintf(__fdiv_rn(load_any(w, base + j0 + k, w_dt) - bias, scale));
            q = fminf(fmaxf(q, 0.0f), n_bins);
            word |= uint32_t(q) << (k * bits);
        }
        wq[size_t(row) * words_row + (size_t(gcol) * group + j0) / per_word] = word;
    }
    store_any(scales, size_t(gi), scale, sb_dt);
    store_any(biases, size_t(gi), bias, sb_dt);
}

__global__ void dequantize_kernel(const uint32_t* wq, const void* s, const void* b, int64_t n_words, int K,
                                  int bits, int group, int dt, void* out) {
    const int64_t wi = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (wi >= n_words) return;
    const int per_word = 32 / bits;
    const int64_t words_row = K / per_word;
    const int64_t row = wi / words_row, kw = wi % words_row;
    const int64_t k0 = kw * per_word;
    const size_t gidx = size_t(row) * (K / group) + size_t(k0 / group);
    const float sc = load_any(s, gidx, dt), bi = load_any(b, gidx, dt);
    const uint32_t word = wq[wi];
    const uint32_t mask = (1u << bits) - 1u;
    for (int k = 0; k < per_word; ++k)
        store_any(out, size_t(row) * K + k0 + k, fmaf(sc, float((word >> (k * bits)) & mask), bi), dt);
}

int quantize_run(const void* w, int w_dt, int N, int K, int bits, int group, uint32_t* wq, void* s, void* b,
                 int sb_dt, cudaStream_t st) {
    const int64_t n_groups = int64_t(N) * (K / group);
    const int threads = 128;
    const int64_t blocks = (n_groups + threads - 1) / threads;
    quantize_kernel<<<unsigned(blocks), threads, 0, st>>>(w, w_dt, n_groups, K, bits, group, wq, s, b, sb_dt);
    return cuda_status(cudaGetLastError());
}

int dequantize_run(const uint32_t* wq, const void* s, const void* b, int N, int K, int bits, int group, int dt,
                   void* out, cudaStream_t st) {
    const int64_t n_words = int64_t(N) * K / (32 / bits);
    const int threads = 256;
    const int64_t blocks = (n_words + threads - 1) / threads;
    dequantize_kernel<<<unsigned(blocks), threads, 0, st>>>(wq, s, b, n_words, K, bits, group, dt, out);
    return cuda_status(cudaGetLastError());
}

}  // namespace lq
