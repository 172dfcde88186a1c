// The steps either side of the quantized projections in a decoder layer:
//   * add_rms: the residual add and the following RMS norm in one pass (locals/norm_kernel.py:16-85):
//       h = T(x + r), n = T(w * T(h * rsqrt(mean(h^2) + eps)))   (sum of squares in fp32);
//   * combine_norm: the MoE combine, the shared expert's output, the layer's residual add and the next
//     layer's input norm (locals/moe.py:353-389):
//       y = T(sum_k weights[t,k] * ys[slot(t,k)]) (fp32, slots in order), y = T(y + shared), h = T(res + y),
//       n as above;
//   * scatter_rows: the scatter half of row packing (locals/kernels.py:840-851): dst row idx[j] = src row j,
//     every other row of dst zero.
// One CTA per row (token); each thread moves 8 consecutive 16-bit values per step, so a row of D values is
// read once with 16-byte loads. HBM-bound: 5 * 2 * D bytes per row for add_rms.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"
#include "lq_status.cuh"

namespace lq {

constexpr int NORM_THREADS = 256;
constexpr int NORM_MAX_VEC = 4;  // 8-value vectors per thread held in registers (D <= 8192)

template <typename T>
__device__ __forceinline__ float nt_f(T v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __bfloat162float(v);
    else
        return __half2float(v);
}
template <typename T>
__device__ __forceinline__ T nt_t(float v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __float2bfloat16_rn(v);
    else
        return __float2half_rn(v);
}

union Vec8 {
    uint4 u;
    uint16_t h[8];
};

template <typename T>
__device__ __forceinline__ T vget(const Vec8& v, int i) {
    T t;
    *reinterpret_cast<uint16_t*>(&t) = v.h[i];
    return t;
}
template <typename T>
__device__ __forceinline__ void vset(Vec8& v, int i, T t) {
    v.h[i] = *reinterpret_cast<uint16_t*>(&t);
}

// Sum over the CTA; every thread gets the total.
__device__ __forceinline__ float norm_block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < NORM_THREADS / 32 ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
    return t;
}

// n = T(w * T(h * inv)) for the thread's held vectors, written to n_row.
template <typename T>
__device__ __forceinline__ void norm_write(const Vec8 (&hv)[NORM_MAX_VEC], int nvec, int D, float inv, const T* w,
                                           T* n_row) {
#pragma unroll
    for (int j = 0; j < NORM_MAX_VEC; ++j) {
        if (j >= nvec) break;
        const int c = (threadIdx.x + j * NORM_THREADS) * 8;
        if (c >= D) break;
        Vec8 wv, nv;
        wv.u = *reinterpret_cast<const uint4*>(w + c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float hn = nt_f(nt_t<T>(nt_f(vget<T>(hv[j], i)) * inv));
            vset(nv, i, nt_t<T>(nt_f(vget<T>(wv, i)) * hn));
        }
        *reinterpret_cast<uint4*>(n_row + c) = nv.u;
    }
}

template <typename T>
__global__ void __launch_bounds__(NORM_THREADS) add_rms_kernel(const T* x, const T* r, const T* w, T* h, T* n, int D,
                                                                float eps) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float red[NORM_THREADS / 32];
    const size_t row = blockIdx.x;
    const int nvec = (D / 8 + NORM_THREADS - 1) / NORM_THREADS;
    Vec8 hv[NORM_MAX_VEC];
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < NORM_MAX_VEC; ++j) {
        if (j >= nvec) break;
        const int c = (threadIdx.x + j * NORM_THREADS) * 8;
        if (c >= D) break;
        Vec8 xv, rv;
        xv.u = *reinterpret_cast<const uint4*>(x + row * D + c);
        rv.u = *reinterpret_cast<const uint4*>(r + row * D + c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const T s = nt_t<T>(nt_f(vget<T>(xv, i)) + nt_f(vget<T>(rv, i)));  // the 16-bit add, rounded once
            vset(hv[j], i, s);
            const float f = nt_f(s);
            sq += f * f;
        }
        *reinterpret_cast<uint4*>(h + row * D + c) = hv[j].u;
    }
    const float total = norm_block_sum(sq, red);
    const float inv = 1.0f / sqrtf(total / float(D) + eps);
    norm_write<T>(hv, nvec, D, inv, w, n + row * D);
}

template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    combine_norm_kernel(const T* ys, const float* wts, const int32_t* pos, const T* shared, const T* res, const T* nw,
                        T* y, T* n, int K, int D, float eps) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float red[NORM_THREADS / 32];
    const size_t t = blockIdx.x;
    const int nvec = (D / 8 + NORM_THREADS - 1) / NORM_THREADS;
    Vec8 hv[NORM_MAX_VEC];
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < NORM_MAX_VEC; ++j) {
        if (j >= nvec) break;
        const int c = (threadIdx.x + j * NORM_THREADS) * 8;
        if (c >= D) break;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        for (int k = 0; k < K; ++k) {
            const int slot = pos ? pos[t * K + k] : int(t * K + k);
            const float wk = wts[t * K + k];
            Vec8 yv;
            yv.u = *reinterpret_cast<const uint4*>(ys + size_t(slot) * D + c);
#pragma unroll
            for (int i = 0; i < 8; ++i)  // product and sum rounded separately (no fused multiply-add), as the C restatement
                acc[i] = __fadd_rn(acc[i], __fmul_rn(nt_f(vget<T>(yv, i)), wk));
        }
        Vec8 sv, rv;
        if (shared) sv.u = *reinterpret_cast<const uint4*>(shared + t * D + c);
        rv.u = *reinterpret_cast<const uint4*>(res + t * D + c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            T v = nt_t<T>(acc[i]);
            if (shared) v = nt_t<T>(nt_f(v) + nt_f(vget<T>(sv, i)));
            v = nt_t<T>(nt_f(vget<T>(rv, i)) + nt_f(v));  // the layer's residual add, as h + mlp(...)
            vset(hv[j], i, v);
            const float f = nt_f(v);
            sq += f * f;
        }
        *reinterpret_cast<uint4*>(y + t * D + c) = hv[j].u;
    }
    const float total = norm_block_sum(sq, red);
    const float inv = 1.0f / sqrtf(total / float(D) + eps);
    norm_write<T>(hv, nvec, D, inv, nw, n + t * D);
}

// dst row idx[j] = src row j (16-byte chunks); dst was zeroed before.
__global__ void scatter_rows_kernel(const uint4* src, const int32_t* idx, int R, int chunks, uint4* dst, int dst_rows) {
    grid_dep_wait();
    grid_dep_launch();
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(R) * chunks) return;
    const int j = int(i / chunks), c = int(i % chunks);
    const int d = idx[j];
    if (d < 0 || d >= dst_rows) {
        record_status(LQ_DEV_BOUNDS);
        return;
    }
    dst[size_t(d) * chunks + c] = src[i];
}

template <typename K, typename... Args>
static int norm_launch(K kern, dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

bool norm_shape_ok(int D) { return D >= 8 && D % 8 == 0 && D <= 8 * NORM_THREADS * NORM_MAX_VEC; }

int add_rms_run(const void* x, const void* r, const void* w, void* h, void* n, int rows, int D, float eps, int dtype,
                cudaStream_t st) {
    if (dtype == LQ_BF16)
        return norm_launch(add_rms_kernel<__nv_bfloat16>, dim3(rows), dim3(NORM_THREADS), st,
                           static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(r),
                           static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(h),
                           static_cast<__nv_bfloat16*>(n), D, eps);
    return norm_launch(add_rms_kernel<__half>, dim3(rows), dim3(NORM_THREADS), st, static_cast<const __half*>(x),
                       static_cast<const __half*>(r), static_cast<const __half*>(w), static_cast<__half*>(h),
                       static_cast<__half*>(n), D, eps);
}

int combine_norm_run(const void* ys, const float* wts, const int32_t* pos, const void* shared, const void* res,
                     const void* nw, void* y, void* n, int T, int K, int D, float eps, int dtype, cudaStream_t st) {
    if (dtype == LQ_BF16) {
        using B = __nv_bfloat16;
        return norm_launch(combine_norm_kernel<B>, dim3(T), dim3(NORM_THREADS), st, static_cast<const B*>(ys), wts, pos,
                           static_cast<const B*>(shared), static_cast<const B*>(res), static_cast<const B*>(nw),
                           static_cast<B*>(y), static_cast<B*>(n), K, D, eps);
    }
    return norm_launch(combine_norm_kernel<__half>, dim3(T), dim3(NORM_THREADS), st, static_cast<const __half*>(ys), wts,
                       pos, static_cast<const __half*>(shared), static_cast<const __half*>(res),
                       static_cast<const __half*>(nw), static_cast<__half*>(y), static_cast<__half*>(n), K, D, eps);
}

int scatter_rows_run(const void* src, const int32_t* idx, int R, int row_bytes, void* dst, int dst_rows,
                     cudaStream_t st) {
    if (cudaMemsetAsync(dst, 0, size_t(dst_rows) * row_bytes, st) != cudaSuccess) return LQ_E_CUDA;
    const int chunks = row_bytes / 16;
    const size_t total = size_t(R) * chunks;
    if (total == 0) return LQ_OK;
    const int threads = 256;
    return norm_launch(scatter_rows_kernel, dim3(unsigned((total + threads - 1) / threads)), dim3(threads), st,
                       static_cast<const uint4*>(src), idx, R, chunks, static_cast<uint4*>(dst), dst_rows);
}

}  // namespace lq
