// Shared pieces of the tcgen05 decode families (tcv.cu and its persistent form tcvp.cu): launch arguments, the
// per-shape tensor-memory and shared-memory budget, the output store, the SwiGLU rounding and the per-row dequant
// of one 64-wide group into packed 16-bit pairs for tcgen05.st.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_ptx.cuh"

namespace lq {

constexpr int TCV_THREADS = 448;  // 8 dequant warps, 4 MMA warps, weight producer, x producer

constexpr int TCV_MAX_SLOTS = 40;

struct TcvArgs {
    int M, N, K;
    int G;         // K / 64 groups
    int ks;        // K slices (cluster size along y)
    int ws, xs;    // weight / x ring slots
    int sbw;       // 32-bit words per row of the scale (and bias) table in shared memory (odd)
    int w_bytes;   // bytes of the weight ring (with the x ring after it, also the split-K partial sums)
    int row_off[2];
    int rows_total[2];
    const void* sptr[2];
    const void* bptr[2];
    void* out[3];
    int seg_end[3];
    int ldo[3];
    int nseg_out;
    // grouped mode (MoE experts): grid z walks token tiles of the expert segments of a counting sort
    // (rows starts[s] .. starts[s+1] of x, expert experts[s], weights at row experts[s] * N of stacked
    // (E, N, ...) arrays); expert id n_experts is the padding bucket, skipped
    int grouped;
    const int32_t* starts;
    const int32_t* experts;
    const int32_t* nseg;
    int n_experts;
};

template <int BITS, int NMAT, int NTOK, bool FULL = false>
struct TcvShape {
    static constexpr int GB = BITS * 8;     // bytes of one row of one group: 32 (4-bit) or 64 (8-bit)
    static constexpr int GW = GB / 4;       // uint32 words of one row of one group
    static constexpr int WG = 128 / GB;     // groups per weight slot (128 bytes of every row)
    static constexpr int WSLOT = 128 * 128;  // one matrix, one slot, 128 rows of 128 bytes (SW128)
    static constexpr int XSLOT = NTOK * 128;  // one group of x for NTOK tokens, SW128 rows of 128 bytes
    // MMA issuers = accumulators: small-N MMAs are bound by the issue rate of one thread (~24 ns each on
    // B200), so narrow token tiles spread them over several issuing warps; a multiple of NMAT
    static constexpr int NACC = NTOK <= 16 ? 4 : (NTOK <= 64 || NMAT == 2) ? 2 : 1;
    // decode tiles keep half the tensor memory so the next launch's CTA can work beside this one; FULL (one CTA per SM,
    // for weights large enough to keep the SM streaming on their own) and wide tiles take all 512 columns
    static constexpr int TMEM_COLS = (NTOK <= 64 && !FULL) ? 256 : 512;
    static constexpr int DCOLS = NACC * NTOK;
    static constexpr int AS = (TMEM_COLS - DCOLS) / 32;  // tensor-memory A ring, one group (32 columns) each
    static_assert(AS >= 2 && DCOLS + 32 * AS <= TMEM_COLS, "accumulators and A ring exceed the TMEM allocation");
    static constexpr int RED_BYTES = NMAT * NTOK * 128 * 4;
    static constexpr int CT = NTOK / 2 < 16 ? NTOK / 2 : 16;  // tokens per epilogue chunk of one warp
};

template <typename A>
__device__ __forceinline__ void tcv_store(const A& a, int tok, int n, float v, bool bf16) {
    int seg = 0, start = 0;
    if (a.nseg_out > 1 && n >= a.seg_end[0]) {
        seg = 1;
        start = a.seg_end[0];
        if (a.nseg_out > 2 && n >= a.seg_end[1]) {
            seg = 2;
            start = a.seg_end[1];
        }
    }
    const size_t off = size_t(tok) * a.ldo[seg] + (n - start);
    if (bf16)
        reinterpret_cast<__nv_bfloat16*>(a.out[seg])[off] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<__half*>(a.out[seg])[off] = __float2half_rn(v);
}

template <typename T>
__device__ __forceinline__ float tcv_round(float v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __bfloat162float(__float2bfloat16_rn(v));
    else
        return __half2float(__float2half_rn(v));
}

// silu(gate) * up with the activation-dtype rounding points of the reference's SwiGLU (gate and up
// rounded, sigmoid rounded, silu rounded, product rounded by the store).
template <typename T>
__device__ __forceinline__ float tcv_swiglu(float g, float u) {
    const float gt = tcv_round<T>(g), ut = tcv_round<T>(u);
    const float sig = tcv_round<T>(1.0f / (1.0f + expf(-gt)));
    return tcv_round<T>(gt * sig) * ut;
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 8)
        tmem_ld_32x32b_x8(taddr, r);
    else if constexpr (N == 16)
        tmem_ld_32x32b_x16(taddr, r);
    else
        tmem_ld_32x32b_x32(taddr, r);
}

// One weight row of one 64-wide group -> 32 packed pairs (k = 2j, 2j+1) in the activation dtype. The
// row's 128 bytes in the slot are in the SW128 layout (16-byte chunk c stored at c ^ (row & 7)), which
// keeps the warp's 32 row reads conflict-free; the group starts at chunk c0.
template <typename T, int BITS>
__device__ __forceinline__ void tcv_dequant_row(uint32_t rowp, int r, int c0, uint32_t s16, uint32_t b16,
                                                uint32_t (&v)[32]) {
    using TR = F16Traits<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    const int sw = r & 7;
    if constexpr (BITS == 4) {
        const uint4 u0 = lds128(rowp + (((c0 + 0) ^ sw) << 4));
        const uint4 u1 = lds128(rowp + (((c0 + 1) ^ sw) << 4));
        const uint32_t wd[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        const uint32_t s2 = s16 | (s16 << 16), b2 = b16 | (b16 << 16);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t w = wd[j], w4 = w >> 4;
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                // code 2p is the low nibble of byte p of w, code 2p+1 the low nibble of byte p of w >> 4
                const uint32_t sel = uint32_t(p) | (uint32_t(p) << 4) | (uint32_t(4 + p) << 8) | (uint32_t(p) << 12);
                v[4 * j + p] = TR::sub_magic_fma(lop3_and_or(prmt(w, w4, sel), 0x000F000Fu, TR::kMagic2), s2, b2);
            }
        }
    } else {
        uint32_t wd[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 u = lds128(rowp + (((c0 + c) ^ sw) << 4));
            wd[4 * c + 0] = u.x;
            wd[4 * c + 1] = u.y;
            wd[4 * c + 2] = u.z;
            wd[4 * c + 3] = u.w;
        }
        if constexpr (kBF16) {
            // a byte code as float: OR it into the mantissa of 2^23, subtract 2^23; s*q + b in fp32, one rounding
            const float sf = TR::to_f32(s16), bf = TR::to_f32(b16);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float f[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    f[i] = fmaf(__uint_as_float(prmt(wd[j], 0x4B000000u, 0x7540u + i)) - 8388608.0f, sf, bf);
                v[2 * j] = cvt_bf16x2(f[1], f[0]);
                v[2 * j + 1] = cvt_bf16x2(f[3], f[2]);
            }
        } else {
            const uint32_t s2 = s16 | (s16 << 16), b2 = b16 | (b16 << 16);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                v[2 * j] = TR::sub_magic_fma(prmt(wd[j], 0x64646464u, 0x5140u), s2, b2);
                v[2 * j + 1] = TR::sub_magic_fma(prmt(wd[j], 0x64646464u, 0x5342u), s2, b2);
            }
        }
    }
}

}  // namespace lq
