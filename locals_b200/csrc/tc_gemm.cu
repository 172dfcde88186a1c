// Prefill-size quantized GEMM ("tc" family) on the 5th-generation tensor cores:
// y (M, N) = x (M, K) . dequant(W)^T for M >= 128 (the reference's M >= PREFILL_M path,
// locals/kernels.py:854-866,1020-1025: dequantize + dense GEMM, here fused).
//
// One CTA computes a 128 x BN output tile over the whole K (non-persistent), ten warps:
//   warp 8      producer: TMA loads of the x tile (128 x 64, 128-byte swizzle) and of the packed weight
//               words (BN rows x 64 K) per 64-wide K block into a 3-stage ring; cp.async loads of the
//               16-bit scales and biases, eight groups at a time, into a 2-deep ring.
//   warps 0-7   dequantize the packed words of each K block straight into the B operand tile in shared
//               memory (BN rows x 64 K bf16/fp16, K-major, 128-byte swizzle): per 32-bit word one shift,
//               one lop3 with the 16-bit float "magic" exponent, one subtract and one fma per code pair
//               (the weight rounded once to the activation dtype, as mx.dequantize rounds it), then a
//               fence.proxy.async so the tensor core sees the stores.
//   warp 9      allocates BN TMEM columns and, from one elected lane, issues tcgen05.mma
//               (kind::f16, M = 128, N = BN, K = 16, fp32 accumulator in TMEM) from shared-memory
//               descriptors, committing each stage back to the producer.
//   epilogue    warps 0-7 read the accumulator with tcgen05.ld (warp w: TMEM lanes 32 (w % 4) ..,
//               column half w / 4), round to the activation dtype and store.
// Every mbarrier wait is bounded (LQ_DEV_TIMEOUT and an orderly exit: TMEM is always freed).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"

namespace lq {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;
constexpr int TC_MAX_STAGES = 5;  // x + packed-weight ring (fewer when the tiles are large)
constexpr int TC_BSTAGES = 2;  // dequantized weight tiles
constexpr int TC_THREADS = 320;
constexpr int TC_DEQ_THREADS = 256;

template <int BITS, int BN>
struct TcShape {
    static constexpr int A_BYTES = TC_BM * TC_BK * 2;        // 16 KB
    static constexpr int B_BYTES = BN * TC_BK * 2;           // dequantized weights
    static constexpr int WP_ROW = TC_BK * BITS / 8;          // packed bytes per row per K block (32 / 64)
    static constexpr int WP_BYTES = BN * WP_ROW;
    static constexpr int STAGE = A_BYTES + WP_BYTES;          // one slot of the load ring
    static constexpr int SB_BYTES = 2 * BN * 16;             // scales + biases, 8 groups per row
    static constexpr int STAGES_FIT = (225 * 1024 - TC_BSTAGES * B_BYTES - 2 * SB_BYTES) / STAGE;
    static constexpr int NS = STAGES_FIT < TC_MAX_STAGES ? STAGES_FIT : TC_MAX_STAGES;
    static constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0 && WP_BYTES % 1024 == 0, "1 KB alignment");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
};

struct TcArgs {
    int M, N, K;
    int nk;  // K / 64
    int sb_vec;
    const void* s;
    const void* b;
    void* y;
};

template <typename T, int BITS, int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, const TcArgs a) {
    using S = TcShape<BITS, BN>;
    using TR = F16Traits<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* b_ring = smem + S::NS * S::STAGE;           // [TC_BSTAGES][B_BYTES]
    uint8_t* sb_ring = b_ring + TC_BSTAGES * S::B_BYTES;      // [2][SB_BYTES]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sb_ring + 2 * S::SB_BYTES);
    uint64_t* tma_full = bars;                                // [S::NS]  x + packed words landed
    uint64_t* ld_empty = tma_full + S::NS;                // [S::NS]  the MMA is done with the x slot
    uint64_t* b_full = ld_empty + S::NS;                  // [TC_BSTAGES] dequantized tile written
    uint64_t* b_empty = b_full + TC_BSTAGES;                  // [TC_BSTAGES] the MMA is done with it
    uint64_t* sb_full = b_empty + TC_BSTAGES;                 // [2]
    uint64_t* sb_empty = sb_full + 2;                         // [2]
    uint64_t* acc_full = sb_empty + 2;                        // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * BN;
    const int nk = a.nk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::NS; ++s) {
            mbar_init(&tma_full[s], 1);
            mbar_init(&ld_empty[s], 1);
        }
        for (int s = 0; s < TC_BSTAGES; ++s) {
            mbar_init(&b_full[s], TC_DEQ_THREADS);
            mbar_init(&b_empty[s], 1);
        }
        for (int j = 0; j < 2; ++j) {
            mbar_init(&sb_full[j], 32);
            mbar_init(&sb_empty[j], TC_DEQ_THREADS);
        }
        mbar_init(acc_full, 1);
        fence_barrier_init();
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 8) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            prefetch_tmap(&tm_x);
            prefetch_tmap(&tm_w);
        }
        const uint64_t pol_w = policy_evict_first();
        const uint64_t pol_x = policy_evict_last();
        grid_dep_wait();
        const int kg = a.K / 64;
        const int vb = a.sb_vec;
        const int units_row = 16 / vb;
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int s = kb % S::NS;
            if (kb >= S::NS) ok = mbar_wait(&ld_empty[s], ((kb / S::NS) - 1) & 1);
            if (!ok) break;
            if ((kb & 7) == 0) {
                const int j = (kb >> 3) & 1;
                if (kb >= 16) ok = mbar_wait(&sb_empty[j], ((kb >> 4) - 1) & 1);
                if (!ok) break;
                const uint32_t dst0 = smem_u32(sb_ring + j * S::SB_BYTES);
                const uint8_t* sbase = reinterpret_cast<const uint8_t*>(a.s);
                const uint8_t* bbase = reinterpret_cast<const uint8_t*>(a.b);
                for (int r = lane; r < BN; r += 32) {
                    const int grow = n0 + r;
                    for (int pi = 0; pi < units_row; ++pi) {
                        const int gcol = kb + pi * (vb >> 1);
                        const bool valid = grow < a.N && gcol < kg;
                        const size_t off = valid ? (size_t(grow) * kg + gcol) * 2 : 0;
                        const uint32_t d = dst0 + r * 16 + pi * vb;
                        cp_async(d, sbase + off, vb, valid);
                        cp_async(d + BN * 16, bbase + off, vb, valid);
                    }
                }
                cp_async_arrive(&sb_full[j]);
            }
            if (lane == 0) {
                uint8_t* st = smem + s * S::STAGE;
                mbar_arrive_expect_tx(&tma_full[s], S::A_BYTES + S::WP_BYTES);
                tma_load_2d(st, &tm_x, &tma_full[s], kb * TC_BK, m0, pol_x);
                tma_load_2d(st + S::A_BYTES, &tm_w, &tma_full[s], kb * (TC_BK * BITS / 32), n0, pol_w);
            }
            __syncwarp();
        }
        if (lane == 0) grid_dep_launch();
    } else if (warp == 9) {
        // ------------------------------ MMA issuer ------------------------------
        constexpr uint32_t idesc = umma_idesc_f16(kBF16 ? 1 : 0, TC_BM, BN);
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int s = kb % S::NS, bs = kb % TC_BSTAGES;
            ok = mbar_wait(&b_full[bs], (kb / TC_BSTAGES) & 1);  // (the dequant warps waited for tma_full)
            if (!ok) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t a_base = smem_u32(smem + s * S::STAGE);
                const uint32_t b_base = smem_u32(b_ring + bs * S::B_BYTES);
#pragma unroll
                for (int k = 0; k < TC_BK / 16; ++k)
                    tc_mma_f16(tmem, umma_desc_sw128(a_base + k * 32), umma_desc_sw128(b_base + k * 32), idesc,
                               (kb > 0 || k > 0) ? 1u : 0u);
                tc_commit(&ld_empty[s]);
                tc_commit(&b_empty[bs]);
            }
            __syncwarp();
        }
        if (lane == 0) tc_commit(acc_full);  // (also on an error path: completes once issued MMAs finish)
        __syncwarp();
    } else {
        // ------------------------------ dequant warps 0-7 ------------------------------
        const int d = threadIdx.x;  // 0..255
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % S::NS, bs = kb % TC_BSTAGES;
            const int j = (kb >> 3) & 1;
            if (ok) ok = mbar_wait(&tma_full[s], (kb / S::NS) & 1);
            if (ok && (kb & 7) == 0) ok = mbar_wait(&sb_full[j], (kb >> 4) & 1);
            if (ok && kb >= TC_BSTAGES) ok = mbar_wait(&b_empty[bs], ((kb / TC_BSTAGES) - 1) & 1);
            if (ok) {
                uint8_t* st = smem + s * S::STAGE;
                const uint32_t bt = smem_u32(b_ring + bs * S::B_BYTES);
                const uint32_t wp = smem_u32(st + S::A_BYTES);
                const uint32_t sbt = smem_u32(sb_ring + j * S::SB_BYTES);
                const int g8 = kb & 7;
                // units: (row, half) -- half covers 4 of the row's 8 chunks of 8 K values. A thread owns
                // UPT units: every shared-memory load is issued first, then the arithmetic, then the stores,
                // so the units' latency chains overlap.
                constexpr int UPT = (2 * BN + TC_DEQ_THREADS - 1) / TC_DEQ_THREADS;
                constexpr int NW = BITS == 4 ? 4 : 8;  // packed words per unit
                uint32_t wv[UPT][NW];
                uint32_t s16[UPT], b16[UPT];
#pragma unroll
                for (int q = 0; q < UPT; ++q) {
                    const int u = d + q * TC_DEQ_THREADS;
                    const int row = (u < 2 * BN ? u : 0) >> 1, half = u & 1;
                    s16[q] = lds_u16(sbt + row * 16 + g8 * 2);
                    b16[q] = lds_u16(sbt + BN * 16 + row * 16 + g8 * 2);
#pragma unroll
                    for (int h2 = 0; h2 < NW / 4; ++h2) {
                        const uint4 w4 = lds128(wp + row * S::WP_ROW + half * (NW * 4) + h2 * 16);
                        wv[q][4 * h2] = w4.x;
                        wv[q][4 * h2 + 1] = w4.y;
                        wv[q][4 * h2 + 2] = w4.z;
                        wv[q][4 * h2 + 3] = w4.w;
                    }
                }
#pragma unroll
                for (int q = 0; q < UPT; ++q) {
                    const int u = d + q * TC_DEQ_THREADS;
                    if (u >= 2 * BN) break;
                    const int row = u >> 1, half = u & 1;
                    const uint32_t rsw = row & 7;
                    uint32_t o[4][4];
                    if constexpr (BITS == 4) {
                        const uint32_t s2 = prmt(s16[q], s16[q], 0x1010), b2 = prmt(b16[q], b16[q], 0x1010);
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            const uint32_t w = wv[q][c4];
                            uint32_t p[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e)  // codes (e, e + 4) -> dequantized pair
                                p[e] = TR::sub_magic_fma(lop3_and_or(w >> (4 * e), 0x000F000Fu, TR::kMagic2), s2, b2);
                            // K order inside the chunk: (0,1) (2,3) (4,5) (6,7)
                            o[c4][0] = prmt(p[0], p[1], 0x5410);
                            o[c4][1] = prmt(p[2], p[3], 0x5410);
                            o[c4][2] = prmt(p[0], p[1], 0x7632);
                            o[c4][3] = prmt(p[2], p[3], 0x7632);
                        }
                    } else {
                        const float sf = TR::to_f32(s16[q]), bf = TR::to_f32(b16[q]);
                        const uint32_t s2 = prmt(s16[q], s16[q], 0x1010), b2 = prmt(b16[q], b16[q], 0x1010);
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {  // chunk = 2 words = 8 K values
#pragma unroll
                            for (int wi = 0; wi < 2; ++wi) {
                                const uint32_t w = wv[q][2 * c4 + wi];
                                if constexpr (kBF16) {
                                    float f[4];
#pragma unroll
                                    for (int e = 0; e < 4; ++e)
                                        f[e] = fmaf(__uint_as_float(prmt(w, 0x4B000000u, 0x7540u + e)) - 8388608.0f, sf,
                                                    bf);
                                    o[c4][2 * wi] = cvt_bf16x2(f[1], f[0]);
                                    o[c4][2 * wi + 1] = cvt_bf16x2(f[3], f[2]);
                                } else {
                                    o[c4][2 * wi] = TR::sub_magic_fma(prmt(w, 0x64646464u, 0x5140u), s2, b2);
                                    o[c4][2 * wi + 1] = TR::sub_magic_fma(prmt(w, 0x64646464u, 0x5342u), s2, b2);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) {
                        const uint32_t c = half * 4 + c4;
                        const uint32_t dst = bt + row * 128 + ((c ^ rsw) << 4);
                        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(o[c4][0]), "r"(o[c4][1]),
                                     "r"(o[c4][2]), "r"(o[c4][3]));
                    }
                }
            }
            fence_proxy_async();  // generic-proxy stores -> visible to the tensor core (async proxy)
            mbar_arrive(&b_full[bs]);
            if ((kb & 7) == 7 || kb == nk - 1) mbar_arrive(&sb_empty[j]);
        }
        // ------------------------------ epilogue ------------------------------
        if (ok) ok = mbar_wait(acc_full, 0);
        tc_fence_after();
        const int lg = warp & 3, ch = warp >> 2;  // lane group (rows), column half
        const int m = m0 + 32 * lg + lane;
        constexpr int HALF = BN / 2;
#pragma unroll 1
        for (int c0 = 0; c0 < HALF; c0 += 32) {
            const int col = ch * HALF + c0;
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + (uint32_t(32 * lg) << 16) + uint32_t(col), r);
            tmem_wait_ld();
            if (!ok || m >= a.M) continue;
            const int n = n0 + col;
            T* yrow = reinterpret_cast<T*>(a.y) + size_t(m) * a.N;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                if (c0 + 8 * v >= HALF) break;  // (BN / 2 need not be a multiple of 32: stay inside the tile)
                const int nn = n + 8 * v;
                uint32_t o[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    o[q] = TR::pack2(__uint_as_float(r[8 * v + 2 * q + 1]), __uint_as_float(r[8 * v + 2 * q]));
                if (nn + 8 <= a.N && (a.N & 7) == 0) {
                    *reinterpret_cast<uint4*>(yrow + nn) = make_uint4(o[0], o[1], o[2], o[3]);
                } else {
                    for (int q = 0; q < 8; ++q)
                        if (nn + q < a.N) {
                            const uint32_t word = o[q >> 1];
                            const uint16_t h = (q & 1) ? uint16_t(word >> 16) : uint16_t(word & 0xFFFF);
                            reinterpret_cast<uint16_t*>(yrow)[nn + q] = h;
                        }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------

bool tc_shape_ok(int M, int N, int K, int bits) {
    (void)M;
    if (bits != 4 && bits != 8) return false;
    if (K < 64 || K % 128) return false;  // scale rows: 4-byte cp.async units need an even group count
    if (N < 16) return false;
    return true;
}

template <typename T, int BITS, int BN>
static int tc_launch_t(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K,
                       cudaStream_t st) {
    using S = TcShape<BITS, BN>;
    TcArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.nk = K / TC_BK;
    const int kg = K / 64;
    a.sb_vec = (kg % 8 == 0) ? 16 : (kg % 4 == 0) ? 8 : 4;
    a.s = s;
    a.b = b;
    a.y = y;
    CUtensorMap tx, tw;
    {
        const uint64_t dims[2] = {uint64_t(K), uint64_t(M)};
        const uint64_t str[1] = {uint64_t(K) * 2};
        const uint32_t box[2] = {TC_BK, TC_BM};
        int rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        const uint64_t dims[2] = {uint64_t(K) * BITS / 32, uint64_t(N)};
        const uint64_t str[1] = {uint64_t(K) * BITS / 8};
        const uint32_t box[2] = {uint32_t(TC_BK * BITS / 32), uint32_t(BN)};
        int rc = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, w, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    const size_t smem = 1024 + size_t(S::NS) * S::STAGE + size_t(TC_BSTAGES) * S::B_BYTES + 2 * S::SB_BYTES + 256;
    if (smem > device_info().smem_optin) return LQ_E_SHAPE;
    auto kern = tc_kernel<T, BITS, BN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((N + BN - 1) / BN, (M + TC_BM - 1) / TC_BM, 1);
    cfg.blockDim = dim3(TC_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, tx, tw, a);
    return e == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

// p = {BN} (0 = 224 when that divides N, else 256)
int tc_run(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K, int bits,
           int dtype, const int* p, cudaStream_t st) {
    int bn = p ? p[0] : 0;
    // 224-wide tiles measured faster than 256 on config 5 (more tiles per wave, 7 full waves on 148 SMs)
    if (bn == 0) bn = (N % 224 == 0) ? 224 : 256;
    const bool bf16 = dtype == LQ_BF16;
#define LQ_TC_CASE(BITS_, BN_)                                                                      \
    if (bits == BITS_ && bn == BN_)                                                                 \
        return bf16 ? tc_launch_t<__nv_bfloat16, BITS_, BN_>(x, w, s, b, y, M, N, K, st)            \
                    : tc_launch_t<__half, BITS_, BN_>(x, w, s, b, y, M, N, K, st);
    LQ_TC_CASE(4, 256)
    LQ_TC_CASE(4, 224)
    LQ_TC_CASE(4, 128)
    LQ_TC_CASE(8, 256)
    LQ_TC_CASE(8, 128)
#undef LQ_TC_CASE
    return LQ_E_UNSUPPORTED;
}

}  // namespace lq
