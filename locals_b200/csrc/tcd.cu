// Prefill as the reference's dense path: the weights dequantized once into the activation dtype, then a dense
// GEMM on the 5th-generation tensor cores (locals/kernels.py:999-1025, `_dense_matmul`: mx.dequantize into a
// temporary, then x @ w.T; used by the reference for N x K <= 2^27 weights, kernels.py:858-866).
//
// Why a second prefill form. The fused tc kernel dequantizes each weight tile inside every CTA that uses it, so at
// M = 2048 each weight is dequantized 16 times (once per 128-row token tile), and the dequant warps, not the tensor
// cores, bound it. Dequantizing once costs one HBM pass (read the 4-bit words, write the 16-bit weights: ~150 MB at
// config 5), after which the GEMM streams both operands by TMA and only the tensor pipe works.
//
// dequant4_kernel: one thread per 16 bytes of packed words (32 codes, half a group): one 16-byte load, per word one
//   shift, one lop3 with the 16-bit float magic exponent, one subtract and one fma per code pair (the weight
//   rounded once to the activation dtype, as mx.dequantize rounds it), four 16-byte stores in K order.
// tcd_kernel: persistent, one CTA per SM walking 128 x BN output tiles (token tiles fastest), six warps: warp 4
//   streams the x tile (128 x 64) and the weight tile (BN x 64), both 128-byte swizzled K-major (the UMMA canonical
//   layout), into a ring by TMA, running ahead across tiles; warp 5 allocates two BN-column TMEM accumulators and
//   issues tcgen05.mma (kind::f16, M = 128, N = BN, K = 16, fp32) from one lane, committing each slot back to the
//   producer and each finished tile to the epilogue; warps 0-3 read a finished accumulator with tcgen05.ld (warp w:
//   TMEM lanes 32w ..), store rounded rows and hand the accumulator back -- so a tile's epilogue runs under the next
//   tile's MMAs. Every mbarrier wait is bounded; TMEM is always freed.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"

namespace lq {

// ---- dequantize (4-bit, group 64) -----------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(256) dequant4_kernel(const uint4* __restrict__ wq, const uint16_t* __restrict__ s,
                                                       const uint16_t* __restrict__ b, uint32_t n_units, uint32_t K,
                                                       uint4* __restrict__ out) {
    using TR = F16Traits<T>;
    constexpr int UNR = 4;  // units a thread per step: every load is issued before any arithmetic
    grid_dep_wait();
    const uint32_t units_row = K / 32;  // 16-byte units (32 codes) a row
    const uint32_t groups_row = K / 64;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t u0 = blockIdx.x * blockDim.x + threadIdx.x; u0 < n_units; u0 += UNR * stride) {
        uint4 w4[UNR];
        uint32_t sv[UNR], bv[UNR];
#pragma unroll
        for (int j = 0; j < UNR; ++j) {
            const uint32_t u = u0 + j * stride;
            if (u < n_units) {
                const uint32_t row = u / units_row, piece = u - row * units_row;
                const size_t g = size_t(row) * groups_row + (piece >> 1);
                w4[j] = wq[u];
                sv[j] = s[g];
                bv[j] = b[g];
            }
        }
#pragma unroll
        for (int j = 0; j < UNR; ++j) {
            const uint32_t u = u0 + j * stride;
            if (u >= n_units) break;
            const uint32_t s2 = prmt(sv[j], sv[j], 0x1010), b2 = prmt(bv[j], bv[j], 0x1010);
            const uint32_t ws[4] = {w4[j].x, w4[j].y, w4[j].z, w4[j].w};
            uint4* dst = out + size_t(u) * 4;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t p[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)  // codes (e, e + 4) of the word
                    p[e] = TR::sub_magic_fma(lop3_and_or(ws[c] >> (4 * e), 0x000F000Fu, TR::kMagic2), s2, b2);
                dst[c] = make_uint4(prmt(p[0], p[1], 0x5410), prmt(p[2], p[3], 0x5410), prmt(p[0], p[1], 0x7632),
                                    prmt(p[2], p[3], 0x7632));  // K order (0,1) (2,3) (4,5) (6,7)
            }
        }
    }
    grid_dep_launch();
}

// ---- dense GEMM ---------------------------------------------------------------------------------

constexpr int TCD_BM = 128;
constexpr int TCD_BK = 64;
constexpr int TCD_THREADS = 192;
constexpr int TCD_MAX_STAGES = 6;

template <int BN>
struct TcdShape {
    static constexpr int A_BYTES = TCD_BM * TCD_BK * 2;  // 16 KB
    static constexpr int B_BYTES = BN * TCD_BK * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int FIT = (225 * 1024) / STAGE;
    static constexpr int NS = FIT < TCD_MAX_STAGES ? FIT : TCD_MAX_STAGES;
    static constexpr int ACC_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;  // one accumulator
    static constexpr int TMEM_COLS = 2 * ACC_COLS;                                           // double-buffered
    static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "1 KB alignment of swizzled tiles");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
};

constexpr int TCD_MAX_DST = 8;

struct TcdArgs {
    int M, N, K, nk;
    int mt, ntiles;  // token tiles, all tiles
    void* y;
    // Column-sharded output: ndst > 0 stores output element (m, n) at column col_off + n of row m (leading dimension
    // ldo) of dst[0] -- this rank's slice written in place into the gathered (M, ldo) layout -- instead of y.
    int ndst, col_off, ldo;
    void* dst[TCD_MAX_DST];
};

template <typename T, int BN>
__global__ void __launch_bounds__(TCD_THREADS, 1)
    tcd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, const TcdArgs a) {
    using S = TcdShape<BN>;
    using TR = F16Traits<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::NS * S::STAGE);
    uint64_t* empty = full + S::NS;
    uint64_t* acc_full = empty + S::NS;  // [2] the MMAs of a tile are done
    uint64_t* acc_empty = acc_full + 2;  // [2] the epilogue has read the accumulator
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = a.nk;
    // tiles of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...; token tiles vary fastest, so the CTAs working at
    // one time share their weight tiles (read once from DRAM, then from L2)
    const int my_tiles = a.ntiles > int(blockIdx.x) ? (a.ntiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int j = 0; j < 2; ++j) {
            mbar_init(&acc_full[j], 1);
            mbar_init(&acc_empty[j], 4);  // lane 0 of each epilogue warp
        }
        fence_barrier_init();
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 4) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            prefetch_tmap(&tm_x);
            prefetch_tmap(&tm_w);
            const uint64_t pol_x = policy_evict_last();
            const uint64_t pol_w = policy_evict_last();
            grid_dep_wait();  // x and the dequantized weights come from earlier kernels
            int it = 0;
            for (int j = 0; j < my_tiles && ok; ++j) {
                const int tile = int(blockIdx.x) + j * int(gridDim.x);
                const int m0 = (tile % a.mt) * TCD_BM, n0 = (tile / a.mt) * BN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % S::NS;
                    if (it >= S::NS && !(ok = mbar_wait(&empty[s], ((it / S::NS) - 1) & 1))) break;
                    uint8_t* st = smem + s * S::STAGE;
                    mbar_arrive_expect_tx(&full[s], S::STAGE);
                    tma_load_2d(st, &tm_x, &full[s], kb * TCD_BK, m0, pol_x);
                    tma_load_2d(st + S::A_BYTES, &tm_w, &full[s], kb * TCD_BK, n0, pol_w);
                }
            }
            grid_dep_launch();
        }
        __syncwarp();
    } else if (warp == 5) {
        // ------------------------------ MMA issuer ------------------------------
        constexpr uint32_t idesc = umma_idesc_f16(kBF16 ? 1 : 0, TCD_BM, BN);
        int it = 0;
        for (int j = 0; j < my_tiles && ok; ++j) {
            const int buf = j & 1;
            if (j >= 2) ok = mbar_wait(&acc_empty[buf], ((j >> 1) - 1) & 1);  // the epilogue read this accumulator
            if (!ok) break;
            tc_fence_after();
            const uint32_t acc = tmem + uint32_t(buf * S::ACC_COLS);
            for (int kb = 0; kb < nk && ok; ++kb, ++it) {
                const int s = it % S::NS;
                ok = mbar_wait(&full[s], (it / S::NS) & 1);
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_base = smem_u32(smem + s * S::STAGE);
                    const uint32_t b_base = a_base + S::A_BYTES;
#pragma unroll
                    for (int k = 0; k < TCD_BK / 16; ++k)
                        tc_mma_f16(acc, umma_desc_sw128(a_base + k * 32), umma_desc_sw128(b_base + k * 32), idesc,
                                   (kb > 0 || k > 0) ? 1u : 0u);
                    tc_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (lane == 0) tc_commit(&acc_full[buf]);  // (also after an error: completes once issued MMAs finish)
            __syncwarp();
        }
    } else {
        // ------------------------------ epilogue warps 0-3 ------------------------------
        const int ldo = a.ndst > 0 ? a.ldo : a.N, col_off = a.ndst > 0 ? a.col_off : 0;
        const bool vec = ((a.N | ldo | col_off) & 7) == 0;
        for (int j = 0; j < my_tiles; ++j) {
            const int buf = j & 1;
            const int tile = int(blockIdx.x) + j * int(gridDim.x);
            const int m0 = (tile % a.mt) * TCD_BM, n0 = (tile / a.mt) * BN;
            if (ok) ok = mbar_wait(&acc_full[buf], (j >> 1) & 1);
            if (!ok) break;
            tc_fence_after();
            const int m = m0 + 32 * warp + lane;
            const size_t row_off = size_t(m) * ldo + col_off;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem + (uint32_t(32 * warp) << 16) + uint32_t(buf * S::ACC_COLS + c0), r);
                tmem_wait_ld();
                if (m >= a.M) continue;
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int nn = n0 + c0 + 8 * v;
                    if (c0 + 8 * v >= BN || nn >= a.N) break;
                    uint32_t o[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        o[q] = TR::pack2(__uint_as_float(r[8 * v + 2 * q + 1]), __uint_as_float(r[8 * v + 2 * q]));
                    T* yrow = reinterpret_cast<T*>(a.ndst > 0 ? a.dst[0] : a.y) + row_off;
                    if (vec && nn + 8 <= a.N) {
                        *reinterpret_cast<uint4*>(yrow + nn) = make_uint4(o[0], o[1], o[2], o[3]);
                    } else {
                        for (int q = 0; q < 8; ++q)
                            if (nn + q < a.N) {
                                const uint32_t word = o[q >> 1];
                                reinterpret_cast<uint16_t*>(yrow)[nn + q] =
                                    (q & 1) ? uint16_t(word >> 16) : uint16_t(word & 0xFFFF);
                            }
                    }
                }
            }
            tc_fence_before();  // (the accumulator reads are complete before the MMA issuer reuses it)
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------

static int pdl_launch(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, func, args) == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

template <typename T>
static int dequant4_launch(const uint32_t* w, const void* s, const void* b, int N, int K, void* out, cudaStream_t st) {
    const int64_t units = int64_t(N) * (K / 32);
    if (units >= (int64_t(1) << 31)) return LQ_E_SHAPE;  // (32-bit unit indices)
    uint32_t n_units = uint32_t(units);
    const int threads = 256;
    int64_t blocks = (units + threads - 1) / threads;
    const int64_t cap = int64_t(device_info().sm_count) * 8;  // 2048 threads a SM, each 4 units a step
    if (blocks > cap) blocks = cap;
    const uint4* wq = reinterpret_cast<const uint4*>(w);
    const uint16_t* sp = static_cast<const uint16_t*>(s);
    const uint16_t* bp = static_cast<const uint16_t*>(b);
    uint32_t K_ = uint32_t(K);
    uint4* o = static_cast<uint4*>(out);
    void* args[] = {&wq, &sp, &bp, &n_units, &K_, &o};
    return pdl_launch(reinterpret_cast<const void*>(dequant4_kernel<T>), dim3(unsigned(blocks)), dim3(threads), 0, st,
                      args);
}

template <typename T, int BN>
static int tcd_launch_t(const void* x, const void* wd, void* y, int M, int N, int K, const TcdArgs* gather,
                        cudaStream_t st) {
    using S = TcdShape<BN>;
    TcdArgs a = {};
    if (gather) a = *gather;
    a.M = M;
    a.N = N;
    a.K = K;
    a.nk = K / TCD_BK;
    a.mt = (M + TCD_BM - 1) / TCD_BM;
    a.ntiles = a.mt * ((N + BN - 1) / BN);
    a.y = y;
    CUtensorMap tx, tw;
    {
        const uint64_t dims[2] = {uint64_t(K), uint64_t(M)};
        const uint64_t str[1] = {uint64_t(K) * 2};
        const uint32_t box[2] = {TCD_BK, TCD_BM};
        int rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        const uint64_t dims[2] = {uint64_t(K), uint64_t(N)};
        const uint64_t str[1] = {uint64_t(K) * 2};
        const uint32_t box[2] = {TCD_BK, uint32_t(BN)};
        int rc = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, wd, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    const size_t smem = 1024 + size_t(S::NS) * S::STAGE + (2 * S::NS + 4) * 8 + 64;
    if (smem > device_info().smem_optin) return LQ_E_SHAPE;
    auto kern = tcd_kernel<T, BN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    void* args[] = {&tx, &tw, &a};
    const int grid = a.ntiles < device_info().sm_count ? a.ntiles : device_info().sm_count;
    return pdl_launch(reinterpret_cast<const void*>(kern), dim3(grid, 1, 1), dim3(TCD_THREADS), smem, st, args);
}

size_t qmm_dense_workspace_bytes(int N, int K) { return size_t(N) * size_t(K) * 2; }

bool qmm_dense_shape_ok(int M, int N, int K, int bits) {
    return M >= 1 && N >= 16 && K >= 64 && K % 64 == 0 && (bits == 4 || bits == 8);
}

int dequantize_run(const uint32_t* wq, const void* s, const void* b, int N, int K, int bits, int group, int dt,
                   void* out, cudaStream_t st);

static int qmm_dense_impl(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K,
                          int bits, int dtype, void* workspace, const int* p, const TcdArgs* gather, cudaStream_t st) {
    const bool bf16 = dtype == LQ_BF16;
    int rc;
    if (bits == 4)
        rc = bf16 ? dequant4_launch<__nv_bfloat16>(w, s, b, N, K, workspace, st)
                  : dequant4_launch<__half>(w, s, b, N, K, workspace, st);
    else
        rc = dequantize_run(w, s, b, N, K, bits, 64, dtype, workspace, st);
    if (rc) return rc;
    int bn = p ? p[0] : 0;
    if (bn == 0) bn = (N % 224 == 0) ? 224 : 256;
#define LQ_TCD_CASE(BN_) \
    if (bn == BN_)       \
        return bf16 ? tcd_launch_t<__nv_bfloat16, BN_>(x, workspace, y, M, N, K, gather, st) : tcd_launch_t<__half, BN_>(x, workspace, y, M, N, K, gather, st);
    LQ_TCD_CASE(256)
    LQ_TCD_CASE(224)
    LQ_TCD_CASE(128)
#undef LQ_TCD_CASE
    return LQ_E_ARG;
}

// p = {BN (0 = 224 when that divides N, else 256)}. workspace: N x K weights in the activation dtype.
int qmm_dense_run(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K,
                  int bits, int dtype, void* workspace, const int* p, cudaStream_t st) {
    return qmm_dense_impl(x, w, s, b, y, M, N, K, bits, dtype, workspace, p, nullptr, st);
}

// Columns [col_off, col_off + ncols) of the row-major (M, ldo) buffer src copied into the same place of each of the
// ndst buffers dst[] (peers' buffers, P2P pointers over NVLink). One thread a 16-byte piece, consecutive threads
// along a row: every warp store is a run of 512 contiguous bytes, which NVLink carries at full width (one row per
// lane, as the GEMM epilogue stores, reached only a third of the link's rate on B200).
struct PushDst {
    uint4* p[TCD_MAX_DST];
};

__global__ void __launch_bounds__(256) push_cols_kernel_p(const uint4* __restrict__ src, const PushDst dst, int ndst,
                                                          int M, int pieces_row, int ld_pieces, int off_pieces) {
    grid_dep_wait();
    const int64_t total = int64_t(M) * pieces_row;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t m = i / pieces_row, c = i - m * pieces_row;
        const int64_t off = m * ld_pieces + off_pieces + c;
        const uint4 v = src[off];
#pragma unroll
        for (int d = 0; d < TCD_MAX_DST; ++d)
            if (d < ndst) dst.p[d][off] = v;
    }
}

// The column-sharded form: this rank's N output columns are written in place into columns [col_off, col_off + N)
// of its own (M, ldo) buffer dst[0] by the GEMM, then pushed to the same columns of dst[1 .. ndst) (the peers').
int qmm_dense_gather_run(const void* x, const uint32_t* w, const void* s, const void* b, void* const* dst, int ndst,
                         int col_off, int ldo, int M, int N, int K, int bits, int dtype, void* workspace, const int* p,
                         cudaStream_t st) {
    if (ndst < 1 || ndst > TCD_MAX_DST || col_off < 0 || ldo < col_off + N) return LQ_E_ARG;
    TcdArgs g = {};
    g.ndst = ndst;
    g.col_off = col_off;
    g.ldo = ldo;
    for (int d = 0; d < ndst; ++d) {
        if (!dst[d]) return LQ_E_ARG;
        g.dst[d] = dst[d];
    }
    int rc = qmm_dense_impl(x, w, s, b, dst[0], M, N, K, bits, dtype, workspace, p, &g, st);
    if (rc || ndst == 1) return rc;
    if ((N | col_off | ldo) % 8) return LQ_E_ALIGN;  // (16-byte pieces: the host checks before the GEMM)
    PushDst pd = {};
    for (int d = 1; d < ndst; ++d) pd.p[d - 1] = static_cast<uint4*>(dst[d]);
    const uint4* src = static_cast<const uint4*>(dst[0]);
    int nd = ndst - 1, M_ = M, pr = N / 8, ldp = ldo / 8, offp = col_off / 8;
    const int64_t total = int64_t(M) * pr;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = int64_t(device_info().sm_count) * 8;
    if (blocks > cap) blocks = cap;
    void* args[] = {&src, &pd, &nd, &M_, &pr, &ldp, &offp};
    return pdl_launch(reinterpret_cast<const void*>(push_cols_kernel_p), dim3(unsigned(blocks)), dim3(256), 0, st, args);
}

}  // namespace lq
