// Decode on the 5th-generation tensor cores (the "tcv" family): y (M <= 64 tokens) = x . dequant(w)^T.
//
// Per CTA: 128 weight rows (the MMA's M side) x a slice of K (split-K across a thread-block cluster);
// tokens are the MMA's N side (16, 32 or 64 columns).
//   * warp 12 streams the packed weight rows by TMA into a shared-memory ring, 128 bytes of each row per
//     slot (four 64-wide groups at 4 bits, two at 8 bits: narrower boxes cost the TMA unit far more per
//     byte and delay the x loads queued behind them);
//     it starts before the previous kernel has finished (programmatic dependent launch), so a layer's
//     weights are in flight while the layer before it still runs;
//   * warps 0-7 dequantize one group per step -- each thread one weight row, 64 values -- straight
//     into a tensor-memory ring with tcgen05.st (no shared-memory round trip for the bf16 weights);
//   * warp 13 waits for the previous kernel and streams x's groups by TMA (SW128, the canonical
//     K-major operand layout);
//   * warps 8-11 (one per SM sub-partition) each issue the tcgen05.mma of every fourth group into
//     their own accumulator: the per-issuer rate of small-N MMAs (~24 ns per M128xN16xK16 on B200)
//     would otherwise bound the kernel, four issuers run ~3.4x faster;
//   * warps 0-7 sum the accumulators, apply SwiGLU when gate and up rows are paired, and either store
//     (one K slice) or reduce the cluster's partial sums through distributed shared memory.
//
// Token tiles (grid z) of up to 256 columns make the same kernel a prefill GEMM in which every dequantized
// weight feeds 256 tokens and never passes through shared memory.
//
// The dequantized weight is s*q + b rounded once to the activation dtype (the reference's dequantize
// semantics, mlx quantized.h affine dequant), multiplied in the tensor core with fp32 accumulation.
// Token tiles of up to 64 (decode) take 256 tensor-memory columns and at most half an SM's shared memory:
// one launch places one CTA per SM (the occupancy calculator reports one block per SM for any kernel that
// allocates tensor memory), but the next launch's CTAs can then start beside it and load their weights
// while this launch still computes. Wider tiles (prefill) take all 512 columns and the opt-in shared memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"
#include "lq_status.cuh"
#include "qmv.h"
#include "tcv_common.cuh"

namespace lq {

template <typename T, int BITS, int NMAT, int NTOK, bool FULL>
__device__ __forceinline__ void tcv_body(const CUtensorMap& tm_w0, const CUtensorMap& tm_w1, const CUtensorMap& tm_x,
                                         const TcvArgs& a) {
    using S = TcvShape<BITS, NMAT, NTOK, FULL>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int WS = a.ws, XS = a.xs;
    uint8_t* wring = smem;
    uint8_t* xring = smem + a.w_bytes;
    uint32_t* sbm = reinterpret_cast<uint32_t*>(xring + XS * S::XSLOT);
    uint64_t* w_full = reinterpret_cast<uint64_t*>(sbm + NMAT * 2 * 128 * a.sbw);  // 256*sbw words: 8-byte aligned
    uint64_t* w_empty = w_full + TCV_MAX_SLOTS;
    uint64_t* x_full = w_empty + TCV_MAX_SLOTS;
    uint64_t* x_empty = x_full + TCV_MAX_SLOTS;
    uint64_t* a_full = x_empty + TCV_MAX_SLOTS;
    uint64_t* a_empty = a_full + S::AS;
    uint64_t* acc_full = a_empty + S::AS;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_full + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * 128;
    const int rank = blockIdx.y;
    int tok0 = blockIdx.z * NTOK;                     // first x row of this tile
    int mt = a.M - tok0 < NTOK ? a.M - tok0 : NTOK;   // rows of this tile
    int wrow = 0;                                     // first weight row of this tile's matrix
    if (a.grouped) {
        // segments come from the grouping kernel; tile z of the concatenated per-segment tile lists
        grid_dep_wait();
        int* tile_info = reinterpret_cast<int*>(smem_raw);  // (before anything else uses shared memory)
        if (warp == 0) {
            const int ns = a.nseg[0];
            const int z = blockIdx.z;
            int base = 0, seg = -1, tile = 0;
            for (int c = 0; c < ns; c += 32) {
                const int sg = c + lane;
                int t = 0;
                if (sg < ns) {
                    const int e = a.experts[sg], r = a.starts[sg + 1] - a.starts[sg];
                    if (e < 0 || e > a.n_experts || r < 0) record_status(LQ_DEV_BOUNDS);
                    else if (e < a.n_experts) t = (r + NTOK - 1) / NTOK;
                }
                int incl = t;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const int v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
                    if (lane >= d) incl += v;
                }
                const bool mine = z >= base + incl - t && z < base + incl;
                const unsigned hit = __ballot_sync(0xFFFFFFFFu, mine);
                if (hit) {
                    const int l = __ffs(hit) - 1;
                    seg = __shfl_sync(0xFFFFFFFFu, sg, l);
                    tile = z - base - __shfl_sync(0xFFFFFFFFu, incl - t, l);
                    break;
                }
                base += __shfl_sync(0xFFFFFFFFu, incl, 31);
            }
            if (lane == 0) {
                tile_info[0] = seg;
                if (seg >= 0) {
                    const int r0 = a.starts[seg] + tile * NTOK, r1 = a.starts[seg + 1];
                    tile_info[1] = r0;
                    tile_info[2] = r1 - r0 < NTOK ? r1 - r0 : NTOK;
                    tile_info[3] = a.experts[seg] * a.N;
                }
            }
        }
        __syncthreads();
        if (tile_info[0] < 0) return;  // past the last tile (the whole cluster shares blockIdx.z)
        tok0 = tile_info[1];
        mt = tile_info[2];
        wrow = tile_info[3];
        __syncthreads();  // the shared words are overwritten by the rings below
    }
    const int pairs = a.G >> 1;
    const int pb = rank * pairs / a.ks, pe = (rank + 1) * pairs / a.ks;
    const int g_begin = 2 * pb, GC = 2 * (pe - pb);  // this CTA's groups
    const int U = GC * NMAT;                         // dequant/MMA steps: (group, matrix)

    if (tid == 0) {
        for (int i = 0; i < WS; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 4 * NMAT * S::WG);  // every (group, matrix) step's four warps
        }
        for (int i = 0; i < XS; ++i) {
            mbar_init(&x_full[i], 1);
            mbar_init(&x_empty[i], NMAT);
        }
        for (int i = 0; i < S::AS; ++i) {
            mbar_init(&a_full[i], 4);
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(acc_full, U < S::NACC ? (U > 0 ? U : 1) : S::NACC);
        fence_barrier_init();
    }
    if (warp == 8) {
        tmem_alloc(tslot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    grid_dep_launch();

    // Producer and MMA roles run their loops with the whole warp (one lane issues): a lone lane whose warp
    // mates already wait at the CTA barrier below is scheduled so rarely that its TMAs and MMAs trickle out.
    if (warp == 12) {
        // ---- weight producer: every slot of this CTA's K slice, ahead of everything else
        if (lane == 0) {
            prefetch_tmap(&tm_w0);
            if (NMAT == 2) prefetch_tmap(&tm_w1);
        }
        const uint64_t pol = policy_evict_first();
        const int NW = (GC + S::WG - 1) / S::WG;  // slots of this CTA's K slice (the last may be partial)
        for (int wi = 0; wi < NW; ++wi) {
            const int s = wi % WS;
            if (wi >= WS) mbar_wait(&w_empty[s], ((wi / WS) - 1) & 1);
            if (lane == 0) {
                mbar_arrive_expect_tx(&w_full[s], NMAT * S::WSLOT);
                const int kx = (g_begin + wi * S::WG) * S::GW;
                tma_load_2d(wring + (s * NMAT) * S::WSLOT, &tm_w0, &w_full[s], kx, a.row_off[0] + wrow + n0, pol);
                if (NMAT == 2)
                    tma_load_2d(wring + (s * NMAT + 1) * S::WSLOT, &tm_w1, &w_full[s], kx, a.row_off[1] + wrow + n0,
                                pol);
            }
            __syncwarp();
        }
        // drain: the last fill of every slot has landed before the CTA may exit
        for (int s = 0; s < WS && s < NW; ++s) {
            const int wl = s + WS * ((NW - 1 - s) / WS);
            mbar_wait(&w_full[s], (wl / WS) & 1);
        }
    } else if (warp == 13) {
        // ---- x producer: waits for the kernel that wrote x
        if (lane == 0) prefetch_tmap(&tm_x);
        grid_dep_wait();
        const uint64_t pol = policy_evict_last();
        for (int gi = 0; gi < GC; ++gi) {
            const int s = gi % XS;
            if (gi >= XS) mbar_wait(&x_empty[s], ((gi / XS) - 1) & 1);
            if (lane == 0) {
                mbar_arrive_expect_tx(&x_full[s], S::XSLOT);
                tma_load_2d(xring + s * S::XSLOT, &tm_x, &x_full[s], (g_begin + gi) * 64, tok0, pol);
            }
            __syncwarp();
        }
        for (int s = 0; s < XS && s < GC; ++s) {
            const int gl = s + XS * ((GC - 1 - s) / XS);
            mbar_wait(&x_full[s], (gl / XS) & 1);
        }
    } else if (warp >= 8) {
        // ---- MMA issuers: issuer j takes steps j, j + NACC, ... into accumulator j
        const int j = warp - 8;
        if (j < S::NACC) {
            const uint32_t idesc = umma_idesc_f16(kBF16 ? 1 : 0, 128, NTOK);
            const uint64_t xd0 = umma_desc_sw128(smem_u32(xring));
            const uint32_t dcol = tbase + uint32_t(j * NTOK);
            for (int u = j; u < U; u += S::NACC) {
                const int gi = u / NMAT, xs = gi % XS, au = u % S::AS;
                mbar_wait(&a_full[au], (u / S::AS) & 1);
                mbar_wait(&x_full[xs], (gi / XS) & 1);
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t acol = tbase + uint32_t(S::DCOLS + au * 32);
                    const uint64_t xd = xd0 + uint64_t((xs * S::XSLOT) >> 4);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_ts(dcol, acol + 8 * kk, xd + 2 * kk, idesc, (u != j || kk != 0) ? 1u : 0u);
                    tc_commit(&a_empty[au]);
                    tc_commit(&x_empty[xs]);
                }
                __syncwarp();
            }
            if (j < U && lane == 0) tc_commit(acc_full);
            __syncwarp();
        }
    } else {
        // ---- dequant warps: quadrant q owns TMEM lanes / weight rows 32q..32q+31, half h takes every
        // other step
        const int q = warp & 3, h = warp >> 2;
        const int r = 32 * q + lane;
        {
            // this CTA's scales and biases, one row per thread, into a [matrix][s|b][row][pair] table
            const int npairs = GC >> 1;
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const int grow = a.row_off[m] + wrow + n0 + r;
                const bool ok = grow < a.rows_total[m];
                const size_t off = ok ? (size_t(grow) * a.G + g_begin) * 2 : 0;
                const char* sg = reinterpret_cast<const char*>(a.sptr[m]) + off;
                const char* bg = reinterpret_cast<const char*>(a.bptr[m]) + off;
                uint32_t* srow = sbm + ((m * 2 + 0) * 128 + r) * a.sbw;
                uint32_t* brow = sbm + ((m * 2 + 1) * 128 + r) * a.sbw;
                for (int w = h; w < npairs; w += 2) {
                    cp_async(smem_u32(srow + w), sg + 4 * w, 4, ok);
                    cp_async(smem_u32(brow + w), bg + 4 * w, 4, ok);
                }
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
            named_barrier(1, 256);
        }
        const uint32_t trow = tbase + (uint32_t(32 * q) << 16);
        for (int u = h; u < U; u += 2) {
            const int gi = u / NMAT, m = u % NMAT;
            const int wi = gi / S::WG, s = wi % WS, au = u % S::AS;
            mbar_wait(&w_full[s], (wi / WS) & 1);
            if (u >= S::AS) mbar_wait(&a_empty[au], ((u / S::AS) - 1) & 1);
            tc_fence_after();
            const uint32_t sw = sbm[((m * 2 + 0) * 128 + r) * a.sbw + (gi >> 1)];
            const uint32_t bw = sbm[((m * 2 + 1) * 128 + r) * a.sbw + (gi >> 1)];
            const uint32_t s16 = (gi & 1) ? (sw >> 16) : (sw & 0xFFFFu);
            const uint32_t b16 = (gi & 1) ? (bw >> 16) : (bw & 0xFFFFu);
            uint32_t v[32];
            tcv_dequant_row<T, BITS>(smem_u32(wring + (s * NMAT + m) * S::WSLOT) + r * 128, r,
                                     (gi % S::WG) * (S::GB / 16), s16, b16, v);
            tmem_st_32x32b_x32(trow + uint32_t(S::DCOLS + au * 32), v);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[au]);
                mbar_arrive(&w_empty[s]);
            }
        }

        // ---- epilogue: accumulators -> registers, summed per matrix
        mbar_wait(acc_full, 0);
        tc_fence_after();
        const int n = n0 + r;
        float* red = reinterpret_cast<float*>(wring);
        constexpr int HT = NTOK / 2;
#pragma unroll
        for (int c = 0; c < HT / S::CT; ++c) {
            const int t0 = h * HT + c * S::CT;
            float acc[NMAT][S::CT];
#pragma unroll
            for (int mm = 0; mm < NMAT; ++mm)
#pragma unroll
                for (int t = 0; t < S::CT; ++t) acc[mm][t] = 0.0f;
#pragma unroll
            for (int jj = 0; jj < S::NACC; ++jj) {
                if (jj >= U) break;
                uint32_t rv[S::CT];
                tmem_ld_cols<S::CT>(trow + uint32_t(jj * NTOK + t0), rv);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < S::CT; ++t) acc[jj % NMAT][t] += __uint_as_float(rv[t]);
            }
            if (a.ks == 1) {
                if (n < a.N) {
#pragma unroll
                    for (int t = 0; t < S::CT; ++t) {
                        const int tok = t0 + t;
                        if (tok >= mt) break;
                        float v0 = acc[0][t];
                        if constexpr (NMAT == 2) v0 = tcv_swiglu<T>(v0, acc[1][t]);
                        tcv_store(a, tok0 + tok, n, v0, kBF16);
                    }
                }
            } else {
#pragma unroll
                for (int mm = 0; mm < NMAT; ++mm)
#pragma unroll
                    for (int t = 0; t < S::CT; ++t) red[(mm * NTOK + t0 + t) * 128 + r] = acc[mm][t];
            }
        }
    }

    // tensor memory is free once every accumulator has been read
    tc_fence_before();
    __syncthreads();
    if (warp == 8) tmem_dealloc(tbase, S::TMEM_COLS);

    if (a.ks > 1) {
        // split-K: partial sums of the cluster's CTAs meet in distributed shared memory; CTA `rank`
        // finishes rows [rank*128/ks, (rank+1)*128/ks) of the tile for every token
        cluster_sync();
        if (warp < 8) {
            const float* red = reinterpret_cast<const float*>(wring);
            const int r0 = rank * 128 / a.ks, r1 = (rank + 1) * 128 / a.ks, nr = r1 - r0;
            const int total = mt * nr;
            for (int e = tid; e < total; e += 256) {
                const int tok = e / nr, row = r0 + e % nr;
                const int n = n0 + row;
                float v[NMAT];
#pragma unroll
                for (int mm = 0; mm < NMAT; ++mm) v[mm] = 0.0f;
                for (int p = 0; p < a.ks; ++p) {
#pragma unroll
                    for (int mm = 0; mm < NMAT; ++mm)
                        v[mm] += ld_dsmem_f(map_peer(smem_u32(&red[(mm * NTOK + tok) * 128 + row]), uint32_t(p)));
                }
                if (n < a.N) {
                    float v0 = v[0];
                    if constexpr (NMAT == 2) v0 = tcv_swiglu<T>(v0, v[NMAT - 1]);
                    tcv_store(a, tok0 + tok, n, v0, kBF16);
                }
            }
        }
        cluster_sync();  // peers keep their shared memory until every CTA has read it
    }
}

// Decode tiles (up to 64 tokens) at 64 registers: the register file is split over the SM's four
// sub-partitions and a 14-warp CTA puts four warps on some of them, so a second CTA -- the next launch's,
// loading its weights while this one computes -- fits beside it only at <= 64 registers (one launch still
// places one CTA per SM: the kernel holds tensor memory). Wide tiles (prefill) take what they need.
template <typename T, int BITS, int NMAT, int NTOK>
__global__ void __maxnreg__(64)
    tcv_kernel_dec(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                   const __grid_constant__ CUtensorMap tm_x, const TcvArgs a) {
    tcv_body<T, BITS, NMAT, NTOK, false>(tm_w0, tm_w1, tm_x, a);
}

// Wide tiles (prefill), and decode tiles in the FULL form (all of an SM's tensor memory, registers and shared memory:
// one CTA per SM and no room for the next launch's CTA, for weights large enough to keep the SM streaming alone).
template <typename T, int BITS, int NMAT, int NTOK, bool FULL>
__global__ void __launch_bounds__(TCV_THREADS, 1)
    tcv_kernel_wide(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_x, const TcvArgs a) {
    tcv_body<T, BITS, NMAT, NTOK, FULL>(tm_w0, tm_w1, tm_x, a);
}

// ------------------------------------------------------------------------------------------------

template <typename T, int BITS, int NMAT, int NTOK, bool FULL>
static int tcv_launch_t(const void* x, int x_rows, const QmvMats& mats, TcvArgs a, int ks, int ws_req, int gz,
                        cudaStream_t st) {
    using S = TcvShape<BITS, NMAT, NTOK, FULL>;
    const DeviceInfo& di = device_info();
    const int pairs = a.G / 2;
    if (ks < 1) ks = 1;
    if (ks > 8) ks = 8;
    if (ks > pairs) ks = pairs;
    a.ks = ks;
    const int gc_max = 2 * ((pairs + ks - 1) / ks);
    a.sbw = (gc_max / 2) | 1;
    const size_t sb_bytes = size_t(NMAT) * 2 * 128 * a.sbw * 4;
    const size_t bar_bytes = (4 * TCV_MAX_SLOTS + 2 * S::AS + 1) * 8 + 16;
    size_t budget = (NTOK <= 64 && !FULL) ? di.smem_per_sm / 2 - 2048 : di.smem_optin - 1024;
    const int nw_max = (gc_max + S::WG - 1) / S::WG;
    int ws = nw_max < TCV_MAX_SLOTS ? nw_max : TCV_MAX_SLOTS;
    int xs = gc_max < TCV_MAX_SLOTS ? gc_max : TCV_MAX_SLOTS;
    if (ws_req > 0 && ws_req < ws) ws = ws_req;
    // the split-K partial sums (ks > 1) overlay the weight and x rings, idle by then
    const size_t red = ks > 1 ? size_t(S::RED_BYTES) : 0;
    auto ring_bytes = [&](int w, int x) {
        size_t wb = size_t(w) * NMAT * S::WSLOT;
        const size_t xb = size_t(x) * S::XSLOT;
        if (wb + xb < red) wb = (red - xb + 1023) / 1024 * 1024;
        return wb;
    };
    auto total = [&](int w, int x) { return ring_bytes(w, x) + size_t(x) * S::XSLOT + sb_bytes + bar_bytes + 1024; };
    // half an SM when the rings fit (the next launch's CTAs can then start beside this one), else all of it
    if (total(2, 2) > budget) budget = di.smem_optin - 1024;
    // weights first (their loads run ahead of the dependency), then x
    while (total(ws, xs) > budget && xs > 4) --xs;
    while (total(ws, xs) > budget && ws > 2) --ws;
    while (total(ws, xs) > budget && xs > 2) --xs;
    if (total(ws, xs) > budget) return LQ_E_SHAPE;
    a.ws = ws;
    a.xs = xs;
    a.w_bytes = int(ring_bytes(ws, xs));
    const size_t smem = total(ws, xs);

    CUtensorMap tw[2], tx;
    for (int m = 0; m < NMAT; ++m) {
        const uint64_t wdims[2] = {uint64_t(a.K) * BITS / 32, uint64_t(mats.rows_total[m])};
        const uint64_t wstr[1] = {uint64_t(a.K) * BITS / 8};
        const uint32_t wbox[2] = {32, 128};
        const int rc = make_tmap(&tw[m], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, mats.w[m], wdims, wstr, wbox,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        a.sptr[m] = mats.s[m];
        a.bptr[m] = mats.b[m];
        a.rows_total[m] = mats.rows_total[m];
        a.row_off[m] = mats.row_off[m];
    }
    if (NMAT == 1) {
        tw[1] = tw[0];
        a.sptr[1] = a.sptr[0];
        a.bptr[1] = a.bptr[0];
        a.rows_total[1] = a.rows_total[0];
        a.row_off[1] = a.row_off[0];
    }
    {
        const uint64_t xdims[2] = {uint64_t(a.K), uint64_t(x_rows)};
        const uint64_t xstr[1] = {uint64_t(a.K) * 2};
        const uint32_t xbox[2] = {64, uint32_t(NTOK)};
        const int rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, xdims, xstr, xbox,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }

    void (*kern)(CUtensorMap, CUtensorMap, CUtensorMap, TcvArgs);
    if constexpr (NTOK <= 64 && !FULL)
        kern = tcv_kernel_dec<T, BITS, NMAT, NTOK>;
    else
        kern = tcv_kernel_wide<T, BITS, NMAT, NTOK, FULL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.N + 127) / 128, ks, gz > 0 ? gz : (a.M + NTOK - 1) / NTOK);
    cfg.blockDim = dim3(TCV_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (ks > 1) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = 1;
        attrs[na].val.clusterDim.y = ks;
        attrs[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    e = cudaLaunchKernelEx(&cfg, kern, tw[0], tw[1], tx, a);
    return e == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

template <typename T, int BITS, int NMAT>
static int tcv_dispatch_tok(int ntok, bool full, const void* x, int x_rows, const QmvMats& mats, const TcvArgs& a,
                            int ks, int ws, int gz, cudaStream_t st) {
    if (ntok == 16)
        return full ? tcv_launch_t<T, BITS, NMAT, 16, true>(x, x_rows, mats, a, ks, ws, gz, st)
                    : tcv_launch_t<T, BITS, NMAT, 16, false>(x, x_rows, mats, a, ks, ws, gz, st);
    if (ntok == 32)
        return full ? tcv_launch_t<T, BITS, NMAT, 32, true>(x, x_rows, mats, a, ks, ws, gz, st)
                    : tcv_launch_t<T, BITS, NMAT, 32, false>(x, x_rows, mats, a, ks, ws, gz, st);
    if (ntok == 64)
        return full ? tcv_launch_t<T, BITS, NMAT, 64, true>(x, x_rows, mats, a, ks, ws, gz, st)
                    : tcv_launch_t<T, BITS, NMAT, 64, false>(x, x_rows, mats, a, ks, ws, gz, st);
    if (ntok == 128) return tcv_launch_t<T, BITS, NMAT, 128, false>(x, x_rows, mats, a, ks, ws, gz, st);
    if constexpr (NMAT == 1) {
        if (ntok == 256) return tcv_launch_t<T, BITS, NMAT, 256, false>(x, x_rows, mats, a, ks, ws, gz, st);
    }
    return LQ_E_UNSUPPORTED;
}

static int tcv_dispatch(const void* x, int x_rows, const QmvMats& mats, int nmat, const TcvArgs& a, int bits, int dtype,
                        int ntok, bool full, int ks, int ws, int gz, cudaStream_t st) {
    const bool bf16 = dtype == LQ_BF16;
    if (bits == 4) {
        if (nmat == 1)
            return bf16 ? tcv_dispatch_tok<__nv_bfloat16, 4, 1>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st)
                        : tcv_dispatch_tok<__half, 4, 1>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st);
        return bf16 ? tcv_dispatch_tok<__nv_bfloat16, 4, 2>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st)
                    : tcv_dispatch_tok<__half, 4, 2>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st);
    }
    if (nmat == 1)
        return bf16 ? tcv_dispatch_tok<__nv_bfloat16, 8, 1>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st)
                    : tcv_dispatch_tok<__half, 8, 1>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st);
    return bf16 ? tcv_dispatch_tok<__nv_bfloat16, 8, 2>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st)
                : tcv_dispatch_tok<__half, 8, 2>(ntok, full, x, x_rows, mats, a, ks, ws, gz, st);
}

// K slices for rb row tiles: about 1.3 CTAs per SM in total (measured on B200 over the fused QKV,
// 8-bit gate/up and 8-bit down projections at 16-64 tokens: a kernel that holds tensor memory runs one CTA
// per SM, and clusters of more than two CTAs do not pack every SM, so a second partial wave of smaller
// slices beats one wave of large ones), at most 8 (portable cluster size).
static int tcv_default_ks(int rb, int pairs, int sms) {
    int ks = int(1.3 * sms / rb + 0.5);
    if (ks < 1) ks = 1;
    if (ks > 8) ks = 8;
    if (ks > pairs) ks = pairs;
    return ks;
}

bool tcv_shape_ok(int M, int K, int bits) {
    if (M < 1) return false;
    if (K < 128 || K % 128) return false;
    return bits == 4 || bits == 8;
}

// p = {NTOK, KS, WS, FORM} (0 = choose; FORM 2 = the full-SM form of a decode tile).
int tcv_run(const void* x, int M, const QmvMats& mats, int nmat, int N, int K, int nout, void* const* outs,
            const int* seg_end, const int* ldo, int bits, int dtype, const int* p, cudaStream_t st) {
    if (!tcv_shape_ok(M, K, bits)) return LQ_E_SHAPE;
    TcvArgs a = {};
    a.M = M;
    a.N = N;
    a.K = K;
    a.G = K / 64;
    a.nseg_out = nout;
    for (int i = 0; i < nout; ++i) {
        a.out[i] = outs[i];
        a.seg_end[i] = seg_end[i];
        a.ldo[i] = ldo[i];
    }
    int ntok = p ? p[0] : 0, ks = p ? p[1] : 0, ws = p ? p[2] : 0;
    if (ntok == 0) ntok = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 || nmat == 2 ? 128 : 256;
    if (ntok != 16 && ntok != 32 && ntok != 64 && ntok != 128 && ntok != 256) return LQ_E_ARG;
    if (ks == 0) ks = tcv_default_ks((N + 127) / 128 * ((M + ntok - 1) / ntok), a.G / 2, device_info().sm_count);
    const bool full = p && p[3] == 2 && ntok <= 64;
    return tcv_dispatch(x, M, mats, nmat, a, bits, dtype, ntok, full, ks, ws, 0, st);
}

// Grouped expert GEMMs (the MoE path): x = the expert-sorted rows xs (P rows), weights stacked (E, N, ...).
// Token tiles of 16/32/64 rows from the expected rows per expert; one K slice (the grid is large).
int tcv_run_grouped(const void* xs, int P, const QmvMats& mats, int nmat, int N, int K, void* out,
                    const int32_t* starts, const int32_t* experts, const int32_t* nseg, int E, int bits, int dtype,
                    const int* p, cudaStream_t st) {
    if (!tcv_shape_ok(P, K, bits)) return LQ_E_SHAPE;
    TcvArgs a = {};
    a.M = P;
    a.N = N;
    a.K = K;
    a.G = K / 64;
    a.nseg_out = 1;
    a.out[0] = out;
    a.seg_end[0] = N;
    a.ldo[0] = N;
    a.grouped = 1;
    a.starts = starts;
    a.experts = experts;
    a.nseg = nseg;
    a.n_experts = E;
    const int used = E < P ? E : P;
    const int expect = (P + used - 1) / used;
    int ntok = p ? p[0] : 0;
    if (ntok == 0) ntok = expect >= 24 ? 64 : expect >= 12 ? 32 : 16;
    if (ntok != 16 && ntok != 32 && ntok != 64) return LQ_E_ARG;
    // tiles: at most one partial tile per used expert plus P / ntok full ones
    const int gz = used + (P + ntok - 1) / ntok;
    return tcv_dispatch(xs, P, mats, nmat, a, bits, dtype, ntok, false, 1, p ? p[2] : 0, gz, st);
}

}  // namespace lq
