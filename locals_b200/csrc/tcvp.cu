// Persistent form of the tcv family: one CTA per SM walks tiles (128 weight rows x a token tile) with
// its rings running on across tiles, for launches with more tiles than SMs -- the grouped MoE expert
// GEMMs and wide-token (prefill) inputs. Against one CTA per tile it removes the per-tile prologue
// (barrier set-up, tensor-memory allocation, scale loads, the first HBM round trip) from every wave
// after the first and lets a tile's weights stream in while the previous tile computes:
//   * warp 12 streams each 128-byte weight slot (four 4-bit groups / two 8-bit groups per row) by TMA
//     together with the slot's scales and biases (cp.async), for tile after tile;
//   * warp 13 streams x groups (SW128) for tile after tile;
//   * warps 0-7 dequantize into the tensor-memory A ring; after filling the ring with the first steps
//     of tile i they run the epilogue of tile i-1 (its accumulator is double-buffered when tensor
//     memory allows, so the MMAs of tile i do not wait for it);
//   * warps 8-11 issue the MMAs, one accumulator each.
// Only for K slices of whole slots (K % 256 == 0 at 4 bits, K % 128 == 0 at 8 bits) and one K slice
// per tile.
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

constexpr int TCVP_MAX_SLOTS = 24;
constexpr int TCVP_MAX_SEGS = 1040;  // segments of a grouping (experts + the padding bucket)

template <int BITS, int NMAT, int NTOK>
struct TcvpShape {
    static constexpr int GB = BITS * 8;     // bytes of one row of one group
    static constexpr int GW = GB / 4;
    static constexpr int WG = 128 / GB;     // groups per weight slot
    static constexpr int WSLOT = 128 * 128;  // packed words of one matrix, one slot (SW128)
    static constexpr int SBSLOT = 2 * 128 * WG * 2;  // scales then biases, [row][group] of one matrix, one slot
    static constexpr int MSLOT = WSLOT + SBSLOT;     // one matrix of one slot (a multiple of 1024)
    static constexpr int XSLOT = NTOK * 128;
    static constexpr int NACC = NTOK <= 16 ? 4 : (NTOK <= 64 || NMAT == 2) ? 2 : 1;
    static constexpr int DCOLS = NACC * NTOK;
    static constexpr int NDB = (2 * DCOLS + 4 * 32 <= 512) ? 2 : 1;  // accumulator buffers
    static constexpr int AS = (512 - NDB * DCOLS) / 32;               // A ring, one group per step
    static constexpr int CT = NTOK / 2 < 16 ? NTOK / 2 : (NMAT == 1 && NTOK >= 64) ? 32 : 16;
    static_assert(MSLOT % 1024 == 0, "slot layout");
    static_assert(AS >= 4 && NDB * DCOLS + 32 * AS <= 512, "tensor memory budget");
};

struct TcvpTile {
    int n0, tok0, mt, wrow;
};

template <int NTOK>
__device__ __forceinline__ TcvpTile tcvp_tile(const TcvArgs& a, int rb_count, int t, const int* prefix, int nseg) {
    TcvpTile r;
    if (!a.grouped) {
        // token tile fastest: the CTAs running together read different x tiles and share each weight
        // tile through L2
        const int zt = (a.M + NTOK - 1) / NTOK;
        const int z = t % zt, rb = t / zt;
        r.n0 = rb * 128;
        r.tok0 = z * NTOK;
        r.mt = a.M - r.tok0 < NTOK ? a.M - r.tok0 : NTOK;
        r.wrow = 0;
        return r;
    }
    const int rb = t % rb_count, z = t / rb_count;
    r.n0 = rb * 128;
    int lo = 0, hi = nseg;  // prefix[lo] <= z < prefix[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] <= z) lo = mid;
        else hi = mid;
    }
    const int r0 = a.starts[lo] + (z - prefix[lo]) * NTOK, r1 = a.starts[lo + 1];
    r.tok0 = r0;
    r.mt = r1 - r0 < NTOK ? r1 - r0 : NTOK;
    r.wrow = a.experts[lo] * a.N;
    return r;
}

template <typename T, int BITS, int NMAT, int NTOK>
__global__ void __launch_bounds__(448, 1)
    tcvp_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                const __grid_constant__ CUtensorMap tm_x, const TcvArgs a) {
    using S = TcvpShape<BITS, NMAT, NTOK>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int WS = a.ws, XS = a.xs;
    uint8_t* wring = smem;                         // WS slots x NMAT x (packed words | scales | biases)
    uint8_t* xring = smem + WS * NMAT * S::MSLOT;  // XS groups of x
    uint64_t* bars = reinterpret_cast<uint64_t*>(xring + XS * S::XSLOT);
    uint64_t* w_full = bars;
    uint64_t* w_empty = w_full + TCVP_MAX_SLOTS;
    uint64_t* x_full = w_empty + TCVP_MAX_SLOTS;
    uint64_t* x_empty = x_full + TCVP_MAX_SLOTS;
    uint64_t* a_full = x_empty + TCVP_MAX_SLOTS;
    uint64_t* a_empty = a_full + S::AS;
    uint64_t* acc_full = a_empty + S::AS;
    uint64_t* d_empty = acc_full + S::NDB;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(d_empty + S::NDB);
    int* prefix = reinterpret_cast<int*>(tslot + 4);  // grouped: tiles before segment s (nseg + 1 entries)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.G;                    // groups per row (K / 64): one tile's steps per matrix
    const int NW = G / S::WG;             // weight slots per tile
    const int U = G * NMAT;               // dequant / MMA steps per tile
    const int RB = (a.N + 127) / 128;     // row tiles
    const int rot = blockIdx.x % NW;      // first slot of every tile's K walk: CTAs spread over K

    // ---- tiles of this launch (grouped: from the counting sort of the previous kernel)
    int nseg = 0, ntiles;
    if (a.grouped) {
        grid_dep_wait();
        if (warp == 0) {
            nseg = a.nseg[0];
            if (nseg > TCVP_MAX_SEGS - 1) {
                if (lane == 0) record_status(LQ_DEV_BOUNDS);
                nseg = TCVP_MAX_SEGS - 1;
            }
            int base = 0;
            for (int c = 0; c < nseg; c += 32) {
                const int sg = c + lane;
                int t = 0;
                if (sg < nseg) {
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
                if (sg < nseg) prefix[sg] = base + incl - t;
                base += __shfl_sync(0xFFFFFFFFu, incl, 31);
            }
            if (lane == 0) prefix[nseg] = base;
        }
    }

    if (tid == 0) {
        for (int i = 0; i < WS; ++i) {
            mbar_init(&w_full[i], 1 + 32);               // expect_tx arrival + 32 cp.async arrivals
            mbar_init(&w_empty[i], 4 * NMAT * S::WG);    // every (group, matrix) step's four warps
        }
        for (int i = 0; i < XS; ++i) {
            mbar_init(&x_full[i], 1);
            mbar_init(&x_empty[i], NMAT);
        }
        for (int i = 0; i < S::AS; ++i) {
            mbar_init(&a_full[i], 4);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < S::NDB; ++i) {
            mbar_init(&acc_full[i], S::NACC);
            mbar_init(&d_empty[i], 8);
        }
        fence_barrier_init();
    }
    if (warp == 8) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    if (a.grouped) nseg = a.nseg[0] < TCVP_MAX_SEGS - 1 ? a.nseg[0] : TCVP_MAX_SEGS - 1;
    ntiles = RB * (a.grouped ? prefix[nseg] : (a.M + NTOK - 1) / NTOK);
    grid_dep_launch();

    if (warp == 12) {
        // ---- weights and their scales / biases, slot by slot, tile after tile
        if (lane == 0) {
            prefetch_tmap(&tm_w0);
            if (NMAT == 2) prefetch_tmap(&tm_w1);
        }
        const uint64_t pol = policy_evict_first();
        int wc = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
            const TcvpTile tl = tcvp_tile<NTOK>(a, RB, t, prefix, nseg);
            for (int wi = 0; wi < NW; ++wi, ++wc) {
                const int s = wc % WS;
                if (wc >= WS) mbar_wait(&w_empty[s], ((wc / WS) - 1) & 1);
                uint8_t* slot = wring + s * NMAT * S::MSLOT;
                if (lane == 0) {
                    mbar_arrive_expect_tx(&w_full[s], NMAT * S::WSLOT);
                    const int kx = ((wi + rot) % NW) * S::WG * S::GW;
                    tma_load_2d(slot, &tm_w0, &w_full[s], kx, a.row_off[0] + tl.wrow + tl.n0, pol);
                    if (NMAT == 2)
                        tma_load_2d(slot + S::MSLOT, &tm_w1, &w_full[s], kx, a.row_off[1] + tl.wrow + tl.n0, pol);
                }
                // scales and biases of the slot's groups: one row per lane and pass, WG * 2 bytes each
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint8_t* sg = reinterpret_cast<const uint8_t*>(a.sptr[m]);
                    const uint8_t* bg = reinterpret_cast<const uint8_t*>(a.bptr[m]);
                    const uint32_t dst = smem_u32(slot + m * S::MSLOT + S::WSLOT);
#pragma unroll
                    for (int rr = 0; rr < 128; rr += 32) {
                        const int r = rr + lane;
                        const int grow = a.row_off[m] + tl.wrow + tl.n0 + r;
                        const bool ok = grow < a.rows_total[m];
                        const size_t off = ok ? (size_t(grow) * G + ((wi + rot) % NW) * S::WG) * 2 : 0;
                        cp_async(dst + r * (S::WG * 2), sg + off, S::WG * 2, ok);
                        cp_async(dst + 128 * S::WG * 2 + r * (S::WG * 2), bg + off, S::WG * 2, ok);
                    }
                }
                cp_async_arrive(&w_full[s]);
                __syncwarp();
            }
        }
        for (int s = 0; s < WS && s < wc; ++s) {
            const int wl = s + WS * ((wc - 1 - s) / WS);
            mbar_wait(&w_full[s], (wl / WS) & 1);
        }
    } else if (warp == 13) {
        // ---- x, group by group, tile after tile
        if (lane == 0) prefetch_tmap(&tm_x);
        if (!a.grouped) grid_dep_wait();
        const uint64_t pol = policy_evict_last();
        int xc = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
            const TcvpTile tl = tcvp_tile<NTOK>(a, RB, t, prefix, nseg);
            for (int gi = 0; gi < G; ++gi, ++xc) {
                const int s = xc % XS;
                if (xc >= XS) mbar_wait(&x_empty[s], ((xc / XS) - 1) & 1);
                if (lane == 0) {
                    mbar_arrive_expect_tx(&x_full[s], S::XSLOT);
                    const int ga = ((gi / S::WG + rot) % NW) * S::WG + gi % S::WG;  // the group this step holds
                    tma_load_2d(xring + s * S::XSLOT, &tm_x, &x_full[s], ga * 64, tl.tok0, pol);
                }
                __syncwarp();
            }
        }
        for (int s = 0; s < XS && s < xc; ++s) {
            const int xl = s + XS * ((xc - 1 - s) / XS);
            mbar_wait(&x_full[s], (xl / XS) & 1);
        }
    } else if (warp >= 8) {
        // ---- MMA issuers
        const int j = warp - 8;
        if (j < S::NACC) {
            const uint32_t idesc = umma_idesc_f16(kBF16 ? 1 : 0, 128, NTOK);
            const uint64_t xd0 = umma_desc_sw128(smem_u32(xring));
            int it = 0, ub = 0, xb = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it, ub += U, xb += G) {
                const int db = it % S::NDB;
                if (it >= S::NDB) mbar_wait(&d_empty[db], ((it / S::NDB) - 1) & 1);
                tc_fence_after();
                const uint32_t dcol = tbase + uint32_t((db * S::NACC + j) * NTOK);
                for (int u = j; u < U; u += S::NACC) {
                    const int ug = ub + u, gi = u / NMAT, xg = xb + gi;
                    const int au = ug % S::AS, xs = xg % XS;
                    mbar_wait(&a_full[au], (ug / S::AS) & 1);
                    mbar_wait(&x_full[xs], (xg / XS) & 1);
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t acol = tbase + uint32_t(S::NDB * S::DCOLS + au * 32);
                        const uint64_t xd = xd0 + uint64_t((xs * S::XSLOT) >> 4);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc_mma_ts(dcol, acol + 8 * kk, xd + 2 * kk, idesc, (u != j || kk != 0) ? 1u : 0u);
                        tc_commit(&a_empty[au]);
                        tc_commit(&x_empty[xs]);
                    }
                    __syncwarp();
                }
                if (lane == 0) tc_commit(&acc_full[db]);
                __syncwarp();
            }
        }
    } else {
        // ---- dequant warps (+ the epilogue of the previous tile)
        const int q = warp & 3, h = warp >> 2;
        const int r = 32 * q + lane;
        const uint32_t trow = tbase + (uint32_t(32 * q) << 16);
        auto epilogue = [&](int it, const TcvpTile& tl) {
            const int db = it % S::NDB;
            mbar_wait(&acc_full[db], (it / S::NDB) & 1);
            tc_fence_after();
            constexpr int HT = NTOK / 2;
            const int n = tl.n0 + r;
#pragma unroll 1
            for (int c = 0; c < HT / S::CT; ++c) {
                const int t0 = h * HT + c * S::CT;
                float acc[NMAT][S::CT];
#pragma unroll
                for (int mm = 0; mm < NMAT; ++mm)
#pragma unroll
                    for (int tt = 0; tt < S::CT; ++tt) acc[mm][tt] = 0.0f;
#pragma unroll
                for (int jj = 0; jj < S::NACC; ++jj) {
                    if (jj >= U) break;  // (an issuer without steps never wrote its accumulator)
                    uint32_t rv[S::CT];
                    tmem_ld_cols<S::CT>(trow + uint32_t((db * S::NACC + jj) * NTOK + t0), rv);
                    tmem_wait_ld();
#pragma unroll
                    for (int tt = 0; tt < S::CT; ++tt) acc[jj % NMAT][tt] += __uint_as_float(rv[tt]);
                }
                if (c == HT / S::CT - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&d_empty[db]);
                }
                if (n < a.N) {
#pragma unroll
                    for (int tt = 0; tt < S::CT; ++tt) {
                        const int tok = t0 + tt;
                        if (tok >= tl.mt) break;
                        float v0 = acc[0][tt];
                        if constexpr (NMAT == 2) v0 = tcv_swiglu<T>(v0, acc[1][tt]);
                        tcv_store(a, tl.tok0 + tok, n, v0, kBF16);
                    }
                }
            }
        };
        int it = 0, ub = 0, wb = 0;
        TcvpTile prev = {0, 0, 0, 0};
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it, ub += U, wb += NW) {
            const TcvpTile tl = tcvp_tile<NTOK>(a, RB, t, prefix, nseg);
            bool pending = it > 0;
            for (int u = h; u < U; u += 2) {
                if (pending && u >= S::AS) {  // the ring holds this tile's first steps: finish the last tile
                    epilogue(it - 1, prev);
                    pending = false;
                }
                const int gi = u / NMAT, m = u % NMAT;
                const int ug = ub + u, wi = wb + gi / S::WG;
                const int s = wi % WS, au = ug % S::AS;
                mbar_wait(&w_full[s], (wi / WS) & 1);
                if (ug >= S::AS) mbar_wait(&a_empty[au], ((ug / S::AS) - 1) & 1);
                tc_fence_after();
                const uint8_t* mslot = wring + (s * NMAT + m) * S::MSLOT;
                const uint32_t sbp = smem_u32(mslot + S::WSLOT) + r * (S::WG * 2) + (gi % S::WG) * 2;
                const uint32_t s16 = lds_u16(sbp), b16 = lds_u16(sbp + 128 * S::WG * 2);
                uint32_t v[32];
                tcv_dequant_row<T, BITS>(smem_u32(mslot) + r * 128, r, (gi % S::WG) * (S::GB / 16), s16, b16, v);
                tmem_st_32x32b_x32(trow + uint32_t(S::NDB * S::DCOLS + au * 32), v);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[au]);
                    mbar_arrive(&w_empty[s]);
                }
            }
            if (pending) epilogue(it - 1, prev);
            prev = tl;
        }
        if (it > 0) epilogue(it - 1, prev);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 8) tmem_dealloc(tbase, 512);
}

// ------------------------------------------------------------------------------------------------

template <typename T, int BITS, int NMAT, int NTOK>
static int tcvp_launch_t(const void* x, int x_rows, const QmvMats& mats, TcvArgs a, int tiles_max, cudaStream_t st) {
    using S = TcvpShape<BITS, NMAT, NTOK>;
    const DeviceInfo& di = device_info();
    const size_t budget = di.smem_optin - 1024;
    const size_t fixed = (4 * TCVP_MAX_SLOTS + 2 * S::AS + 2 * S::NDB) * 8 + 16 + TCVP_MAX_SEGS * 4 + 1024;
    // the same look-ahead in groups for weights (from HBM) and x (from L2): a short x ring starved the MMAs
    auto total = [&](int w, int xg) { return size_t(w) * NMAT * S::MSLOT + size_t(xg) * S::XSLOT + fixed; };
    int ws = 2, xs = 2;
    for (int L = TCVP_MAX_SLOTS; L >= 2; --L) {
        const int w = (L + S::WG - 1) / S::WG < 2 ? 2 : (L + S::WG - 1) / S::WG;
        if (w <= TCVP_MAX_SLOTS && total(w, L) <= budget) {
            ws = w;
            xs = L;
            break;
        }
    }
    if (total(ws, xs) > budget) return LQ_E_SHAPE;
    a.ws = ws;
    a.xs = xs;
    const size_t smem = total(ws, xs);
    for (int m = 0; m < NMAT; ++m)  // scales / biases move WG * 2 bytes per row and slot
        if ((reinterpret_cast<uintptr_t>(mats.s[m]) | reinterpret_cast<uintptr_t>(mats.b[m])) % (S::WG * 2))
            return LQ_E_SHAPE;

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
    auto kern = tcvp_kernel<T, BITS, NMAT, NTOK>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    const int grid = tiles_max < di.sm_count ? tiles_max : di.sm_count;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(448, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, tw[0], tw[1], tx, a);
    return e == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

template <typename T, int BITS, int NMAT>
static int tcvp_dispatch_tok(int ntok, const void* x, int x_rows, const QmvMats& mats, const TcvArgs& a, int tiles_max,
                             cudaStream_t st) {
    if (ntok == 16) return tcvp_launch_t<T, BITS, NMAT, 16>(x, x_rows, mats, a, tiles_max, st);
    if (ntok == 32) return tcvp_launch_t<T, BITS, NMAT, 32>(x, x_rows, mats, a, tiles_max, st);
    if (ntok == 64) return tcvp_launch_t<T, BITS, NMAT, 64>(x, x_rows, mats, a, tiles_max, st);
    if (ntok == 128) return tcvp_launch_t<T, BITS, NMAT, 128>(x, x_rows, mats, a, tiles_max, st);
    if constexpr (NMAT == 1) {
        if (ntok == 256) return tcvp_launch_t<T, BITS, NMAT, 256>(x, x_rows, mats, a, tiles_max, st);
    }
    return LQ_E_UNSUPPORTED;
}

static int tcvp_dispatch(const void* x, int x_rows, const QmvMats& mats, int nmat, const TcvArgs& a, int bits,
                         int dtype, int ntok, int tiles_max, cudaStream_t st) {
    const bool bf16 = dtype == LQ_BF16;
    if (bits == 4) {
        if (nmat == 1)
            return bf16 ? tcvp_dispatch_tok<__nv_bfloat16, 4, 1>(ntok, x, x_rows, mats, a, tiles_max, st)
                        : tcvp_dispatch_tok<__half, 4, 1>(ntok, x, x_rows, mats, a, tiles_max, st);
        return bf16 ? tcvp_dispatch_tok<__nv_bfloat16, 4, 2>(ntok, x, x_rows, mats, a, tiles_max, st)
                    : tcvp_dispatch_tok<__half, 4, 2>(ntok, x, x_rows, mats, a, tiles_max, st);
    }
    if (nmat == 1)
        return bf16 ? tcvp_dispatch_tok<__nv_bfloat16, 8, 1>(ntok, x, x_rows, mats, a, tiles_max, st)
                    : tcvp_dispatch_tok<__half, 8, 1>(ntok, x, x_rows, mats, a, tiles_max, st);
    return bf16 ? tcvp_dispatch_tok<__nv_bfloat16, 8, 2>(ntok, x, x_rows, mats, a, tiles_max, st)
                : tcvp_dispatch_tok<__half, 8, 2>(ntok, x, x_rows, mats, a, tiles_max, st);
}

bool tcvp_shape_ok(int M, int K, int bits) {
    if (M < 1 || K < 128) return false;
    if (bits == 4) return K % 256 == 0;
    if (bits == 8) return K % 128 == 0;
    return false;
}

// Dense persistent call: token tiles of ntok (0 = 16/32/64 by M, 128 from 65 rows, 256 from 129 rows
// with one matrix).
int tcvp_run(const void* x, int M, const QmvMats& mats, int nmat, int N, int K, int nout, void* const* outs,
             const int* seg_end, const int* ldo, int bits, int dtype, int ntok, cudaStream_t st) {
    if (!tcvp_shape_ok(M, K, bits)) return LQ_E_SHAPE;
    TcvArgs a = {};
    a.M = M;
    a.N = N;
    a.K = K;
    a.G = K / 64;
    a.ks = 1;
    a.nseg_out = nout;
    for (int i = 0; i < nout; ++i) {
        a.out[i] = outs[i];
        a.seg_end[i] = seg_end[i];
        a.ldo[i] = ldo[i];
    }
    if (ntok == 0) ntok = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 || nmat == 2 ? 128 : 256;
    if (ntok != 16 && ntok != 32 && ntok != 64 && ntok != 128 && ntok != 256) return LQ_E_ARG;
    const int tiles = ((N + 127) / 128) * ((M + ntok - 1) / ntok);
    return tcvp_dispatch(x, M, mats, nmat, a, bits, dtype, ntok, tiles, st);
}

// Grouped persistent call (MoE experts): x = the expert-sorted rows (P), weights stacked (E, N, ...).
int tcvp_run_grouped(const void* xs, int P, const QmvMats& mats, int nmat, int N, int K, void* out,
                     const int32_t* starts, const int32_t* experts, const int32_t* nseg, int E, int bits, int dtype,
                     int ntok, cudaStream_t st) {
    if (!tcvp_shape_ok(P, K, bits)) return LQ_E_SHAPE;
    if (E + 1 > TCVP_MAX_SEGS - 1) return LQ_E_SHAPE;
    TcvArgs a = {};
    a.M = P;
    a.N = N;
    a.K = K;
    a.G = K / 64;
    a.ks = 1;
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
    if (ntok == 0) ntok = expect >= 24 ? 64 : expect >= 12 ? 32 : 16;
    if (ntok != 16 && ntok != 32 && ntok != 64) return LQ_E_ARG;
    const int tiles = ((N + 127) / 128) * (used + (P + ntok - 1) / ntok);
    return tcvp_dispatch(xs, P, mats, nmat, a, bits, dtype, ntok, tiles, st);
}

}  // namespace lq
