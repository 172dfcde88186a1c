// Grouped expert projections in the folded form ("qmvqg"): the decode-size MoE expert GEMMs (a few tokens an expert)
// with the codes fed raw to mma.sync and each group's scale and bias folded in fp32, as in qmvq.cu, over every SM.
//
// The work: after the expert grouping (counting sort of the (token, slot) pairs, locals/moe_kernel.py:28-66), segment
// s holds rows [starts[s], starts[s+1]) of the pairs, all routed to expert experts[s]. A work item is one segment and
// one chunk of FR 16-row fragments of that expert's matrix (or of its gate and up matrices, SwiGLU epilogue); the CTAs
// (one an SM) take items c, c + grid, ... and stream each item's weights through one ring of stages that runs on from
// item to item, so every SM keeps streaming while the per-expert row counts stay tiny (1-2 at 16 tokens over 64
// experts). Inside an item the split is qmvq's: warp w takes group w of every 512-wide stage for all FR fragments, the
// x rows are the segment's tokens (fetched straight into registers, through the grouping's order for the gate/up
// projection), the eight warps' sums meet in a shared-memory table (its own region: the ring is busy with the next
// item) and the item's rows are stored in expert order, as the grouped mma kernels store them.
// Reference: moe_kernel._launch / switch_glu (locals/moe_kernel.py:68-155,206-239) and moe.experts_up / experts_down
// (locals/moe.py:243-349,442-512), the fold of locals/qmv_frag.py:368-540.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"

namespace lq {

constexpr int QG2_CW = 8;
constexpr int QG2_THREADS = 32 * (QG2_CW + 1);
constexpr int QG2_MAX_STAGES = 8;

template <int BITS, int MT, int FR, int NMAT>
struct Qg2Shape {
    static constexpr int MTOK = 8 * MT;
    static constexpr int RB = BITS * 64;             // bytes of a row a stage (512 K values)
    static constexpr int SEGS = RB / 128;
    static constexpr int W_FRAG = 16 * RB;
    static constexpr int W_MAT = FR * W_FRAG;
    static constexpr int W_BYTES = NMAT * W_MAT;
    static constexpr int SB_MAT = FR * 16 * 16;
    static constexpr int STAGE_BYTES = (W_BYTES + NMAT * 2 * SB_MAT + 1023) / 1024 * 1024;
    static constexpr int RRP = NMAT * FR * 16 + 4;   // padded row stride of the warps' sums (see qmvq.cu)
    static constexpr int RED_BYTES = (QG2_CW * MTOK * RRP * 4 + 1023) / 1024 * 1024;
};

struct Qg2Args {
    int N, K;          // N: rows of each expert matrix
    int E;             // experts (segments of expert E are the grouping's padding bucket: skipped)
    int kg, nchunk;    // groups a row, stages of 512 K values
    int chunks_e;      // items an expert segment: (N / 16) / FR
    int ns, sb_vec;
    const int32_t* starts;
    const int32_t* experts;
    const int32_t* nseg;
    const int32_t* gather;  // null: segment row j is x row j; else x row gather[j] / gather_k (the pairs' tokens)
    int gather_k;
    const void* x;
    const void* s[2];
    const void* b[2];
    void* out;  // (P, N) rows in the grouping's order
};

template <typename T>
struct Qg2Magic;
template <>
struct Qg2Magic<__nv_bfloat16> {
    static constexpr uint32_t kCode2 = 0x43004300u, kOne2 = 0x3F803F80u;
    static constexpr float kVal = 128.0f;
};
template <>
struct Qg2Magic<__half> {
    static constexpr uint32_t kCode2 = 0x64006400u, kOne2 = 0x3C003C00u;
    static constexpr float kVal = 1024.0f;
};

template <typename T>
__device__ __forceinline__ void qg2_mma(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 qg2_lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 qg2_lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

template <typename T>
__device__ __forceinline__ float qg2_round(float v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __bfloat162float(__float2bfloat16_rn(v));
    else
        return __half2float(__float2half_rn(v));
}

// silu(g) * u with the activation-dtype rounding points of locals/moe.py:284-289 (the store rounds the product)
template <typename T>
__device__ __forceinline__ float qg2_swiglu(float g, float u) {
    const float gt = qg2_round<T>(g), ut = qg2_round<T>(u);
    const float sig = qg2_round<T>(1.0f / (1.0f + expf(-gt)));
    return qg2_round<T>(gt * sig) * ut;
}

// The item's expert and rows, or false for an item nobody asked for (the padding bucket) or a bad segment.
__device__ __forceinline__ bool qg2_item(const Qg2Args& a, int it, int mtok, int* e, int* row0, int* rows, int* ch) {
    const int s = it / a.chunks_e;
    *ch = it - s * a.chunks_e;
    *e = a.experts[s];
    *row0 = a.starts[s];
    *rows = a.starts[s + 1] - *row0;
    if (*e == a.E) return false;
    if (*e < 0 || *e > a.E || *rows < 0 || *rows > mtok) {
        record_status(LQ_DEV_BOUNDS);
        return false;
    }
    return *rows > 0;
}

template <typename T, int BITS, int MT, int FR, int NMAT>
__global__ void __launch_bounds__(QG2_THREADS, 1)
    qmvqg_kernel(const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1, const Qg2Args a) {
    using S = Qg2Shape<BITS, MT, FR, NMAT>;
    using TR = F16Traits<T>;
    using MG = Qg2Magic<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr float kFold = BITS == 4 ? MG::kVal : 17.0f * MG::kVal;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int ns = a.ns;
    float* red = reinterpret_cast<float*>(smem + ns * S::STAGE_BYTES);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ns * S::STAGE_BYTES + S::RED_BYTES);
    uint64_t* empty = full + QG2_MAX_STAGES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; ++s) {
            mbar_init(&full[s], 1 + 32);
            mbar_init(&empty[s], QG2_CW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    grid_dep_wait();  // the segments (and the expert ids that pick the weights) come from the grouping kernel
    const int n_items = a.nseg[0] * a.chunks_e;
    bool ok = true;

    if (warp == QG2_CW) {
        // ------------------------------ producer warp ------------------------------
        const uint64_t pol_w = policy_evict_first();
        if (lane == 0) {
            prefetch_tmap(&tm0);
            if (NMAT == 2) prefetch_tmap(&tm1);
        }
        const uint32_t smem_base = smem_u32(smem);
        const int vb = a.sb_vec;
        const int units = 16 / vb;
        int gs = 0;  // stages issued so far (the ring's running count)
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            int e, row0, rows, ch;
            if (!qg2_item(a, it, S::MTOK, &e, &row0, &rows, &ch)) continue;
            const int wrow = e * a.N + ch * FR * 16;
            for (int c = 0; c < a.nchunk; ++c, ++gs) {
                const int s = gs % ns;
                if (gs >= ns) {
                    ok = mbar_wait(&empty[s], ((gs / ns) - 1) & 1);
                    if (!ok) break;
                }
                uint8_t* st = smem + s * S::STAGE_BYTES;
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], NMAT * FR * S::W_FRAG);
                    tma_load_3d(st, &tm0, &full[s], 0, wrow, S::SEGS * c, pol_w);
                    if (NMAT == 2) tma_load_3d(st + S::W_MAT, &tm1, &full[s], 0, wrow, S::SEGS * c, pol_w);
                }
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint32_t sdst = smem_base + s * S::STAGE_BYTES + S::W_BYTES + m * 2 * S::SB_MAT;
                    for (int r = lane; r < FR * 16; r += 32) {
                        const int grow = wrow + r;
                        for (int u = 0; u < units; ++u) {
                            const int gcol = 8 * c + u * (vb >> 1);
                            const bool valid = gcol < a.kg;
                            const size_t off = valid ? (size_t(grow) * a.kg + gcol) * 2 : 0;
                            const uint32_t d = sdst + r * 16 + u * vb;
                            cp_async(d, reinterpret_cast<const uint8_t*>(a.s[m]) + off, vb, valid);
                            cp_async(d + S::SB_MAT, reinterpret_cast<const uint8_t*>(a.b[m]) + off, vb, valid);
                        }
                    }
                }
                cp_async_arrive(&full[s]);
            }
        }
        __syncwarp();
        return;
    }

    // ------------------------------ consumer warps ------------------------------
    const int g = lane >> 2, t = lane & 3;
    const uint32_t smem_base = smem_u32(smem);
    const int r_lo = BITS == 4 ? g : ((g >> 1) | ((g & 1) << 2));
    const uint32_t w_off = BITS == 4
                               ? (warp >> 2) * (FR * 2048) + r_lo * 128 + (((2 * (warp & 3) + (t >> 1)) ^ r_lo) << 4) +
                                     8 * (t & 1)
                               : (warp >> 1) * (FR * 2048) + r_lo * 128 + (((4 * (warp & 1) + t) ^ r_lo) << 4);
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(a.x);
    int gs = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
        int e, row0, rows, ch;
        if (!qg2_item(a, it, S::MTOK, &e, &row0, &rows, &ch)) continue;
        // this lane's token rows of x (token g + 8 mt of the segment); past the segment's rows the registers keep
        // what they held: an MMA's output column depends on its own input column only, and those are never stored
        const bool two = MT > 1 && rows > 8;  // a second token tile only for segments past 8 rows (warp-uniform)
        size_t xrow[MT];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int j = 8 * mt + g;
            int r = row0 + (j < rows ? j : 0);
            if (a.gather) r = a.gather[r] / a.gather_k;
            xrow[mt] = size_t(r) * a.K;
        }
        auto fetch_x = [&](int c, uint4 (&u)[MT][2]) {
            const int gi = 8 * c + warp;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                if (8 * mt + g < rows && gi < a.kg) {
                    const uint4* p = reinterpret_cast<const uint4*>(xg + (xrow[mt] + gi * 64 + 16 * t) * 2);
                    u[mt][0] = p[0];
                    u[mt][1] = p[1];
                }
        };
        float acc[NMAT][FR][MT][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int f = 0; f < FR; ++f)
#pragma unroll
                for (int q = 0; q < MT; ++q)
#pragma unroll
                    for (int ee = 0; ee < 4; ++ee) acc[m][f][q][ee] = 0.0f;
        uint4 xc[MT][2], xn[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) xc[mt][h] = xn[mt][h] = make_uint4(0u, 0u, 0u, 0u);
        fetch_x(0, xc);
        for (int c = 0; c < a.nchunk; ++c, ++gs) {
            const int s = gs % ns;
            if (c + 1 < a.nchunk) fetch_x(c + 1, xn);
            if (ok) ok = mbar_wait(&full[s], (gs / ns) & 1);
            if (ok && 8 * c + warp < a.kg) {
                const uint32_t st = smem_base + s * S::STAGE_BYTES;
                uint32_t xb[MT][4][2];
                float sx[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint32_t xw[8] = {xc[mt][0].x, xc[mt][0].y, xc[mt][0].z, xc[mt][0].w,
                                            xc[mt][1].x, xc[mt][1].y, xc[mt][1].z, xc[mt][1].w};
#pragma unroll
                    for (int step = 0; step < 4; ++step) {
                        const int wa = BITS == 4 ? (step >> 1) * 4 + (step & 1) : 2 * step;
                        const int wb = BITS == 4 ? wa + 2 : wa + 1;
                        xb[mt][step][0] = prmt(xw[wa], xw[wb], 0x5410);
                        xb[mt][step][1] = prmt(xw[wa], xw[wb], 0x7632);
                    }
#pragma unroll
                    for (int ee = 0; ee < 4; ++ee) sx[mt][ee] = 0.0f;
                    if (mt == 0 || two)
#pragma unroll
                        for (int step = 0; step < 4; ++step)
                            qg2_mma<T>(sx[mt], MG::kOne2, MG::kOne2, MG::kOne2, MG::kOne2, xb[mt][step][0],
                                       xb[mt][step][1]);
                }
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint32_t sb = st + S::W_BYTES + m * 2 * S::SB_MAT + 2 * warp;
#pragma unroll
                    for (int f = 0; f < FR; ++f) {
                        const uint32_t fb = st + m * S::W_MAT + f * 2048 + w_off;
                        const int ra = 16 * f + r_lo, rb = ra + 8;
                        const float sa = TR::to_f32(lds_u16(sb + ra * 16)), sbb = TR::to_f32(lds_u16(sb + rb * 16));
                        const float ca = fmaf(-kFold, sa, TR::to_f32(lds_u16(sb + S::SB_MAT + ra * 16)));
                        const float cb = fmaf(-kFold, sbb, TR::to_f32(lds_u16(sb + S::SB_MAT + rb * 16)));
                        float part[MT][4];
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int ee = 0; ee < 4; ++ee) part[mt][ee] = 0.0f;
                        if constexpr (BITS == 4) {
                            const uint2 wa = qg2_lds64(fb), wb = qg2_lds64(fb + 8 * 128);
#pragma unroll
                            for (int step = 0; step < 4; ++step) {
                                const uint32_t va = step < 2 ? wa.x : wa.y, vbw = step < 2 ? wb.x : wb.y;
                                const int sh = 8 * (step & 1);
                                const uint32_t a0 = lop3_and_or(va >> sh, 0x000F000Fu, MG::kCode2);
                                const uint32_t a2 = lop3_and_or(va >> (sh + 4), 0x000F000Fu, MG::kCode2);
                                const uint32_t a1 = lop3_and_or(vbw >> sh, 0x000F000Fu, MG::kCode2);
                                const uint32_t a3 = lop3_and_or(vbw >> (sh + 4), 0x000F000Fu, MG::kCode2);
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt)
                                    if (mt == 0 || two) qg2_mma<T>(part[mt], a0, a1, a2, a3, xb[mt][step][0], xb[mt][step][1]);
                            }
                        } else {
                            const uint4 wa = qg2_lds128(fb), wb = qg2_lds128(fb + 8 * 128);
                            const uint32_t va4[4] = {wa.x, wa.y, wa.z, wa.w}, vb4[4] = {wb.x, wb.y, wb.z, wb.w};
                            float hi[MT][4];
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                for (int ee = 0; ee < 4; ++ee) hi[mt][ee] = 0.0f;
#pragma unroll
                            for (int step = 0; step < 4; ++step) {
                                const uint32_t va = va4[step], vbw = vb4[step];
                                const uint32_t l0 = lop3_and_or(va, 0x000F000Fu, MG::kCode2);
                                const uint32_t l2 = lop3_and_or(va >> 8, 0x000F000Fu, MG::kCode2);
                                const uint32_t l1 = lop3_and_or(vbw, 0x000F000Fu, MG::kCode2);
                                const uint32_t l3 = lop3_and_or(vbw >> 8, 0x000F000Fu, MG::kCode2);
                                const uint32_t h0 = lop3_and_or(va >> 4, 0x000F000Fu, MG::kCode2);
                                const uint32_t h2 = lop3_and_or(va >> 12, 0x000F000Fu, MG::kCode2);
                                const uint32_t h1 = lop3_and_or(vbw >> 4, 0x000F000Fu, MG::kCode2);
                                const uint32_t h3 = lop3_and_or(vbw >> 12, 0x000F000Fu, MG::kCode2);
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt)
                                    if (mt == 0 || two) {
                                        qg2_mma<T>(part[mt], l0, l1, l2, l3, xb[mt][step][0], xb[mt][step][1]);
                                        qg2_mma<T>(hi[mt], h0, h1, h2, h3, xb[mt][step][0], xb[mt][step][1]);
                                    }
                            }
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                for (int ee = 0; ee < 4; ++ee) part[mt][ee] = fmaf(16.0f, hi[mt][ee], part[mt][ee]);
                        }
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            acc[m][f][mt][0] = fmaf(sa, part[mt][0], fmaf(ca, sx[mt][0], acc[m][f][mt][0]));
                            acc[m][f][mt][1] = fmaf(sa, part[mt][1], fmaf(ca, sx[mt][1], acc[m][f][mt][1]));
                            acc[m][f][mt][2] = fmaf(sbb, part[mt][2], fmaf(cb, sx[mt][0], acc[m][f][mt][2]));
                            acc[m][f][mt][3] = fmaf(sbb, part[mt][3], fmaf(cb, sx[mt][1], acc[m][f][mt][3]));
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                xc[mt][0] = xn[mt][0];
                xc[mt][1] = xn[mt][1];
            }
        }

        // the eight warps' sums of this item (a table of its own: the ring is streaming the next item)
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int f = 0; f < FR; ++f)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int ee = 0; ee < 4; ++ee) {
                        const int row = (m * FR + f) * 16 + r_lo + 8 * (ee >> 1), tok = 8 * mt + 2 * t + (ee & 1);
                        red[(warp * S::MTOK + tok) * S::RRP + row] = acc[m][f][mt][ee];
                    }
        named_barrier(1, 32 * QG2_CW);
        auto sum_warps = [&](int tok, int row) {
            float p[QG2_CW];
#pragma unroll
            for (int w = 0; w < QG2_CW; ++w) p[w] = red[(w * S::MTOK + tok) * S::RRP + row];
            return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
        };
        constexpr int R = FR * 16;
        for (int idx = threadIdx.x; idx < R * rows; idx += 32 * QG2_CW) {
            const int tok = idx / R, row = idx - tok * R;
            float v;
            if constexpr (NMAT == 2)
                v = qg2_swiglu<T>(sum_warps(tok, row), sum_warps(tok, FR * 16 + row));
            else
                v = sum_warps(tok, row);
            const size_t off = size_t(row0 + tok) * a.N + size_t(ch) * R + row;
            if (ok) {
                if (kBF16)
                    reinterpret_cast<__nv_bfloat16*>(a.out)[off] = __float2bfloat16_rn(v);
                else
                    reinterpret_cast<__half*>(a.out)[off] = __float2half_rn(v);
            }
        }
        named_barrier(1, 32 * QG2_CW);  // (the table is rewritten by the next item)
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------

template <typename T, int BITS, int MT, int FR, int NMAT>
static int qmvqg_launch_t(const uint32_t* const* w, Qg2Args a, int P, cudaStream_t st) {
    using S = Qg2Shape<BITS, MT, FR, NMAT>;
    const DeviceInfo& di = device_info();
    const size_t fixed = S::RED_BYTES + 2 * QG2_MAX_STAGES * 8 + 1024;
    int ns = di.smem_optin > fixed ? int((di.smem_optin - fixed) / S::STAGE_BYTES) : 0;
    if (ns > QG2_MAX_STAGES) ns = QG2_MAX_STAGES;
    if (ns < 2) return LQ_E_SHAPE;
    a.ns = ns;
    const size_t smem = fixed + size_t(ns) * S::STAGE_BYTES;
    a.chunks_e = (a.N / 16) / FR;
    CUtensorMap tw[2];
    for (int m = 0; m < 2; ++m) {
        const uint64_t dims[3] = {32, uint64_t(a.E) * a.N, uint64_t(a.K) * BITS / 1024};
        const uint64_t str[2] = {uint64_t(a.K) * BITS / 8, 128};
        const uint32_t box[3] = {32, uint32_t(FR * 16), uint32_t(S::SEGS)};
        const int rc = make_tmap(&tw[m], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, w[m < NMAT ? m : 0], dims, str, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    uintptr_t sb_addr = 0;
    for (int m = 0; m < NMAT; ++m)
        sb_addr |= reinterpret_cast<uintptr_t>(a.s[m]) | reinterpret_cast<uintptr_t>(a.b[m]);
    a.sb_vec = (a.kg % 8 == 0 && sb_addr % 16 == 0) ? 16 : (a.kg % 4 == 0 && sb_addr % 8 == 0) ? 8 : 4;
    auto kern = qmvqg_kernel<T, BITS, MT, FR, NMAT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    // items: at most (segments) x chunks_e; the segments are not known on the host (they come from the grouping
    // kernel), so the grid covers every SM and each CTA walks its share of whatever items there are
    const int segs_max = (a.E + 1) < P ? (a.E + 1) : P;
    const long items_max = long(segs_max) * a.chunks_e;
    const int grid = items_max < di.sm_count ? int(items_max) : di.sm_count;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(QG2_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, tw[0], tw[1], a);
    return e == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

template <typename T, int BITS, int MT, int NMAT>
static int qmvqg_dispatch_fr(int FR, const uint32_t* const* w, const Qg2Args& a, int P, cudaStream_t st) {
    switch (FR) {
        case 1: return qmvqg_launch_t<T, BITS, MT, 1, NMAT>(w, a, P, st);
        case 2: return qmvqg_launch_t<T, BITS, MT, 2, NMAT>(w, a, P, st);
        case 3: return qmvqg_launch_t<T, BITS, MT, 3, NMAT>(w, a, P, st);
        case 4: return qmvqg_launch_t<T, BITS, MT, 4, NMAT>(w, a, P, st);
        case 8:
            if constexpr (NMAT == 1) return qmvqg_launch_t<T, BITS, MT, 8, NMAT>(w, a, P, st);
            return LQ_E_SHAPE;
        default: return LQ_E_SHAPE;
    }
}

template <typename T, int NMAT>
static int qmvqg_dispatch(int bits, int MT, int FR, const uint32_t* const* w, const Qg2Args& a, int P,
                          cudaStream_t st) {
    if (bits == 4)
        return MT == 1 ? qmvqg_dispatch_fr<T, 4, 1, NMAT>(FR, w, a, P, st) : qmvqg_dispatch_fr<T, 4, 2, NMAT>(FR, w, a, P, st);
    return MT == 1 ? qmvqg_dispatch_fr<T, 8, 1, NMAT>(FR, w, a, P, st) : qmvqg_dispatch_fr<T, 8, 2, NMAT>(FR, w, a, P, st);
}

// Whether the grouped folded kernel takes a call: every segment at most 16 rows (max_rows), K % 256 == 0, and N a
// multiple of 16 fragments a chunk can divide.
bool qmvqg_shape_ok(int max_rows, int N, int K, int bits) {
    return (bits == 4 || bits == 8) && max_rows >= 1 && max_rows <= 16 && K >= 256 && K % 256 == 0 && N >= 16 &&
           N % 16 == 0;
}

// Segments of the grouping (starts / experts / nseg, the padding bucket E skipped) through the experts' (E, N, K)
// matrices: out (P, N) in the grouping's row order; glu: out = swiglu(gate, up). x rows: gather ? x[gather[j] / k]
// : xs[j]. max_rows bounds the rows of one segment (<= 16; a longer one records LQ_DEV_BOUNDS and is skipped).
int qmvqg_run(const void* x, const int32_t* gather, int gather_k, const int32_t* starts, const int32_t* experts,
              const int32_t* nseg, int P, int max_rows, int glu, const uint32_t* w0, const void* s0, const void* b0,
              const uint32_t* w1, const void* s1, const void* b1, void* out, int E, int N, int K, int bits, int dtype,
              cudaStream_t st) {
    if (!qmvqg_shape_ok(max_rows, N, K, bits)) return LQ_E_SHAPE;
    Qg2Args a = {};
    a.N = N;
    a.K = K;
    a.E = E;
    a.kg = K / 64;
    a.nchunk = (K + 511) / 512;
    a.starts = starts;
    a.experts = experts;
    a.nseg = nseg;
    a.gather = gather;
    a.gather_k = gather_k;
    a.x = x;
    a.s[0] = s0;
    a.b[0] = b0;
    a.s[1] = glu ? s1 : s0;
    a.b[1] = glu ? b1 : b0;
    a.out = out;
    const uint32_t* w[2] = {w0, glu ? w1 : w0};
    const int units = N / 16;
    // fragments an item: the most that divide the expert's fragments (up to 8 for one matrix, 4 for a gate/up pair):
    // larger items spread the per-item reduction over more weights
    int FR = 1;
    const int frs[5] = {8, 4, 3, 2, 1};
    for (int f : frs)
        if ((f <= 4 || !glu) && units % f == 0) {
            FR = f;
            break;
        }
    const int MT = max_rows <= 8 ? 1 : 2;
    const bool bf16 = dtype == LQ_BF16;
    if (glu)
        return bf16 ? qmvqg_dispatch<__nv_bfloat16, 2>(bits, MT, FR, w, a, P, st)
                    : qmvqg_dispatch<__half, 2>(bits, MT, FR, w, a, P, st);
    return bf16 ? qmvqg_dispatch<__nv_bfloat16, 1>(bits, MT, FR, w, a, P, st)
                : qmvqg_dispatch<__half, 1>(bits, MT, FR, w, a, P, st);
}

}  // namespace lq
