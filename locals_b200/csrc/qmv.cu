// Decode-size quantized matmul ("qmv" family): y (M, N) = x (M, K) . dequant(W)^T for few rows,
// dense or grouped by expert.
//
// HBM-bound design for sm_100a:
//  * One producer warp per CTA streams the CTA's K-range through a ring of shared-memory stages.
//    Lane 0 issues TMA (cp.async.bulk.tensor, no multicast) for the packed weight words (3-D boxes
//    [128-byte segment][BN rows][K segments], 128-byte swizzle, L2 evict-first: each byte is used
//    once) and for x (3-D swizzled boxes, L2 evict-last: every CTA reads it). All 32 lanes fetch the
//    16-bit scales and biases with cp.async (their rows are K/32 bytes, not always 16-byte aligned)
//    and zero-fill groups past K.
//  * Dense calls issue the weight loads of the first stages BEFORE griddepcontrol.wait: with
//    programmatic dependent launch they overlap the previous kernel's tail; only x waits.
//  * Four consumer warps each own 16*R output rows. A lane loads one 16-byte chunk of packed words
//    per row (conflict-free under the swizzle thanks to the row permutation pi_row) and dequantizes
//    code pairs straight into mma.sync m16n8k16 A-fragments (one shift, one lop3 with the 16-bit
//    float "magic" exponent -- 128 + q in bf16, 1024 + q in fp16 -- one subtract, one fma with the
//    group's scale and bias: the weight rounded once to the activation dtype, as mx.dequantize
//    rounds it). Tokens sit on the MMA's n = 8 side (Y^T = W X^T, the idea of the reference's
//    locals/qmv_frag.py:1-19); x pairs are permuted with prmt to match the code order.
//  * Split-K across a thread-block cluster along y: each CTA of the cluster takes a slice of K and the
//    partial tiles are summed through distributed shared memory (no global scratch, no atomics).
//  * Grouped mode (MoE experts, locals/moe_kernel.py:68-155): blockIdx.z is a segment of the
//    expert-sorted pairs; the weights are expert experts[s]'s rows of the stacked (E*N, ...) arrays and
//    x / out rows are the segment's rows [starts[s], starts[s+1]) of pair-ordered buffers. A segment
//    longer than the token tile is handled by a loop that streams the weights again.
//  * Epilogues: plain store, a column-split store (fused q/k/v outputs) or the SwiGLU of two matrices
//    (gate/up) with the rounding points of locals/moe.py:284-289.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"
#include "qmv.h"

namespace lq {

constexpr int QMV_CW = 8;  // consumer warps
constexpr int QMV_THREADS = 32 * (QMV_CW + 1);
constexpr int QMV_MAX_STAGES = 8;

// Tile geometry. A stage holds 256 bytes of packed words per weight row (512 K values at 4 bits, 256 at
// 8 bits): two 128-byte swizzle segments. Each consumer warp owns one 16-row MMA fragment; WK warps
// share a fragment and split each stage's four 64-byte iterations between them (K split inside the CTA,
// summed through shared memory at the end), so a CTA has 8 / WK fragments = BN rows.
template <typename T, int BITS, int MT, int WK, int NMAT>
struct QmvShape {
    static constexpr int RF = QMV_CW / WK;              // row fragments per CTA
    static constexpr int BN = 16 * RF;                  // rows of each matrix per CTA
    static constexpr int MTOK = 8 * MT;                 // token slots per pass
    static constexpr int BK = 2048 / BITS;              // K values per stage
    static constexpr int GPS = BK / 64;                 // groups per stage
    static constexpr int SBROW = GPS * 2;               // bytes per row of a scale (or bias) tile
    static constexpr int W_BYTES = BN * 256;            // one matrix
    static constexpr int SB_BYTES = BN * SBROW;         // one array of one matrix
    static constexpr int X_BYTES = MTOK * BK * 2;       // x slice: BK / 64 swizzled 64-value segments
    static constexpr int TMA_BYTES = NMAT * W_BYTES + X_BYTES;
    static constexpr int RAW_STAGE = NMAT * (W_BYTES + 2 * SB_BYTES) + X_BYTES;
    static constexpr int STAGE_BYTES = (RAW_STAGE + 1023) / 1024 * 1024;
    static constexpr int IT = 4;                        // 64-byte iterations per stage
    static constexpr int ITW = IT / WK;                 // iterations per warp per stage
    static constexpr int RED_BYTES = (WK - 1) * NMAT * BN * MTOK * 4;
    static constexpr int PART_BYTES = NMAT * BN * MTOK * 4;
    static_assert(W_BYTES % 1024 == 0 && X_BYTES % 1024 == 0, "1 KB alignment of swizzled tiles");
};

// Fragment row g of a 16-row MMA tile -> tile row. Rows 2i and 2i+1 of a quarter-warp differ in bit 2
// so their 16-byte chunks land in different halves of the 128-byte swizzle atom (no bank conflicts).
__device__ __forceinline__ int pi_row(int g) { return (g >> 1) | ((g & 1) << 2); }

template <typename T>
__device__ __forceinline__ float round_t(float v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __bfloat162float(__float2bfloat16_rn(v));
    else
        return __half2float(__float2half_rn(v));
}

// silu(g) * u with the activation-dtype rounding points of locals/moe.py:284-289.
template <typename T>
__device__ __forceinline__ float swiglu_t(float g, float u) {
    const float gt = round_t<T>(g), ut = round_t<T>(u);
    const float sig = round_t<T>(1.0f / (1.0f + expf(-gt)));
    const float act = round_t<T>(gt * sig);
    return act * ut;
}

__device__ __forceinline__ void store_out(const QmvArgs& a, int row, int n, float v, bool bf16) {
    int seg = 0, start = 0;
    if (a.nseg_out > 1 && n >= a.seg_end[0]) {
        seg = 1;
        start = a.seg_end[0];
        if (a.nseg_out > 2 && n >= a.seg_end[1]) {
            seg = 2;
            start = a.seg_end[1];
        }
    }
    const size_t off = size_t(row) * a.ldo[seg] + (n - start);
    if (bf16)
        reinterpret_cast<__nv_bfloat16*>(a.out[seg])[off] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<__half*>(a.out[seg])[off] = __float2half_rn(v);
}

// One 64-byte iteration of one warp: 16 rows x (128 K at 4 bits | 64 K at 8 bits) against MT token tiles.
template <typename T, int BITS, int MT, int WK, int NMAT>
__device__ __forceinline__ void qmv_iteration(float (&acc)[NMAT][MT][4], uint32_t st, int it, int ra, int g, int t) {
    using S = QmvShape<T, BITS, MT, WK, NMAT>;
    using TR = F16Traits<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    const int rb = ra + 8;
    const uint32_t xs = st + NMAT * S::W_BYTES;
    const uint32_t sbs = xs + S::X_BYTES;
    const int wseg = it >> 1;
    const int wchunk = 4 * (it & 1) + t;
    const int grp = (BITS == 4) ? (2 * it + (t >> 1)) : it;
    uint4 wa[NMAT], wb[NMAT];
    uint32_t s2a[NMAT], b2a[NMAT], s2b[NMAT], b2b[NMAT];
    float sfa[NMAT], bfa[NMAT], sfb[NMAT], bfb[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        const uint32_t wbase = st + m * S::W_BYTES + wseg * (S::BN * 128);
        wa[m] = lds128(wbase + ra * 128 + ((wchunk ^ (ra & 7)) << 4));
        wb[m] = lds128(wbase + rb * 128 + ((wchunk ^ (rb & 7)) << 4));
        const uint32_t sp = sbs + 2 * m * S::SB_BYTES;
        const uint32_t bp = sp + S::SB_BYTES;
        const uint32_t sa = lds_u16(sp + ra * S::SBROW + grp * 2), ba = lds_u16(bp + ra * S::SBROW + grp * 2);
        const uint32_t sb = lds_u16(sp + rb * S::SBROW + grp * 2), bb = lds_u16(bp + rb * S::SBROW + grp * 2);
        if constexpr (BITS == 8 && kBF16) {
            sfa[m] = TR::to_f32(sa);
            bfa[m] = TR::to_f32(ba);
            sfb[m] = TR::to_f32(sb);
            bfb[m] = TR::to_f32(bb);
        } else {
            s2a[m] = prmt(sa, sa, 0x1010);
            b2a[m] = prmt(ba, ba, 0x1010);
            s2b[m] = prmt(sb, sb, 0x1010);
            b2b[m] = prmt(bb, bb, 0x1010);
        }
    }
    if constexpr (BITS == 4) {
        const int xseg = 2 * it + (t >> 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t xp[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int tok = 8 * mt + g;
                const int xc = 4 * (t & 1) + j;
                const uint4 u = lds128(xs + xseg * (S::MTOK * 128) + tok * 128 + ((xc ^ (tok & 7)) << 4));
                xp[mt][0] = prmt(u.x, u.z, 0x5410);  // (x0, x4)
                xp[mt][1] = prmt(u.x, u.z, 0x7632);  // (x1, x5)
                xp[mt][2] = prmt(u.y, u.w, 0x5410);  // (x2, x6)
                xp[mt][3] = prmt(u.y, u.w, 0x7632);  // (x3, x7)
            }
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const uint32_t wva = (j == 0) ? wa[m].x : (j == 1) ? wa[m].y : (j == 2) ? wa[m].z : wa[m].w;
                const uint32_t wvb = (j == 0) ? wb[m].x : (j == 1) ? wb[m].y : (j == 2) ? wb[m].z : wb[m].w;
                uint32_t pa[4], pb[4];
#pragma unroll
                for (int p = 0; p < 4; ++p) {  // codes (p, p + 4) of the word
                    pa[p] = TR::sub_magic_fma(lop3_and_or(wva >> (4 * p), 0x000F000Fu, TR::kMagic2), s2a[m], b2a[m]);
                    pb[p] = TR::sub_magic_fma(lop3_and_or(wvb >> (4 * p), 0x000F000Fu, TR::kMagic2), s2b[m], b2b[m]);
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma_16816<T>(acc[m][mt], pa[0], pb[0], pa[1], pb[1], xp[mt][0], xp[mt][1]);
                    mma_16816<T>(acc[m][mt], pa[2], pb[2], pa[3], pb[3], xp[mt][2], xp[mt][3]);
                }
            }
        }
    } else {
        const int xseg = it;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            uint4 xu[MT];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int tok = 8 * mt + g;
                const int xc = 2 * t + jj;
                xu[mt] = lds128(xs + xseg * (S::MTOK * 128) + tok * 128 + ((xc ^ (tok & 7)) << 4));
            }
#pragma unroll
            for (int jh = 0; jh < 2; ++jh) {
                const int j = 2 * jj + jh;
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint32_t wva = (j == 0) ? wa[m].x : (j == 1) ? wa[m].y : (j == 2) ? wa[m].z : wa[m].w;
                    const uint32_t wvb = (j == 0) ? wb[m].x : (j == 1) ? wb[m].y : (j == 2) ? wb[m].z : wb[m].w;
                    uint32_t lo_a, hi_a, lo_b, hi_b;
                    if constexpr (kBF16) {
                        // a byte code as float: OR it into the mantissa of 2^23, subtract 2^23
                        float fa[4], fb[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            fa[q] = fmaf(__uint_as_float(prmt(wva, 0x4B000000u, 0x7540u + q)) - 8388608.0f, sfa[m],
                                         bfa[m]);
                            fb[q] = fmaf(__uint_as_float(prmt(wvb, 0x4B000000u, 0x7540u + q)) - 8388608.0f, sfb[m],
                                         bfb[m]);
                        }
                        lo_a = cvt_bf16x2(fa[1], fa[0]);
                        hi_a = cvt_bf16x2(fa[3], fa[2]);
                        lo_b = cvt_bf16x2(fb[1], fb[0]);
                        hi_b = cvt_bf16x2(fb[3], fb[2]);
                    } else {
                        lo_a = TR::sub_magic_fma(prmt(wva, 0x64646464u, 0x5140u), s2a[m], b2a[m]);
                        hi_a = TR::sub_magic_fma(prmt(wva, 0x64646464u, 0x5342u), s2a[m], b2a[m]);
                        lo_b = TR::sub_magic_fma(prmt(wvb, 0x64646464u, 0x5140u), s2b[m], b2b[m]);
                        hi_b = TR::sub_magic_fma(prmt(wvb, 0x64646464u, 0x5342u), s2b[m], b2b[m]);
                    }
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint32_t xlo = jh ? xu[mt].z : xu[mt].x;
                        const uint32_t xhi = jh ? xu[mt].w : xu[mt].y;
                        mma_16816<T>(acc[m][mt], lo_a, lo_b, hi_a, hi_b, xlo, xhi);
                    }
                }
            }
        }
    }
}

// DENSE: one token segment, no gather, no cluster -- the decode case, compiled without the grouped, gather and
// split-K paths so the hot loop's code stays small (instruction-cache misses were the top stall).
template <typename T, int BITS, int MT, int WK, int NMAT, bool DENSE>
__global__ void __launch_bounds__(QMV_THREADS, (MT * NMAT <= 2) ? 2 : 1)
    qmv_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
               const __grid_constant__ CUtensorMap tm_x, const QmvArgs a) {
    using S = QmvShape<T, BITS, MT, WK, NMAT>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    const bool grouped = !DENSE && a.grouped;
    const int kslices = DENSE ? 1 : a.ks;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int ns = a.ns;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ns * S::STAGE_BYTES);
    uint64_t* empty = full + QMV_MAX_STAGES;
    float* red = reinterpret_cast<float*>(smem + ns * S::STAGE_BYTES + 2 * QMV_MAX_STAGES * 8);
    float* part = red + S::RED_BYTES / 4;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * S::BN;
    const int krank = (kslices > 1) ? int(cluster_ctarank()) : 0;
    const int c_begin = (a.nchunk * krank) / a.ks;
    const int c_end = (a.nchunk * (krank + 1)) / a.ks;
    const int nloc = c_end - c_begin;

    // segment: dense calls have one, rows [0, M), weights at row 0
    int seg_row0 = 0, seg_rows = a.M, wrow0 = 0;
    if (grouped) {
        grid_dep_wait();  // starts / experts / nseg come from the grouping kernel
        const int sgi = blockIdx.z;
        if (sgi >= a.nseg[0]) return;  // the whole cluster shares blockIdx.z: it exits together
        seg_row0 = a.starts[sgi];
        seg_rows = a.starts[sgi + 1] - seg_row0;
        const int e = a.experts[sgi];
        if (e == a.n_experts) return;  // the padding bucket: rows nobody asked for, left unwritten
        if (e < 0 || e > a.n_experts || seg_rows < 0) {
            record_status(LQ_DEV_BOUNDS);
            return;
        }
        wrow0 = e * a.N;
    }
    int ntb = (seg_rows + S::MTOK - 1) / S::MTOK;
    if (kslices > 1 && ntb > 1) ntb = 1;  // (the host never launches split-K with longer segments)
    const int total = ntb * nloc;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; ++s) {
            mbar_init(&full[s], 1 + 32);  // lane 0's expect_tx arrive + 32 cp.async arrivals
            mbar_init(&empty[s], QMV_CW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    float acc[NMAT][MT][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int q = 0; q < MT; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][q][e] = 0.0f;
    bool ok = true;
    const int g = lane >> 2, t = lane & 3;
    const int rf = warp % S::RF, kq = warp / S::RF;
    const int ra = 16 * rf + pi_row(g);

    if (warp == QMV_CW) {
        // ------------------------------ producer warp ------------------------------
        const uint64_t pol_w = policy_evict_first();
        const uint64_t pol_x = policy_evict_last();
        if (lane == 0) {
            prefetch_tmap(&tm_w0);
            prefetch_tmap(&tm_x);
        }
        const CUtensorMap* tw[2] = {&tm_w0, &tm_w1};
        const uint32_t smem_base = smem_u32(smem);
        const int kg = a.K / 64;  // groups per row
        const int vb = a.sb_vec;  // bytes per cp.async
        const int units_row = S::SBROW / vb;
        const bool gather = !DENSE && a.gather != nullptr;
        // weights (TMA, lane 0) and scales/biases (cp.async, all lanes) of local chunk i into stage s
        auto load_weights = [&](int i, int s) {
            const uint32_t st = smem_base + s * S::STAGE_BYTES;
            const int c = c_begin + (i % nloc);
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], gather ? NMAT * S::W_BYTES : S::TMA_BYTES);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
                    tma_load_3d(smem + s * S::STAGE_BYTES + m * S::W_BYTES, tw[m], &full[s], 0,
                                wrow0 + n0 + a.row_off[m], c * 2, pol_w);
            }
            // scales and biases: per matrix 2 arrays x BN rows x SBROW bytes, lane-strided rows, no divisions
            const uint32_t sb_dst = st + NMAT * S::W_BYTES + S::X_BYTES;
            const int gcol0 = c * S::GPS;
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const int row0 = wrow0 + n0 + a.row_off[m];
                const uint8_t* sbase = reinterpret_cast<const uint8_t*>(a.sptr[m]);
                const uint8_t* bbase = reinterpret_cast<const uint8_t*>(a.bptr[m]);
#pragma unroll
                for (int rr = 0; rr < S::BN; rr += 32) {
                    const int r = rr + lane;
                    const int grow = row0 + r;
                    const bool row_ok = (r < S::BN) && grow < a.rows_total[m];
                    const size_t roff = size_t(grow) * kg;
                    for (int part_i = 0; part_i < units_row; ++part_i) {
                        const int gcol = gcol0 + part_i * (vb >> 1);
                        const bool valid = row_ok && gcol < kg;
                        const size_t off = valid ? (roff + gcol) * 2 : 0;
                        const uint32_t d = sb_dst + 2 * m * S::SB_BYTES + r * S::SBROW + part_i * vb;
                        if (r < S::BN) {
                            cp_async(d, sbase + off, vb, valid);
                            cp_async(d + S::SB_BYTES, bbase + off, vb, valid);
                        }
                    }
                }
            }
        };
        // x slice of local chunk i: one TMA box, or (gather) 16-byte cp.async per token row and chunk,
        // written in the same swizzled layout, zero-filled past the segment and past K
        auto load_x = [&](int i, int s) {
            const int tb = i / nloc, c = c_begin + (i % nloc);
            if (!gather) {
                if (lane == 0)
                    tma_load_3d(smem + s * S::STAGE_BYTES + NMAT * S::W_BYTES, &tm_x, &full[s], 0,
                                seg_row0 + tb * S::MTOK, c * (S::BK / 64), pol_x);
                return;
            }
            const uint32_t xdst = smem_base + s * S::STAGE_BYTES + NMAT * S::W_BYTES;
            constexpr int CPR = S::BK / 8;  // 16-byte chunks per token row
            const uint8_t* xb = reinterpret_cast<const uint8_t*>(a.x);
            for (int ci = lane; ci < S::MTOK * CPR; ci += 32) {
                const int tok = ci / CPR, cc = ci % CPR;
                const int seg = cc >> 3, ch = cc & 7;
                const int r = tb * S::MTOK + tok;
                if (r >= seg_rows) continue;  // (token slots past the segment: their outputs are never stored)
                const int kidx = c * S::BK + cc * 8;
                const bool valid = kidx < a.K;
                size_t off = 0;
                if (valid) off = (size_t(a.gather[seg_row0 + r] / a.gather_k) * a.K + kidx) * 2;
                cp_async(xdst + seg * (S::MTOK * 128) + tok * 128 + ((ch ^ (tok & 7)) << 4), xb + off, 16, valid);
            }
        };
        const int pre = total < ns ? total : ns;
        if (!grouped) {
            for (int i = 0; i < pre; ++i) {
                load_weights(i, i);
                cp_async_arrive(&full[i]);
            }
            grid_dep_wait();  // x may be the previous kernel's output
            for (int i = 0; i < pre; ++i) load_x(i, i);
        } else {  // (the grid dependency was resolved at entry: starts / experts come from the grouping)
            for (int i = 0; i < pre; ++i) {
                load_weights(i, i);
                load_x(i, i);
                cp_async_arrive(&full[i]);
            }
        }
        if (lane == 0) grid_dep_launch();
        for (int i = pre; i < total && ok; ++i) {
            const int s = i % ns;
            ok = mbar_wait(&empty[s], ((i / ns) - 1) & 1);
            if (!ok) break;
            load_weights(i, s);
            load_x(i, s);
            cp_async_arrive(&full[s]);
        }
        __syncwarp();
    } else {
        // ------------------------------ consumer warps ------------------------------
        const uint32_t smem_base = smem_u32(smem);
        if (!grouped) grid_dep_wait();  // (before any output store of this kernel)
        for (int i = 0; i < total; ++i) {
            const int s = i % ns;
            if (ok) ok = mbar_wait(&full[s], (i / ns) & 1);
            if (ok) {
                const uint32_t st = smem_base + s * S::STAGE_BYTES;
#pragma unroll
                for (int q = 0; q < S::ITW; ++q) qmv_iteration<T, BITS, MT, WK, NMAT>(acc, st, kq + WK * q, ra, g, t);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);

            if ((i % nloc) == nloc - 1) {
                // token block done: sum the K-split warps of each fragment
                if constexpr (WK > 1) {
                    if (kq > 0) {
#pragma unroll
                        for (int m = 0; m < NMAT; ++m)
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const int row = ra + 8 * (e >> 1), tok = 8 * mt + 2 * t + (e & 1);
                                    red[(((kq - 1) * NMAT + m) * S::MTOK + tok) * S::BN + row] = acc[m][mt][e];
                                }
                    }
                    named_barrier(1, 32 * QMV_CW);
                    if (kq == 0) {
#pragma unroll
                        for (int q = 1; q < WK; ++q)
#pragma unroll
                            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                    for (int e = 0; e < 4; ++e) {
                                        const int row = ra + 8 * (e >> 1), tok = 8 * mt + 2 * t + (e & 1);
                                        acc[m][mt][e] += red[(((q - 1) * NMAT + m) * S::MTOK + tok) * S::BN + row];
                                    }
                    }
                    named_barrier(1, 32 * QMV_CW);
                }
                if (kslices == 1 && kq == 0 && ok) {
                    const int tb = i / nloc;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int n = n0 + ra + 8 * h;
                        if (n >= a.N) continue;
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int tok = tb * S::MTOK + 8 * mt + 2 * t + e;
                                if (tok >= seg_rows) continue;
                                float v = acc[0][mt][2 * h + e];
                                if constexpr (NMAT == 2) v = swiglu_t<T>(v, acc[1][mt][2 * h + e]);
                                store_out(a, seg_row0 + tok, n, v, kBF16);
                            }
                        }
                    }
                }
                if (kslices == 1) {
#pragma unroll
                    for (int m = 0; m < NMAT; ++m)
#pragma unroll
                        for (int q = 0; q < MT; ++q)
#pragma unroll
                            for (int e = 0; e < 4; ++e) acc[m][q][e] = 0.0f;
                }
            }
        }
    }
    if (kslices == 1) return;

    // ------------------ split-K over the cluster (one token block) ------------------
    if (warp < QMV_CW && kq == 0) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int row = ra + 8 * (e >> 1), tok = 8 * mt + 2 * t + (e & 1);
                    part[(m * S::MTOK + tok) * S::BN + row] = ok ? acc[m][mt][e] : 0.0f;
                }
    }
    if (warp == QMV_CW && !grouped) grid_dep_wait();
    cluster_sync();
    const uint32_t part_local = smem_u32(part);
    uint32_t peer[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) peer[q] = q < a.ks ? map_peer(part_local, q) : part_local;
    constexpr int nout = S::BN * S::MTOK;
    for (int idx = krank * QMV_THREADS + threadIdx.x; idx < nout; idx += a.ks * QMV_THREADS) {
        const int tok = idx / S::BN, row = idx % S::BN;  // consecutive threads: consecutive output columns
        const int n = n0 + row;
        if (tok >= seg_rows || n >= a.N) continue;
        // every peer's partial is requested before any is summed (one round of remote latency)
        float v[16], u[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            v[q] = q < a.ks ? ld_dsmem_f(peer[q] + 4 * (tok * S::BN + row)) : 0.0f;
            if constexpr (NMAT == 2) u[q] = q < a.ks ? ld_dsmem_f(peer[q] + 4 * ((S::MTOK + tok) * S::BN + row)) : 0.0f;
        }
        float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            v0 += v[q];
            if constexpr (NMAT == 2) v1 += u[q];
        }
        if constexpr (NMAT == 2) v0 = swiglu_t<T>(v0, v1);
        store_out(a, seg_row0 + tok, n, v0, kBF16);
    }
    cluster_sync();  // peers keep their shared memory until every CTA has read it
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------

template <typename T, int BITS, int MT, int WK, int NMAT>
static int qmv_launch_t(const void* x, int x_rows, const QmvMats& mats, QmvArgs a, int ks, int ns_req, int n_seg_grid,
                        cudaStream_t st) {
    using S = QmvShape<T, BITS, MT, WK, NMAT>;
    const DeviceInfo& di = device_info();
    const int K = a.K;
    a.nchunk = (K + S::BK - 1) / S::BK;
    if (ks < 1) ks = 1;
    if (ks > a.nchunk) ks = a.nchunk;
    if (ks > 16) ks = 16;
    a.ks = ks;
    const int per_cta = (a.nchunk + ks - 1) / ks;
    // stages: as many as the CTA has chunks, within a budget that lets two CTAs share an SM
    const size_t fixed = 2 * QMV_MAX_STAGES * 8 + S::RED_BYTES + (ks > 1 ? S::PART_BYTES : 0) + 1024;
    size_t budget = di.smem_per_sm / 2 - 1024;
    if (fixed + S::STAGE_BYTES > budget) budget = di.smem_optin;
    int ns = int((budget - fixed) / S::STAGE_BYTES);
    if (ns < 1) return LQ_E_SHAPE;
    // a requested depth may use the whole SM's shared memory (one CTA an SM, more bytes in flight)
    if (ns_req > 0) ns = ns_req < int((di.smem_optin - fixed) / S::STAGE_BYTES) ? ns_req
                                                                               : int((di.smem_optin - fixed) / S::STAGE_BYTES);
    if (ns > QMV_MAX_STAGES) ns = QMV_MAX_STAGES;
    const int max_tb = a.grouped ? 64 : (a.M + S::MTOK - 1) / S::MTOK;
    if (ns > per_cta * max_tb) ns = per_cta * max_tb;
    a.ns = ns;
    const size_t smem = fixed + size_t(ns) * S::STAGE_BYTES;
    if (smem > di.smem_optin) return LQ_E_SHAPE;

    CUtensorMap tw[2], tx;
    for (int m = 0; m < NMAT; ++m) {
        const uint64_t rows = uint64_t(mats.rows_total[m]);
        const uint64_t wdims[3] = {32, rows, uint64_t(K) * BITS / 1024};
        const uint64_t wstr[2] = {uint64_t(K) * BITS / 8, 128};
        const uint32_t wbox[3] = {32, uint32_t(S::BN), 2};
        const int rc = make_tmap(&tw[m], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, mats.w[m], wdims, wstr, wbox,
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
        const uint64_t xdims[3] = {64, uint64_t(x_rows), uint64_t(K / 64)};
        const uint64_t xstr[2] = {uint64_t(K) * 2, 128};
        const uint32_t xbox[3] = {64, uint32_t(S::MTOK), uint32_t(S::BK / 64)};
        const int rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, x, xdims, xstr, xbox,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    const int kg = K / 64;
    a.sb_vec = (S::SBROW == 16 && kg % 8 == 0) ? 16 : (kg % 4 == 0) ? 8 : 4;
    a.x = x;

    const bool dense = !a.grouped && a.gather == nullptr && ks == 1;
    auto kern = dense ? qmv_kernel<T, BITS, MT, WK, NMAT, true> : qmv_kernel<T, BITS, MT, WK, NMAT, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    if (ks > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return LQ_E_CUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.N + S::BN - 1) / S::BN, ks, n_seg_grid);
    cfg.blockDim = dim3(QMV_THREADS, 1, 1);
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
static int qmv_dispatch_mt(int MT, int WK, const void* x, int x_rows, const QmvMats& mats, const QmvArgs& a, int ks,
                           int ns, int n_seg_grid, cudaStream_t st) {
#define LQ_QMV_CASE(mt, wk) \
    if (MT == mt && WK == wk) return qmv_launch_t<T, BITS, mt, wk, NMAT>(x, x_rows, mats, a, ks, ns, n_seg_grid, st);
    LQ_QMV_CASE(1, 1)
    LQ_QMV_CASE(1, 2)
    LQ_QMV_CASE(1, 4)
    LQ_QMV_CASE(2, 1)
    LQ_QMV_CASE(2, 2)
    LQ_QMV_CASE(2, 4)
    LQ_QMV_CASE(4, 1)
    LQ_QMV_CASE(4, 2)
    LQ_QMV_CASE(8, 1)
    LQ_QMV_CASE(8, 2)
#undef LQ_QMV_CASE
    return LQ_E_UNSUPPORTED;
}

// Default split-K for a grid of n_ctas row tiles: the largest factor that keeps the CTA count within
// 1.25 per SM (measured on B200: more CTAs than that only queue), preferring factors that split the K
// chunks evenly.
static int qmv_default_ks(int n_ctas, int nchunk, int sm_count) {
    int best = 1;
    double best_score = -1.0;
    const double cap = 1.25 * sm_count;
    for (int ks = 1; ks <= 8 && ks <= nchunk; ++ks) {
        const int ctas = n_ctas * ks;
        if (ks > 1 && ctas > cap) break;
        const int per = (nchunk + ks - 1) / ks;
        const double balance = double(nchunk) / (double(per) * ks);  // uneven K slices idle some CTAs
        const double score = double(ctas) * balance;
        if (score > best_score) {
            best_score = score;
            best = ks;
        }
    }
    return best;
}

bool qmv_shape_ok(int K, int bits) {
    if (K <= 0 || K % 64) return false;
    if (bits == 4) return K % 256 == 0;
    if (bits == 8) return K % 128 == 0;
    return false;
}

int qmv_run(const void* x, int x_rows, const QmvMats& mats, int nmat, QmvArgs a, int bits, int dtype, const int* p,
            int max_seg_rows, int n_seg_grid, cudaStream_t st) {
    int MT = p ? p[0] : 0, WK = p ? p[1] : 0, ks = p ? p[2] : 0, ns = p ? p[3] : 0;
    if (a.M < 1 || max_seg_rows < 1) return LQ_E_SHAPE;
    if (!qmv_shape_ok(a.K, bits)) return LQ_E_SHAPE;
    if (MT == 0) {
        int rows = max_seg_rows;
        if (a.grouped) {
            // rows per used expert, about P / min(E, P) (a token names an expert at most once); longer
            // segments take extra token blocks, which re-read their expert's weights from L2
            const int segs = a.n_experts < a.M ? a.n_experts : a.M;
            const int expect = (a.M + segs - 1) / segs;
            rows = expect * 2 < max_seg_rows ? expect * 2 : max_seg_rows;
        }
        MT = rows <= 8 ? 1 : rows <= 16 ? 2 : rows <= 32 ? 4 : 8;
    }
    if (MT != 1 && MT != 2 && MT != 4 && MT != 8) return LQ_E_ARG;
    const int nchunk = (a.K + (2048 / bits) - 1) / (2048 / bits);
    const int sms = device_info().sm_count;
    if (WK == 0) {
        // 64-row CTAs (two warps per 16-row fragment, each taking half of every stage): the measured best
        // for M <= 16 on B200, where the dequantizing warps, not the loads, bound the kernel
        WK = 2;
        if (MT >= 8) WK = 2;
    }
    const int bn = 16 * (8 / WK);
    const int single_block = max_seg_rows <= 8 * MT;
    if (ks == 0) ks = single_block ? qmv_default_ks(((a.N + bn - 1) / bn) * n_seg_grid, nchunk, sms) : 1;
    if (!single_block) ks = 1;
    const bool bf16 = dtype == LQ_BF16;
    if (bits == 4) {
        if (nmat == 1)
            return bf16 ? qmv_dispatch_mt<__nv_bfloat16, 4, 1>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st)
                        : qmv_dispatch_mt<__half, 4, 1>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st);
        return bf16 ? qmv_dispatch_mt<__nv_bfloat16, 4, 2>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st)
                    : qmv_dispatch_mt<__half, 4, 2>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st);
    }
    if (bits == 8) {
        if (nmat == 1)
            return bf16 ? qmv_dispatch_mt<__nv_bfloat16, 8, 1>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st)
                        : qmv_dispatch_mt<__half, 8, 1>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st);
        return bf16 ? qmv_dispatch_mt<__nv_bfloat16, 8, 2>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st)
                    : qmv_dispatch_mt<__half, 8, 2>(MT, WK, x, x_rows, mats, a, ks, ns, n_seg_grid, st);
    }
    return LQ_E_UNSUPPORTED;
}

}  // namespace lq
