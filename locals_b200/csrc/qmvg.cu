// Dense 4-bit decode, one 64-wide quantization group per warp ("qmvg" family): y (M, N) = x (M, K) . dequant(W)^T for
// M <= 16 tokens, the shape of the fused QKV projection and of every 4-bit decode projection.
//
// Why a second decode kernel. In the row-split qmv kernel each warp owns 16 weight rows and walks K, so every warp
// loads and permutes its own copy of each x slice and a CTA holds 64 rows, which leaves a third of the 148 SMs idle on
// the 6144-row QKV matrix. Here the work is split the other way:
//  * Rows: the N/16 row fragments are dealt out evenly over the CTAs (CTA c takes fragments [c*F/C, (c+1)*F/C)), so
//    the QKV matrix's 384 fragments run 2 or 3 to an SM on all 148 SMs. Every CTA holds FR or FR - 1 fragments.
//  * K: a ring stage holds 512 K values (8 groups) of all of the CTA's rows. Consumer warp w takes group w of every
//    stage for ALL the CTA's fragments: it loads and permutes its x fragments once (two 16-byte loads and 8 prmt a
//    token tile) and reuses them for every fragment. The eight warps' partial sums are added through shared memory
//    at the end (no global scratch, no atomics).
//  * x never passes through shared memory: each consumer warp loads the 32 bytes a lane needs of its own group
//    straight into registers (two 16-byte loads a token tile, one stage ahead of its use). Every CTA needs all of x
//    (80 KB at 16 tokens, more than its share of the weights), and measured on B200 one producer warp feeds an SM at
//    only ~20 GB/s, so x is spread over the 256 consumer lanes instead.
//  * A lane reads 8 bytes (16 codes) of a row per group, so all four lanes of an MMA k-slice hold codes of the same
//    group; codes are dequantized straight into m16n8k16 A fragments (magic exponent: 128 + q exact in bf16, 1024 + q
//    in fp16; one subtract and one fma with the group's scale and bias -- the weight rounded once to the activation
//    dtype, as mx.dequantize rounds it). Tokens sit on the MMA's n side (Y^T = W X^T, the idea of the reference's
//    locals/qmv_frag.py:1-19); lane t's codes (p, p + 4) of word 2t + (s >> 1) meet x values 16t + 8(s >> 1) + p,
//    + p + 4 of the same group, which is the permutation applied to x.
//  * One producer warp: one TMA box a stage for the packed words of all the CTA's rows ([128-byte segment][16 nf rows]
//    [2 segments], 128-byte swizzle, L2 evict-first; one box rather than one a fragment measured faster) and cp.async
//    for scales and biases (zero-filled past K and past N). Nothing it loads comes from the previous kernel, so under
//    programmatic dependent launch the whole ring fills while the previous kernel still runs; only the consumers'
//    x loads wait for the grid dependency.
// Reference: the multi-row GEMV it replaces, locals/qmv_multi.py:16-248 and locals/qmv_frag.py:34-540, behind
// kernels._launcher (locals/kernels.py:516-576).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"

namespace lq {

constexpr int QG_CW = 8;  // consumer warps: group w of every 8-group stage
constexpr int QG_THREADS = 32 * (QG_CW + 1);
constexpr int QG_MAX_STAGES = 6;
constexpr int QG_MAX_FR = 4;

template <int MT, int FR>
struct QgShape {
    static constexpr int MTOK = 8 * MT;                  // token slots
    static constexpr int W_FRAG = 16 * 256;              // one 16-row fragment: 256 bytes (512 codes) a row
    static constexpr int W_BYTES = FR * W_FRAG;
    static constexpr int SB_BYTES = FR * 16 * 16;        // scales (or biases): rows x 8 groups x 2 bytes
    static constexpr int STAGE_BYTES = (W_BYTES + 2 * SB_BYTES + 1023) / 1024 * 1024;
    static constexpr int RED_BYTES = QG_CW * MTOK * FR * 16 * 4;  // the warps' partial sums
    static_assert(W_FRAG % 1024 == 0, "1 KB alignment of swizzled tiles");
};

// MoE decode modes (one token, its k routed (token, slot) pairs; the segments of the expert grouping hold one pair
// each): MOE_GLU -- unit u = (segment u / fpe, fragment u % fpe) of the gate and up stacks of expert experts[seg],
// output h[seg] = swiglu(gate, up); MOE_COMBINE -- unit u = output fragment u of all k slots' down matrices (fragment
// r of a unit uses expert experts[r] and x row r = h[r], which sits in MMA token column r), output
// y = sum_r w[r] * round(y_r) in slot order (the combine of locals/moe.py:339-348 in the down kernel's epilogue).
constexpr int QG_DENSE = 0, QG_MOE_GLU = 1, QG_MOE_COMBINE = 2;

struct QgArgs {
    int M, N, K;
    int mode;             // QG_DENSE / QG_MOE_GLU / QG_MOE_COMBINE
    int fpu;              // fragments per unit (1 dense, 2 GLU, k combine)
    int units;            // units of the launch
    int fpe;              // MoE: fragments per expert matrix (rows per expert / 16)
    int rows_e;           // MoE: rows per expert matrix
    const int32_t* experts;  // MoE: expert of each segment (one pair a segment, in the grouping's order)
    const int32_t* pos;   // MOE_COMBINE: slot r's row of h (null: row r)
    const float* wts;     // MOE_COMBINE: the token's k slot weights
    const void* s1;       // MOE_GLU: the up stack's scales and biases
    const void* b1;
    int kg;      // groups a row (K / 64)
    int nchunk;  // stages of 512 K values
    int nfrag;   // 16-row fragments (ceil(N / 16))
    int ns;      // ring depth
    int sb_vec;  // cp.async width for scale / bias rows
    const void* x;
    const void* s;
    const void* b;
    void* out[3];  // output column segments (fused q / k / v), or out[0] only
    int seg_end[3];
    int ldo[3];
    int nseg_out;
};

__device__ __forceinline__ uint2 qg_lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// mma.sync m16n8k16 with fp32 accumulation, left to the compiler's scheduling (no side effects beyond its registers).
template <typename T>
__device__ __forceinline__ void qg_mma(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
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

// Output element (row, n) of the fused projection: segment chosen with constant indices (no local-memory copy of
// the argument arrays).
__device__ __forceinline__ void qg_store(const QgArgs& a, int row, int n, float v, bool bf16) {
    void* base = a.out[0];
    int start = 0, ld = a.ldo[0];
    if (a.nseg_out > 1 && n >= a.seg_end[0]) {
        const bool third = a.nseg_out > 2 && n >= a.seg_end[1];
        base = third ? a.out[2] : a.out[1];
        start = third ? a.seg_end[1] : a.seg_end[0];
        ld = third ? a.ldo[2] : a.ldo[1];
    }
    const size_t off = size_t(row) * ld + (n - start);
    if (bf16)
        reinterpret_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<__half*>(base)[off] = __float2half_rn(v);
}

template <typename T>
__device__ __forceinline__ float qg_round(float v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __bfloat162float(__float2bfloat16_rn(v));
    else
        return __half2float(__float2half_rn(v));
}

// silu(g) * u with the activation-dtype rounding points of locals/moe.py:284-289 (the store rounds the product)
template <typename T>
__device__ __forceinline__ float qg_swiglu(float g, float u) {
    const float gt = qg_round<T>(g), ut = qg_round<T>(u);
    const float sig = qg_round<T>(1.0f / (1.0f + expf(-gt)));
    return qg_round<T>(gt * sig) * ut;
}

template <typename T, int MT, int FR>
__global__ void __launch_bounds__(QG_THREADS, 2)
    qmvg_kernel(const __grid_constant__ CUtensorMap tm_w_full, const __grid_constant__ CUtensorMap tm_w_less,
                const QgArgs a) {
    using S = QgShape<MT, FR>;
    using TR = F16Traits<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr int RING_MIN = S::RED_BYTES;  // the ring is reused for the partial sums

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int ns = a.ns;
    const int ring = ns * S::STAGE_BYTES > RING_MIN ? ns * S::STAGE_BYTES : RING_MIN;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring);
    uint64_t* empty = full + QG_MAX_STAGES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool moe = a.mode != QG_DENSE;
    // units [u0, u0 + nu) of fpu fragments each: a CTA holds FR or FR - fpu fragments (host-chosen grid)
    const int u0 = int((long long)blockIdx.x * a.units / gridDim.x);
    const int nu = int((long long)(blockIdx.x + 1) * a.units / gridDim.x) - u0;
    const int f0 = u0 * a.fpu;
    const int nf = nu * a.fpu;
    if (nf < 1 || nf > FR || nf < FR - a.fpu) {  // the weight boxes hold 16 FR or 16 (FR - fpu) rows: nothing else fits
        if (threadIdx.x == 0) record_status(LQ_DEV_BOUNDS);
        return;
    }
    const int row0 = 16 * f0;
    const int total = a.nchunk;
    const int mv = a.M < S::MTOK ? a.M : S::MTOK;  // real token rows

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; ++s) {
            mbar_init(&full[s], 1 + 32);  // lane 0's expect_tx arrive + 32 cp.async arrivals
            mbar_init(&empty[s], QG_CW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    bool ok = true;

    if (warp == QG_CW) {
        // ------------------------------ producer warp ------------------------------
        const uint64_t pol_w = policy_evict_first();
        // dense: one box of 16 FR or 16 (FR - 1) rows; MoE: one 16-row box a fragment from matrix 0 or 1
        const CUtensorMap* tm_w = nf == FR ? &tm_w_full : &tm_w_less;
        if (lane == 0) {
            prefetch_tmap(&tm_w_full);
            prefetch_tmap(&tm_w_less);
        }
        // MoE: each fragment's first row in its stack and its matrix (0: gate or down, 1: up); the experts come from the
        // routing kernel, so these loads wait for it
        int frow[FR], fmat[FR];
#pragma unroll
        for (int i = 0; i < FR; ++i) {
            frow[i] = row0 + 16 * i;
            fmat[i] = 0;
        }
        if (moe) {
            grid_dep_wait();
#pragma unroll
            for (int i = 0; i < FR; ++i) {
                const int j = f0 + (i < nf ? i : nf - 1);  // (the unused slots repeat the last fragment)
                int seg, fe;
                if (a.mode == QG_MOE_GLU) {
                    const int u = j >> 1;
                    seg = u / a.fpe;
                    fe = u - seg * a.fpe;
                    fmat[i] = j & 1;
                } else {
                    const int u = j / a.fpu, r = j - u * a.fpu;
                    seg = a.pos ? a.pos[r] : r;
                    fe = u;
                }
                int e = a.experts[seg];
                if (e < 0 || (e + 1) * a.rows_e > a.N) {
                    if (lane == 0) record_status(LQ_DEV_BOUNDS);
                    e = 0;
                }
                frow[i] = e * a.rows_e + 16 * fe;
            }
        }
        const uint32_t smem_base = smem_u32(smem);
        const int vb = a.sb_vec;
        const int units = 16 / vb;
        auto load_weights = [&](int c, int s) {
            uint8_t* st = smem + s * S::STAGE_BYTES;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], nf * S::W_FRAG);
                if (!moe) {
                    tma_load_3d(st, tm_w, &full[s], 0, row0, 2 * c, pol_w);
                } else {
#pragma unroll
                    for (int i = 0; i < FR; ++i)
                        if (i < nf)
                            tma_load_3d(st + i * S::W_FRAG, fmat[i] ? &tm_w_less : &tm_w_full, &full[s], 0, frow[i], 2 * c,
                                        pol_w);
                }
            }
            const uint32_t sdst = smem_base + s * S::STAGE_BYTES + S::W_BYTES;
            for (int r = lane; r < nf * 16; r += 32) {
                const int fi = r >> 4;
                int frow_r = frow[0], fmat_r = fmat[0];
#pragma unroll
                for (int i = 1; i < FR; ++i)
                    if (fi == i) {
                        frow_r = frow[i];
                        fmat_r = fmat[i];
                    }
                const int grow = frow_r + (r & 15);
                const uint8_t* sbase = reinterpret_cast<const uint8_t*>(fmat_r ? a.s1 : a.s);
                const uint8_t* bbase = reinterpret_cast<const uint8_t*>(fmat_r ? a.b1 : a.b);
                for (int u = 0; u < units; ++u) {
                    const int gcol = 8 * c + u * (vb >> 1);
                    const bool valid = grow < a.N && gcol < a.kg;
                    const size_t off = valid ? (size_t(grow) * a.kg + gcol) * 2 : 0;
                    const uint32_t d = sdst + r * 16 + u * vb;
                    cp_async(d, sbase + off, vb, valid);
                    cp_async(d + S::SB_BYTES, bbase + off, vb, valid);
                }
            }
        };
        const int pre = total < ns ? total : ns;
        for (int i = 0; i < pre; ++i) {  // (weights and scales only: nothing here waits for the previous kernel)
            load_weights(i, i);
            cp_async_arrive(&full[i]);
        }
        if (lane == 0) grid_dep_launch();
        for (int i = pre; i < total; ++i) {
            const int s = i % ns;
            ok = mbar_wait(&empty[s], ((i / ns) - 1) & 1);
            if (!ok) break;
            load_weights(i, s);
            cp_async_arrive(&full[s]);
        }
        __syncwarp();
        return;
    }

    // ------------------------------ consumer warps ------------------------------
    grid_dep_wait();  // x may be the previous kernel's output (and before any output store of this kernel)
    const int g = lane >> 2, t = lane & 3;
    const uint32_t smem_base = smem_u32(smem);
    float acc[FR][MT][4];
#pragma unroll
    for (int f = 0; f < FR; ++f)
#pragma unroll
        for (int q = 0; q < MT; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[f][q][e] = 0.0f;

    // this lane's 8 bytes of a row inside group w of a stage (128-byte swizzle: 16-byte chunk c of row r sits at
    // c ^ (r & 7)); dense: the stage's box is [segment][16 nf rows][128 bytes], fragment f's rows at 2048 f of each
    // segment; MoE: fragment f's own box [segment][16 rows][128 bytes] at 4096 f
    const uint32_t frag_stride = moe ? S::W_FRAG : 2048;
    const uint32_t w_off = (warp >> 2) * (moe ? 2048 : nf * 2048) + g * 128 + (((2 * (warp & 3) + (t >> 1)) ^ g) << 4) +
                           8 * (t & 1);
    // x of stage i's group for this lane: values 16t .. 16t + 15 of tokens g + 8 mt (zero past M and past K); the fused
    // down + combine puts slot g's row of h (pos[g]) in token column g
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(a.x);
    int xrow[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int tok = 8 * mt + g;
        xrow[mt] = (a.mode == QG_MOE_COMBINE && a.pos && tok < a.M) ? a.pos[tok] : tok;
    }
    auto fetch_x = [&](int i, uint4 (&u)[MT][2]) {
        const int gi = 8 * i + warp;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int tok = 8 * mt + g;
            if (tok < a.M && gi < a.kg) {
                const uint4* p = reinterpret_cast<const uint4*>(xg + (size_t(xrow[mt]) * a.K + gi * 64 + 16 * t) * 2);
                u[mt][0] = p[0];
                u[mt][1] = p[1];
            } else {
                u[mt][0] = make_uint4(0u, 0u, 0u, 0u);
                u[mt][1] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };
    uint4 xc[MT][2], xn[MT][2];
    fetch_x(0, xc);

    for (int i = 0; i < total; ++i) {
        const int s = i % ns;
        if (i + 1 < total) fetch_x(i + 1, xn);  // one stage ahead of its use
        if (ok) ok = mbar_wait(&full[s], (i / ns) & 1);
        if (ok && 8 * i + warp < a.kg) {
            const uint32_t st = smem_base + s * S::STAGE_BYTES;
            // x fragments of group w permuted to the code order
            uint32_t xb[MT][4][2];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint4 u0 = xc[mt][0], u1 = xc[mt][1];
                xb[mt][0][0] = prmt(u0.x, u0.z, 0x5410);
                xb[mt][0][1] = prmt(u0.x, u0.z, 0x7632);
                xb[mt][1][0] = prmt(u0.y, u0.w, 0x5410);
                xb[mt][1][1] = prmt(u0.y, u0.w, 0x7632);
                xb[mt][2][0] = prmt(u1.x, u1.z, 0x5410);
                xb[mt][2][1] = prmt(u1.x, u1.z, 0x7632);
                xb[mt][3][0] = prmt(u1.y, u1.w, 0x5410);
                xb[mt][3][1] = prmt(u1.y, u1.w, 0x7632);
            }
            const uint32_t sb = st + S::W_BYTES + 2 * warp;
            // All FR fragments run without a branch, so the stage is one straight block whose shared loads the
            // compiler can issue ahead of the arithmetic. A CTA holding nf = FR - 1 fragments computes one extra
            // fragment from stale bytes: every address stays inside the stage (weights below (2 FR - 1) * 2048 <
            // W_BYTES, scales and biases inside their FR * 16-row tables), its partial sums land in rows
            // [16 nf, 16 FR) of the reduction table and the final sum reads rows below 16 nf only. Those CTAs are
            // off the critical path (the FR-fragment CTAs set the kernel's length).
#pragma unroll
            for (int f = 0; f < FR; ++f) {
                {
                    const uint32_t fb = st + f * frag_stride + w_off;
                    const uint2 wa = qg_lds64(fb), wb = qg_lds64(fb + 8 * 128);
                    const int ra = 16 * f + g, rb = ra + 8;
                    const uint32_t sa = lds_u16(sb + ra * 16), ba = lds_u16(sb + S::SB_BYTES + ra * 16);
                    const uint32_t sbv = lds_u16(sb + rb * 16), bbv = lds_u16(sb + S::SB_BYTES + rb * 16);
                    const uint32_t s2a = prmt(sa, sa, 0x1010), b2a = prmt(ba, ba, 0x1010);
                    const uint32_t s2b = prmt(sbv, sbv, 0x1010), b2b = prmt(bbv, bbv, 0x1010);
#pragma unroll
                    for (int step = 0; step < 4; ++step) {
                        const uint32_t va = step < 2 ? wa.x : wa.y, vbw = step < 2 ? wb.x : wb.y;
                        const int sh = 8 * (step & 1);  // codes (p, p + 4) and (p + 1, p + 5), p = 2 (step & 1)
                        const uint32_t a0 = TR::sub_magic_fma(lop3_and_or(va >> sh, 0x000F000Fu, TR::kMagic2), s2a, b2a);
                        const uint32_t a2 =
                            TR::sub_magic_fma(lop3_and_or(va >> (sh + 4), 0x000F000Fu, TR::kMagic2), s2a, b2a);
                        const uint32_t a1 =
                            TR::sub_magic_fma(lop3_and_or(vbw >> sh, 0x000F000Fu, TR::kMagic2), s2b, b2b);
                        const uint32_t a3 =
                            TR::sub_magic_fma(lop3_and_or(vbw >> (sh + 4), 0x000F000Fu, TR::kMagic2), s2b, b2b);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
                            qg_mma<T>(acc[f][mt], a0, a1, a2, a3, xb[mt][step][0], xb[mt][step][1]);
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

    // ---- the eight warps' partial sums, added through shared memory (the ring is free: every stage was consumed) ----
    named_barrier(1, 32 * QG_CW);
    float* red = reinterpret_cast<float*>(smem);  // [warp][token][FR * 16 rows]
    constexpr int RR = FR * 16;
#pragma unroll
    for (int f = 0; f < FR; ++f)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = 16 * f + g + 8 * (e >> 1), tok = 8 * mt + 2 * t + (e & 1);
                red[(warp * S::MTOK + tok) * RR + row] = acc[f][mt][e];
            }
    named_barrier(1, 32 * QG_CW);
    auto sum_warps = [&](int tok, int row) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < QG_CW; ++w) v += red[(w * S::MTOK + tok) * RR + row];
        return v;
    };
    if (a.mode == QG_MOE_GLU) {
        // unit i: gate rows at fragment 2i, up rows at 2i + 1 -> h[segment][16 fe + r]
        for (int idx = threadIdx.x; idx < nu * 16; idx += 32 * QG_CW) {
            const int i = idx >> 4, r = idx & 15;
            const int u = u0 + i, seg = u / a.fpe, fe = u - seg * a.fpe;
            const float v = qg_swiglu<T>(sum_warps(0, 32 * i + r), sum_warps(0, 32 * i + 16 + r));
            if (ok) qg_store(a, seg, 16 * fe + r, v, kBF16);
        }
        return;
    }
    if (a.mode == QG_MOE_COMBINE) {
        // unit i: slot r's rows at fragment k i + r, its token column r; y = sum_r w_r * round(y_r), slots in order
        const int k = a.fpu;
        for (int idx = threadIdx.x; idx < nu * 16; idx += 32 * QG_CW) {
            const int i = idx >> 4, r = idx & 15;
            float y = 0.0f;
            for (int sl = 0; sl < k; ++sl) {
                const float ys = qg_round<T>(sum_warps(sl, 16 * (k * i + sl) + r));
                y = fmaf(ys, a.wts[sl], y);  // as the stand-alone combine kernel sums the slots
            }
            if (ok) qg_store(a, 0, 16 * (u0 + i) + r, y, kBF16);
        }
        return;
    }
    const int R = nf * 16;
    for (int idx = threadIdx.x; idx < R * mv; idx += 32 * QG_CW) {
        const int tok = idx / R, row = idx - tok * R;
        const int n = row0 + row;
        if (n >= a.N) continue;
        const float v = sum_warps(tok, row);
        if (ok) qg_store(a, tok, n, v, kBF16);
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------

template <typename T, int MT, int FR>
static int qmvg_launch_t(const void* x, const uint32_t* w, const uint32_t* w1, QgArgs a, int ns_req, int nctas,
                         cudaStream_t st) {
    using S = QgShape<MT, FR>;
    const DeviceInfo& di = device_info();
    const int K = a.K;
    // stages: within half an SM's shared memory, so the next launch's CTA can start beside a running one
    const size_t fixed = 2 * QG_MAX_STAGES * 8 + 1024;
    const size_t budget = di.smem_per_sm / 2 - 1024;
    int ns = int((budget - fixed) / S::STAGE_BYTES);
    if (ns > QG_MAX_STAGES) ns = QG_MAX_STAGES;
    if (ns > a.nchunk) ns = a.nchunk;
    if (ns_req > 0 && ns_req < ns) ns = ns_req;
    if (ns < 1) return LQ_E_SHAPE;
    a.ns = ns;
    size_t ring = size_t(ns) * S::STAGE_BYTES;
    if (ring < size_t(S::RED_BYTES)) ring = S::RED_BYTES;
    const size_t smem = ring + fixed;
    if (smem > di.smem_optin) return LQ_E_SHAPE;

    // dense: weight boxes of 16 FR rows (CTAs holding FR fragments) and 16 (FR - 1) rows (the others); MoE: 16-row
    // boxes of the two stacked matrices (gate / up, or down twice); two 128-byte segments a stage
    const bool moe = a.mode != QG_DENSE;
    CUtensorMap tw[2];
    for (int m = 0; m < 2; ++m) {
        const int rows = moe ? 16 : 16 * (m == 0 || FR == 1 ? FR : FR - 1);
        const uint64_t dims[3] = {32, uint64_t(a.N), uint64_t(K) / 256};
        const uint64_t str[2] = {uint64_t(K) / 2, 128};
        const uint32_t box[3] = {32, uint32_t(rows), 2};
        const uint32_t* base = (moe && m == 1 && w1) ? w1 : w;
        const int rc =
            make_tmap(&tw[m], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    a.x = x;
    const int kg = a.kg;
    const uintptr_t sb_addr = reinterpret_cast<uintptr_t>(a.s) | reinterpret_cast<uintptr_t>(a.b) |
                              reinterpret_cast<uintptr_t>(a.s1) | reinterpret_cast<uintptr_t>(a.b1);
    a.sb_vec = (kg % 8 == 0 && sb_addr % 16 == 0) ? 16 : (kg % 4 == 0 && sb_addr % 8 == 0) ? 8 : 4;

    auto kern = qmvg_kernel<T, MT, FR>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nctas, 1, 1);
    cfg.blockDim = dim3(QG_THREADS, 1, 1);
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

template <typename T, int MT>
static int qmvg_dispatch_fr(int FR, const void* x, const uint32_t* w, const uint32_t* w1, const QgArgs& a, int ns,
                            int nctas, cudaStream_t st) {
    switch (FR) {
        case 1: return qmvg_launch_t<T, MT, 1>(x, w, w1, a, ns, nctas, st);
        case 2: return qmvg_launch_t<T, MT, 2>(x, w, w1, a, ns, nctas, st);
        case 3: return qmvg_launch_t<T, MT, 3>(x, w, w1, a, ns, nctas, st);
        case 4: return qmvg_launch_t<T, MT, 4>(x, w, w1, a, ns, nctas, st);
        default: return LQ_E_SHAPE;
    }
}

bool qmvg_shape_ok(int M, int K, int bits) { return bits == 4 && M >= 1 && M <= 16 && K >= 256 && K % 256 == 0; }

// p = {FR (max fragments a CTA, 0 = spread over every SM), NS (stages, 0 = choose)}.
int qmvg_run(const void* x, const uint32_t* w, const void* s, const void* b, int nout, void* const* outs,
             const int* seg_end, const int* ldo, int M, int N, int K, int dtype, const int* p, cudaStream_t st) {
    if (!qmvg_shape_ok(M, K, 4) || N < 1) return LQ_E_SHAPE;
    QgArgs a = {};
    a.M = M;
    a.N = N;
    a.K = K;
    a.kg = K / 64;
    a.nchunk = (K + 511) / 512;
    a.nfrag = (N + 15) / 16;
    a.s = s;
    a.b = b;
    for (int i = 0; i < nout; ++i) {
        a.out[i] = outs[i];
        a.seg_end[i] = seg_end[i];
        a.ldo[i] = ldo[i];
    }
    a.nseg_out = nout;
    const int sms = device_info().sm_count;
    const int fr_req = p ? p[0] : 0;
    const int ns = p ? p[1] : 0;
    if (fr_req < 0 || fr_req > QG_MAX_FR) return LQ_E_ARG;
    // CTAs: at most fr fragments each; the library's choice spreads them over every SM. Then every CTA holds FR or
    // FR - 1 fragments with FR = ceil(nfrag / nctas), the two weight-box heights the kernel is given.
    int fr = fr_req;
    if (fr == 0) {
        fr = (a.nfrag + sms - 1) / sms;
        if (fr > QG_MAX_FR) fr = QG_MAX_FR;
    }
    int nctas = (a.nfrag + fr - 1) / fr;
    if (fr_req == 0 && nctas < sms) nctas = a.nfrag < sms ? a.nfrag : sms;
    const int FR = (a.nfrag + nctas - 1) / nctas;
    a.mode = QG_DENSE;
    a.fpu = 1;
    a.units = a.nfrag;
    const bool bf16 = dtype == LQ_BF16;
    if (M <= 8)
        return bf16 ? qmvg_dispatch_fr<__nv_bfloat16, 1>(FR, x, w, nullptr, a, ns, nctas, st)
                    : qmvg_dispatch_fr<__half, 1>(FR, x, w, nullptr, a, ns, nctas, st);
    return bf16 ? qmvg_dispatch_fr<__nv_bfloat16, 2>(FR, x, w, nullptr, a, ns, nctas, st)
                : qmvg_dispatch_fr<__half, 2>(FR, x, w, nullptr, a, ns, nctas, st);
}

// The MoE decode modes for ONE token (its k pairs, one a segment of the grouping) over stacked (E, rows_e, K) 4-bit
// experts. glu: out (k, rows_e) = swiglu(x . gate_e^T, x . up_e^T) of segment s's expert experts[s], rows in segment
// order. combine (k <= 4): out (1, rows_e) = sum_r wts[r] * round(h[pos[r]] . down_e^T), e = experts[pos[r]], slots in
// order. 0 or LQ_E_SHAPE when the shape does not fit these modes (the caller then uses the grouped qmv path).
bool qmvg_moe_ok(int mode, int k, int rows_e, int K, int sms) {
    if (k < 1 || k > 8 || rows_e < 16 || rows_e % 16 || K < 256 || K % 256) return false;
    const int fpe = rows_e / 16;
    if (mode == QG_MOE_GLU) return (k * fpe + sms - 1) / sms * 2 <= QG_MAX_FR;
    return k <= QG_MAX_FR;
}

int qmvg_moe_run(int mode, const void* x, const int32_t* experts, const int32_t* pos, const float* wts,
                 const uint32_t* w0, const void* s0, const void* b0, const uint32_t* w1, const void* s1, const void* b1,
                 void* out, int k, int E, int rows_e, int K, int dtype, cudaStream_t st) {
    const int sms = device_info().sm_count;
    if (!qmvg_moe_ok(mode, k, rows_e, K, sms)) return LQ_E_SHAPE;
    QgArgs a = {};
    a.mode = mode;
    a.K = K;
    a.kg = K / 64;
    a.nchunk = (K + 511) / 512;
    a.N = E * rows_e;  // rows of each stack
    a.rows_e = rows_e;
    a.fpe = rows_e / 16;
    a.experts = experts;
    a.pos = pos;
    a.wts = wts;
    a.s = s0;
    a.b = b0;
    a.s1 = mode == QG_MOE_GLU ? s1 : s0;
    a.b1 = mode == QG_MOE_GLU ? b1 : b0;
    a.out[0] = out;
    a.ldo[0] = rows_e;
    a.seg_end[0] = rows_e;
    a.nseg_out = 1;
    if (mode == QG_MOE_GLU) {
        a.M = 1;  // the one token
        a.fpu = 2;
        a.units = k * a.fpe;
    } else {
        a.M = k;  // slot r's row of h in token column r
        a.fpu = k;
        a.units = a.fpe;
    }
    a.nfrag = a.units * a.fpu;
    const int nctas = a.units < sms ? a.units : sms;
    const int FR = (a.units + nctas - 1) / nctas * a.fpu;
    const bool bf16 = dtype == LQ_BF16;
    const uint32_t* wm1 = mode == QG_MOE_GLU ? w1 : w0;
    return bf16 ? qmvg_dispatch_fr<__nv_bfloat16, 1>(FR, x, w0, wm1, a, 0, nctas, st)
                : qmvg_dispatch_fr<__half, 1>(FR, x, w0, wm1, a, 0, nctas, st);
}

}  // namespace lq
