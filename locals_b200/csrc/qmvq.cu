// Dense 4-bit decode with the codes fed raw to the MMA and scale and bias folded per group in fp32 ("qmvq" family):
// y (M, N) = x (M, K) . dequant(W)^T for M <= 16 tokens. The B200 counterpart of the reference's fragq kernel
// (locals/qmv_frag.py:368-540): there the codes enter the 8x8 MMA as 1 + q/16 in the mantissa and each group's scale
// and bias are applied to the fp32 partial sum; here they enter mma.sync.m16n8k16 as 128 + q (bf16) or 1024 + q
// (fp16) -- one lop3 with the magic exponent per code pair, no subtract, no fma -- and each 64-wide group ends with
//     y += s * acc + (b - magic * s) * sum(x)
// in fp32, where acc = sum((magic + q) x) over the group and sum(x) is the group's x sum, taken by one more MMA with
// an all-ones A operand (so it lands in the accumulator layout the fold needs). The weights are never rounded to the
// activation dtype: the result is the fp32 factoring s . sum(q x) + b . sum(x) of the reference's multi-row kernels
// (locals/qmv_multi.py:57-75), which is what mx.quantized_matmul computes.
//
// Work split as in the group-per-warp family (qmvg.cu): the N/16 row fragments dealt out evenly over every SM, one
// ring stage = 512 K values of all of the CTA's rows (one TMA box), consumer warp w takes group w of every stage for
// all of the CTA's fragments, the eight warps' partial sums added through shared memory at the end, x loaded by each
// consumer lane straight into registers one stage ahead. Nothing the producer loads depends on the previous kernel,
// so under programmatic dependent launch the whole ring fills before the dependency resolves. (A producer that also
// widened each stage's scales into an fp32 (s, b - magic s) table was measured 1.8x slower on B200: one warp doing
// that for every stage delays the ring and the dependent launch; the consumers widen their own two rows instead.)
// Reference: the multi-row GEMV it replaces, locals/qmv_frag.py:368-540 (fragq) behind kernels._launcher
// (locals/kernels.py:516-576).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"

namespace lq {

constexpr int QQ_CW = 8;  // consumer warps: group w of every 8-group stage
constexpr int QQ_THREADS = 32 * (QQ_CW + 1);
constexpr int QQ_MAX_STAGES = 6;
constexpr int QQ_MAX_FR = 4;

template <int MT, int FR>
struct QqShape {
    static constexpr int MTOK = 8 * MT;                  // token slots
    static constexpr int W_FRAG = 16 * 256;              // one 16-row fragment: 256 bytes (512 codes) a row
    static constexpr int W_BYTES = FR * W_FRAG;
    static constexpr int SB_BYTES = FR * 16 * 16;        // scales (or biases): rows x 8 groups x 2 bytes
    static constexpr int STAGE_BYTES = (W_BYTES + 2 * SB_BYTES + 1023) / 1024 * 1024;
    // the warps' partial sums [warp][token][FR * 16 rows + 4]: the 4-float pad puts the four token columns a lane
    // quad writes at once 8 banks apart, so every partial-sum store of a warp is free of bank conflicts
    static constexpr int RRP = FR * 16 + 4;
    static constexpr int RED_BYTES = QQ_CW * MTOK * RRP * 4;
    // x loaded DX stages ahead of its use: two for up to 8 tokens, one for 16 (the register budget of two CTAs an SM)
    static constexpr int DX = MT == 1 ? 2 : 1;
    static_assert(W_FRAG % 1024 == 0, "1 KB alignment of swizzled tiles");
};

struct QqArgs {
    int M, N, K;
    int kg;      // groups a row (K / 64)
    int nchunk;  // stages of 512 K values
    int nfrag;   // 16-row fragments (ceil(N / 16))
    int ns;      // ring depth
    int sb_vec;  // cp.async width for scale / bias rows
    int cpw;     // 1: the consumer threads copy the weights (cp.async, before the grid dependency), 0: TMA
    const uint32_t* w;
    const void* x;
    const void* s;
    const void* b;
    void* out[3];  // output column segments (fused q / k / v), or out[0] only
    int seg_end[3];
    int ldo[3];
    int nseg_out;
};

template <typename T>
struct QqMagic;
template <>
struct QqMagic<__nv_bfloat16> {
    static constexpr uint32_t kCode2 = 0x43004300u;  // bf16x2 (128, 128): 128 + q is exact for q < 128
    static constexpr uint32_t kOne2 = 0x3F803F80u;   // bf16x2 (1, 1)
    static constexpr float kVal = 128.0f;
};
template <>
struct QqMagic<__half> {
    static constexpr uint32_t kCode2 = 0x64006400u;  // fp16x2 (1024, 1024): 1024 + q is exact for q < 1024
    static constexpr uint32_t kOne2 = 0x3C003C00u;   // fp16x2 (1, 1)
    static constexpr float kVal = 1024.0f;
};

// (Shared-memory reads as plain C++ loads, which let the compiler reorder them across fragments, measured slower on
// B200: 5.10 against 4.90 us a layer at one token.)
__device__ __forceinline__ uint2 qq_lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// mma.sync m16n8k16 with fp32 accumulation, left to the compiler's scheduling (no side effects beyond its registers).
template <typename T>
__device__ __forceinline__ void qq_mma(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
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

// Output element (row, n) of the fused projection: segment chosen with constant indices.
__device__ __forceinline__ void qq_store(const QqArgs& a, int row, int n, float v, bool bf16) {
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

// SXA: the group's x sums by fp32 adds and quad shuffles (true) or by an MMA with an all-ones A operand (false)
template <typename T, int MT, int FR, bool SXA>
__global__ void __launch_bounds__(QQ_THREADS, 2)
    qmvq_kernel(const __grid_constant__ CUtensorMap tm_w_full, const __grid_constant__ CUtensorMap tm_w_less,
                const QqArgs a) {
    using S = QqShape<MT, FR>;
    using TR = F16Traits<T>;
    using MG = QqMagic<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr int RING_MIN = S::RED_BYTES;  // the ring is reused for the partial sums

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int ns = a.ns;
    const int ring = ns * S::STAGE_BYTES > RING_MIN ? ns * S::STAGE_BYTES : RING_MIN;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring);
    uint64_t* empty = full + QQ_MAX_STAGES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // fragments [f0, f0 + nf): a CTA holds FR or FR - 1 of them (host-chosen grid)
    const int f0 = int((long long)blockIdx.x * a.nfrag / gridDim.x);
    const int nf = int((long long)(blockIdx.x + 1) * a.nfrag / gridDim.x) - f0;
    if (nf < 1 || nf > FR || nf < FR - 1) {  // the weight boxes hold 16 FR or 16 (FR - 1) rows: nothing else fits
        if (threadIdx.x == 0) record_status(LQ_DEV_BOUNDS);
        return;
    }
    const int row0 = 16 * f0;
    const int total = a.nchunk;
    const int mv = a.M < S::MTOK ? a.M : S::MTOK;  // real token rows

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; ++s) {
            // TMA: lane 0's expect_tx arrive + the producer lanes' cp.async arrivals (scales); consumer-copied
            // weights: the producer lanes' and every consumer thread's cp.async arrivals
            mbar_init(&full[s], a.cpw ? 32 + 32 * QQ_CW : 1 + 32);
            mbar_init(&empty[s], QQ_CW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    bool ok = true;

    if (warp == QQ_CW) {
        // ------------------------------ producer warp ------------------------------
        const uint64_t pol_w = policy_evict_first();
        const CUtensorMap* tm_w = nf == FR ? &tm_w_full : &tm_w_less;
        if (lane == 0) {
            prefetch_tmap(&tm_w_full);
            prefetch_tmap(&tm_w_less);
        }
        const uint32_t smem_base = smem_u32(smem);
        const int vb = a.sb_vec;
        const int units = 16 / vb;
        auto load = [&](int c, int s) {
            uint8_t* st = smem + s * S::STAGE_BYTES;
            if (lane == 0 && !a.cpw) {
                mbar_arrive_expect_tx(&full[s], nf * S::W_FRAG);
                tma_load_3d(st, tm_w, &full[s], 0, row0, 2 * c, pol_w);
            }
            const uint32_t sdst = smem_base + s * S::STAGE_BYTES + S::W_BYTES;
            for (int r = lane; r < nf * 16; r += 32) {
                const int grow = row0 + r;
                for (int u = 0; u < units; ++u) {
                    const int gcol = 8 * c + u * (vb >> 1);
                    const bool valid = grow < a.N && gcol < a.kg;
                    const size_t off = valid ? (size_t(grow) * a.kg + gcol) * 2 : 0;
                    const uint32_t d = sdst + r * 16 + u * vb;
                    cp_async(d, reinterpret_cast<const uint8_t*>(a.s) + off, vb, valid);
                    cp_async(d + S::SB_BYTES, reinterpret_cast<const uint8_t*>(a.b) + off, vb, valid);
                }
            }
            cp_async_arrive(&full[s]);
        };
        const int pre = total < ns ? total : ns;
        for (int i = 0; i < pre; ++i) load(i, i);  // (weights and scales only: nothing here waits for the previous
                                                   // kernel)
        if (lane == 0) grid_dep_launch();
        for (int i = pre; i < total; ++i) {
            const int s = i % ns;
            ok = mbar_wait(&empty[s], ((i / ns) - 1) & 1);
            if (!ok) break;
            load(i, s);
        }
        __syncwarp();
        return;
    }

    // ------------------------------ consumer warps ------------------------------
    const uint32_t smem_base = smem_u32(smem);
    if (a.cpw) {
        // Every stage's packed words by the consumer threads' own 16-byte cp.async, issued before the grid dependency
        // (they do not depend on the previous kernel), into the layout the TMA box would give: chunk c of row r at
        // segment c / 8, 128 r + 16 ((c % 8) ^ (r % 8)). Zero-filled past N and past K. Only used when the ring holds
        // every stage (the host checks).
        const uint8_t* wb = reinterpret_cast<const uint8_t*>(a.w);
        const size_t row_bytes = size_t(a.K) / 2;
        for (int i = 0; i < total; ++i) {
            const uint32_t st = smem_base + i * S::STAGE_BYTES;
            for (int idx = threadIdx.x; idx < nf * 16 * 16; idx += 32 * QQ_CW) {
                const int r = idx >> 4, c = idx & 15;
                const bool valid = row0 + r < a.N && i * 512 + c * 32 < a.K;
                const uint8_t* src = valid ? wb + size_t(row0 + r) * row_bytes + i * 256 + c * 16 : wb;
                cp_async(st + (c >> 3) * (nf * 2048) + r * 128 + (((c & 7) ^ (r & 7)) << 4), src, 16, valid);
            }
            cp_async_arrive(&full[i]);
        }
    }
    grid_dep_wait();  // x may be the previous kernel's output (and before any output store of this kernel)
    const int g = lane >> 2, t = lane & 3;
    float acc[FR][MT][4];
#pragma unroll
    for (int f = 0; f < FR; ++f)
#pragma unroll
        for (int q = 0; q < MT; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[f][q][e] = 0.0f;

    // this lane's 8 bytes of a row inside group w of a stage (128-byte swizzle: 16-byte chunk c of row r sits at
    // c ^ (r & 7)); the stage's box is [segment][16 nf rows][128 bytes], fragment f's rows at 2048 f of each segment
    const uint32_t w_off =
        (warp >> 2) * (nf * 2048) + g * 128 + (((2 * (warp & 3) + (t >> 1)) ^ g) << 4) + 8 * (t & 1);
    // x of stage i's group for this lane: values 16t .. 16t + 15 of tokens g + 8 mt (zero past M and past K), loaded
    // straight into registers ahead of its use. (Staging x in shared memory by the lanes' own cp.async
    // instead -- every stage at once, or one ahead -- measured slower on B200: 7.0 and 7.3 us against 4.8 us a layer
    // on the one-token QKV projection.)
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(a.x);
    // Token columns past M keep whatever their registers held: an MMA's output column n depends on its input column n
    // only (the x sums too), and those columns are never stored. Stages past K are skipped whole.
    auto fetch_x = [&](int i, uint4 (&u)[MT][2]) {
        const int gi = 8 * i + warp;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int tok = 8 * mt + g;
            if (tok < a.M && gi < a.kg) {
                const uint4* p = reinterpret_cast<const uint4*>(xg + (size_t(tok) * a.K + gi * 64 + 16 * t) * 2);
                u[mt][0] = p[0];
                u[mt][1] = p[1];
            }
        }
    };
    uint4 xc[MT][2], xn[MT][2], xnn[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) xc[mt][h] = xn[mt][h] = xnn[mt][h] = make_uint4(0u, 0u, 0u, 0u);
    fetch_x(0, xc);
    if (S::DX == 2 && total > 1) fetch_x(1, xn);

    for (int i = 0; i < total; ++i) {
        const int s = i % ns;
        if (S::DX == 1) {
            if (i + 1 < total) fetch_x(i + 1, xn);  // one stage ahead of its use
        } else {
            if (i + 2 < total) fetch_x(i + 2, xnn);  // two stages ahead of its use
        }
        if (ok) ok = mbar_wait(&full[s], (i / ns) & 1);
        if (ok && 8 * i + warp < a.kg) {
            const uint32_t st = smem_base + s * S::STAGE_BYTES;
            // x fragments of group w permuted to the code order, and the group's x sums in the accumulator layout
            // (sx[mt][e] = sum(x) of token column 2t + (e & 1); rows are alike, so entries 2 and 3 go unused)
            uint32_t xb[MT][4][2];
            float sx[MT][4];
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
                if constexpr (SXA) {
                    // this lane's 16 values of token g + 8 mt, then the quad's 64, then moved to columns 2t, 2t + 1
                    const uint32_t wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                    float sum = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) sum += TR::to_f32(wv[j] & 0xFFFFu) + TR::to_f32(wv[j] >> 16);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                    const float s0 = __shfl_sync(0xffffffffu, sum, 8 * t), s1 = __shfl_sync(0xffffffffu, sum, 8 * t + 4);
                    sx[mt][0] = s0;
                    sx[mt][1] = s1;
                    sx[mt][2] = s0;
                    sx[mt][3] = s1;
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) sx[mt][e] = 0.0f;
#pragma unroll
                    for (int step = 0; step < 4; ++step)
                        qq_mma<T>(sx[mt], MG::kOne2, MG::kOne2, MG::kOne2, MG::kOne2, xb[mt][step][0],
                                  xb[mt][step][1]);
                }
            }
            const uint32_t sb = st + S::W_BYTES + 2 * warp;  // group w's scale of row r at sb + 16 r
            // All FR fragments run without a branch (one straight block). A CTA holding nf = FR - 1 fragments
            // computes one extra fragment from stale bytes of its own stage: every address stays inside the stage's
            // weight box and tables, and its partial sums land in reduction rows the final sum never reads.
#pragma unroll
            for (int f = 0; f < FR; ++f) {
                const uint32_t fb = st + f * 2048 + w_off;
                const uint2 wa = qq_lds64(fb), wb = qq_lds64(fb + 8 * 128);
                // rows g and g + 8: (s, b - magic s) in fp32
                const int ra = 16 * f + g, rb = ra + 8;
                const float sa = TR::to_f32(lds_u16(sb + ra * 16)), sbb = TR::to_f32(lds_u16(sb + rb * 16));
                const float2 pa = make_float2(sa, fmaf(-MG::kVal, sa, TR::to_f32(lds_u16(sb + S::SB_BYTES + ra * 16))));
                const float2 pb = make_float2(sbb, fmaf(-MG::kVal, sbb, TR::to_f32(lds_u16(sb + S::SB_BYTES + rb * 16))));
                float part[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) part[mt][e] = 0.0f;
#pragma unroll
                for (int step = 0; step < 4; ++step) {
                    const uint32_t va = step < 2 ? wa.x : wa.y, vbw = step < 2 ? wb.x : wb.y;
                    const int sh = 8 * (step & 1);  // codes (p, p + 4) and (p + 1, p + 5), p = 2 (step & 1)
                    const uint32_t a0 = lop3_and_or(va >> sh, 0x000F000Fu, MG::kCode2);
                    const uint32_t a2 = lop3_and_or(va >> (sh + 4), 0x000F000Fu, MG::kCode2);
                    const uint32_t a1 = lop3_and_or(vbw >> sh, 0x000F000Fu, MG::kCode2);
                    const uint32_t a3 = lop3_and_or(vbw >> (sh + 4), 0x000F000Fu, MG::kCode2);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        qq_mma<T>(part[mt], a0, a1, a2, a3, xb[mt][step][0], xb[mt][step][1]);
                }
                // y += s * acc + (b - magic s) * sum(x), rows g (pa) and g + 8 (pb)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    acc[f][mt][0] = fmaf(pa.x, part[mt][0], fmaf(pa.y, sx[mt][0], acc[f][mt][0]));
                    acc[f][mt][1] = fmaf(pa.x, part[mt][1], fmaf(pa.y, sx[mt][1], acc[f][mt][1]));
                    acc[f][mt][2] = fmaf(pb.x, part[mt][2], fmaf(pb.y, sx[mt][0], acc[f][mt][2]));
                    acc[f][mt][3] = fmaf(pb.x, part[mt][3], fmaf(pb.y, sx[mt][1], acc[f][mt][3]));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            xc[mt][0] = xn[mt][0];
            xc[mt][1] = xn[mt][1];
            if (S::DX == 2) {
                xn[mt][0] = xnn[mt][0];
                xn[mt][1] = xnn[mt][1];
            }
        }
    }

    // ---- the eight warps' partial sums, added through shared memory (the ring is free: every stage was consumed) ----
    named_barrier(1, 32 * QQ_CW);
    float* red = reinterpret_cast<float*>(smem);  // [warp][token][FR * 16 rows + pad]
#pragma unroll
    for (int f = 0; f < FR; ++f)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = 16 * f + g + 8 * (e >> 1), tok = 8 * mt + 2 * t + (e & 1);
                red[(warp * S::MTOK + tok) * S::RRP + row] = acc[f][mt][e];
            }
    named_barrier(1, 32 * QQ_CW);
    const int R = nf * 16;
    for (int idx = threadIdx.x; idx < R * mv; idx += 32 * QQ_CW) {
        const int tok = idx / R, row = idx - tok * R;
        const int n = row0 + row;
        if (n >= a.N) continue;
        float p[QQ_CW];  // the eight partial sums loaded together, then added as a tree
#pragma unroll
        for (int w = 0; w < QQ_CW; ++w) p[w] = red[(w * S::MTOK + tok) * S::RRP + row];
        const float v = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
        if (ok) qq_store(a, tok, n, v, kBF16);
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------

template <typename T, int MT, int FR, bool SXA>
static int qmvq_launch_t(const void* x, const uint32_t* w, QqArgs a, int ns_req, int nctas, cudaStream_t st) {
    using S = QqShape<MT, FR>;
    const DeviceInfo& di = device_info();
    const int K = a.K;
    // stages: within half an SM's shared memory, so the next launch's CTA can start beside a running one
    const size_t fixed = 2 * QQ_MAX_STAGES * 8 + 1024;
    const size_t budget = di.smem_per_sm / 2 - 1024;
    int ns = int((budget - fixed) / S::STAGE_BYTES);
    if (ns > QQ_MAX_STAGES) ns = QQ_MAX_STAGES;
    if (ns > a.nchunk) ns = a.nchunk;
    if (ns_req > 0 && ns_req < ns) ns = ns_req;
    if (ns < 1) return LQ_E_SHAPE;
    a.ns = ns;
    size_t ring = size_t(ns) * S::STAGE_BYTES;
    if (ring < size_t(S::RED_BYTES)) ring = S::RED_BYTES;
    const size_t smem = ring + fixed;
    if (smem > di.smem_optin) return LQ_E_SHAPE;
    if (a.cpw && ns < a.nchunk) a.cpw = 0;  // consumer-copied weights: only when the ring holds every stage

    // weight boxes of 16 FR rows (CTAs holding FR fragments) and 16 (FR - 1) rows (the others); two 128-byte
    // segments a stage
    CUtensorMap tw[2];
    for (int m = 0; m < 2; ++m) {
        const int rows = 16 * (m == 0 || FR == 1 ? FR : FR - 1);
        const uint64_t dims[3] = {32, uint64_t(a.N), uint64_t(K) / 256};
        const uint64_t str[2] = {uint64_t(K) / 2, 128};
        const uint32_t box[3] = {32, uint32_t(rows), 2};
        const int rc = make_tmap(&tw[m], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, w, dims, str, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    a.x = x;
    a.w = w;
    const int kg = a.kg;
    const uintptr_t sb_addr = reinterpret_cast<uintptr_t>(a.s) | reinterpret_cast<uintptr_t>(a.b);
    a.sb_vec = (kg % 8 == 0 && sb_addr % 16 == 0) ? 16 : (kg % 4 == 0 && sb_addr % 8 == 0) ? 8 : 4;

    auto kern = qmvq_kernel<T, MT, FR, SXA>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nctas, 1, 1);
    cfg.blockDim = dim3(QQ_THREADS, 1, 1);
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

template <typename T, int MT, bool SXA>
static int qmvq_dispatch_fr(int FR, const void* x, const uint32_t* w, const QqArgs& a, int ns, int nctas,
                            cudaStream_t st) {
    switch (FR) {
        case 1: return qmvq_launch_t<T, MT, 1, SXA>(x, w, a, ns, nctas, st);
        case 2: return qmvq_launch_t<T, MT, 2, SXA>(x, w, a, ns, nctas, st);
        case 3: return qmvq_launch_t<T, MT, 3, SXA>(x, w, a, ns, nctas, st);
        case 4: return qmvq_launch_t<T, MT, 4, SXA>(x, w, a, ns, nctas, st);
        default: return LQ_E_SHAPE;
    }
}

template <typename T, int MT>
static int qmvq_dispatch_sx(bool sxa, int FR, const void* x, const uint32_t* w, const QqArgs& a, int ns, int nctas,
                            cudaStream_t st) {
    return sxa ? qmvq_dispatch_fr<T, MT, true>(FR, x, w, a, ns, nctas, st)
               : qmvq_dispatch_fr<T, MT, false>(FR, x, w, a, ns, nctas, st);
}

bool qmvq_shape_ok(int M, int K, int bits) { return bits == 4 && M >= 1 && M <= 16 && K >= 256 && K % 256 == 0; }

// p = {FR (max fragments a CTA, 0 = spread over every SM), NS (stages, 0 = choose), LOADER (weights: 0 = choose,
// 1 = TMA by the producer warp, 2 = cp.async by the consumer threads), SX (group x sums: 0 = choose, 1 = by an
// all-ones MMA, 2 = by fp32 adds and shuffles)}.
int qmvq_run(const void* x, const uint32_t* w, const void* s, const void* b, int nout, void* const* outs,
             const int* seg_end, const int* ldo, int M, int N, int K, int dtype, const int* p, cudaStream_t st) {
    if (!qmvq_shape_ok(M, K, 4) || N < 1) return LQ_E_SHAPE;
    QqArgs a = {};
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
    const int ldm = p ? p[2] : 0;
    const int sxm = p ? p[3] : 0;
    if (fr_req < 0 || fr_req > QQ_MAX_FR || ns < 0 || ldm < 0 || ldm > 2 || sxm < 0 || sxm > 2) return LQ_E_ARG;
    a.cpw = ldm == 2 ? 1 : 0;
    const bool sxa = sxm == 2;
    // CTAs: at most fr fragments each; the library's choice spreads them over every SM. Then every CTA holds FR or
    // FR - 1 fragments with FR = ceil(nfrag / nctas), the two weight-box heights the kernel is given.
    int fr = fr_req;
    if (fr == 0) {
        fr = (a.nfrag + sms - 1) / sms;
        if (fr > QQ_MAX_FR) fr = QQ_MAX_FR;
    }
    int nctas = (a.nfrag + fr - 1) / fr;
    if (fr_req == 0 && nctas < sms) nctas = a.nfrag < sms ? a.nfrag : sms;
    const int FR = (a.nfrag + nctas - 1) / nctas;
    const bool bf16 = dtype == LQ_BF16;
    if (M <= 8)
        return bf16 ? qmvq_dispatch_sx<__nv_bfloat16, 1>(sxa, FR, x, w, a, ns, nctas, st)
                    : qmvq_dispatch_sx<__half, 1>(sxa, FR, x, w, a, ns, nctas, st);
    return bf16 ? qmvq_dispatch_sx<__nv_bfloat16, 2>(sxa, FR, x, w, a, ns, nctas, st)
                : qmvq_dispatch_sx<__half, 2>(sxa, FR, x, w, a, ns, nctas, st);
}

}  // namespace lq
