// Decode with the codes fed raw to the MMA and scale and bias folded per group in fp32 ("qmvq" family):
// y (M, N) = x (M, K) . dequant(W)^T for M <= 16 tokens, 4- or 8-bit codes, one matrix or a gate/up pair with the
// SwiGLU epilogue. The B200 counterpart of the reference's fragq kernel (locals/qmv_frag.py:368-540): there the codes
// enter the 8x8 MMA as 1 + q/16 in the mantissa and each group's scale and bias are applied to the fp32 partial sum;
// here they enter mma.sync.m16n8k16 as magic + q -- magic = 128 in bf16, 1024 in fp16, one lop3 a code pair, no
// subtract, no fma -- and each 64-wide group ends with
//     y += s * acc + (b - magic * s) * sum(x)                       (4-bit: acc = sum((magic + q) x))
//     y += s * (16 acc_hi + acc_lo) + (b - 17 magic s) * sum(x)      (8-bit: the high and low nibbles of each code
//                                                                     enter two MMAs as magic + nibble)
// in fp32, where sum(x) is the group's x sum, taken by one more MMA with an all-ones A operand (so it lands in the
// accumulator layout the fold needs). The weights are never rounded to the activation dtype: the result is the fp32
// factoring s . sum(q x) + b . sum(x) of the reference's multi-row kernels (locals/qmv_multi.py:57-75), which is what
// mx.quantized_matmul computes.
//
// Work split: the 16-row fragments of the matrix (or the (gate, up) fragment pairs) are dealt out evenly over every SM
// (CTA c takes units [cU/C, (c+1)U/C)); one ring stage = 512 K values of all of the CTA's rows (one TMA box a matrix,
// 128-byte swizzle); consumer warp w takes group w of every stage for all of the CTA's fragments, so its x fragments
// are loaded and permuted once and reused for every fragment; the eight warps' partial sums are added through shared
// memory at the end; x is loaded by each consumer lane straight into registers ahead of its use. Nothing the producer
// loads depends on the previous kernel, so under programmatic dependent launch the ring fills while the previous
// kernel runs. Two footprints: 4-bit single matrices keep to half an SM (two CTAs an SM: the next call's CTA loads
// its weights beside the running one -- decode projections are a few MB); 8-bit matrices and gate/up pairs (tens of
// MB a call) take the whole SM for a deeper ring and more registers.
// Measured facts behind the choices (B200, CUDA graphs of weight copies larger than L2): a producer that also widened
// each stage's scales into an fp32 table was 1.8x slower (one warp doing it delays the ring and the dependent launch);
// x staged in shared memory by the lanes' own cp.async was slower than registers (7.0 and 7.3 against 4.8 us a layer
// at one token); weights copied by the 256 consumer threads before the dependency were no faster than TMA; shared
// reads as plain C++ loads were slower than these asm loads (5.10 against 4.90 us). A per-CTA %globaltimer timeline of
// the fused QKV projection at one token: the dependency resolves 0.77 us after the previous call's last CTA ends (every
// weight stage has landed by then), the first x stage 0.4 us later, five stages take 3.0 us of consumer issue (2 warps a
// scheduler, latency-bound: 29% issue active under ncu), the reduction and stores 0.6 us.
// Reference: the multi-row GEMV it replaces, locals/qmv_frag.py:368-540 (fragq) behind kernels._launcher
// (locals/kernels.py:516-576), and the fused MLP's gate/up projection (locals/fuse.py:160-164, locals/moe.py:284-289).
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
constexpr int QQ_MAX_STAGES = 8;

// Two CTAs an SM (4-bit single matrices) or one (8-bit, gate/up pairs). (A second set of eight consumer warps taking
// alternate fragments, which one CTA an SM has the registers for, measured slower on B200: 17.9 against 15.2 us for
// the 8-bit gate/up pair at one token.)
template <int BITS, int NMAT>
struct QqFoot {
    static constexpr bool kHalf = BITS == 4 && NMAT == 1;
    static constexpr int kMinBlocks = kHalf ? 2 : 1;
    static constexpr int kMaxFr = kHalf ? 4 : 6;
};

template <int BITS, int MT, int FR, int NMAT>
struct QqShape {
    static constexpr int MTOK = 8 * MT;                  // token slots
    static constexpr int RB = BITS * 64;                 // bytes of a row a stage (512 K values)
    static constexpr int SEGS = RB / 128;                // 128-byte swizzle segments a row
    static constexpr int W_FRAG = 16 * RB;               // one 16-row fragment
    static constexpr int W_MAT = FR * W_FRAG;            // one matrix's box
    static constexpr int W_BYTES = NMAT * W_MAT;
    static constexpr int SB_MAT = FR * 16 * 16;          // one matrix's scales (or biases): rows x 8 groups x 2 bytes
    static constexpr int SB_OFF = W_BYTES;               // matrix m's scales at SB_OFF + 2 m SB_MAT, biases + SB_MAT
    static constexpr int STAGE_BYTES = (W_BYTES + NMAT * 2 * SB_MAT + 1023) / 1024 * 1024;
    // the warps' partial sums [warp][token][NMAT * FR * 16 rows + 4]: the 4-float pad puts the four token columns a
    // lane quad writes at once 8 banks apart, so every partial-sum store of a warp is free of bank conflicts
    static constexpr int RRP = NMAT * FR * 16 + 4;
    static constexpr int RED_BYTES = QQ_CW * MTOK * RRP * 4;
    static constexpr int PART_BYTES = NMAT * MTOK * FR * 16 * 4;  // a K slice's sums [matrix][token][FR * 16 rows]
    // x loaded DX stages ahead of its use: two for up to 8 tokens, one for 16 (the register budget)
    static constexpr int DX = MT == 1 ? 2 : 1;
    static_assert(W_FRAG % 1024 == 0, "1 KB alignment of swizzled tiles");
};

struct QqArgs {
    int M, N, K;   // N: rows of each matrix
    int kg;        // groups a row (K / 64)
    int nchunk;    // stages of 512 K values
    int units;     // 16-row fragments of each matrix (ceil(N / 16))
    int ns;        // ring depth
    int ks;        // K slices: a thread-block cluster of ks CTAs along y shares the units, each a run of stages
    int sb_vec;    // cp.async width for scale / bias rows
    const void* x;
    const void* s[2];
    const void* b[2];
    void* out[3];  // output column segments (fused q / k / v), or out[0] only (h for gate/up pairs)
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

__device__ __forceinline__ uint4 qq_lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
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

template <typename T>
__device__ __forceinline__ float qq_round(float v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __bfloat162float(__float2bfloat16_rn(v));
    else
        return __half2float(__float2half_rn(v));
}

// silu(g) * u with the activation-dtype rounding points of locals/moe.py:284-289 (the store rounds the product)
template <typename T>
__device__ __forceinline__ float qq_swiglu(float g, float u) {
    const float gt = qq_round<T>(g), ut = qq_round<T>(u);
    const float sig = qq_round<T>(1.0f / (1.0f + expf(-gt)));
    return qq_round<T>(gt * sig) * ut;
}

// SXA: the group's x sums by fp32 adds and quad shuffles (true) or by an MMA with an all-ones A operand (false).
// Matrix m's weight boxes: tm0 / tm2 (CTAs holding FR units) and tm1 / tm3 (FR - 1 units).
template <typename T, int BITS, int MT, int FR, int NMAT, bool SXA>
__global__ void __launch_bounds__(QQ_THREADS, QqFoot<BITS, NMAT>::kMinBlocks)
    qmvq_kernel(const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1,
                const __grid_constant__ CUtensorMap tm2, const __grid_constant__ CUtensorMap tm3, const QqArgs a) {
    using S = QqShape<BITS, MT, FR, NMAT>;
    using TR = F16Traits<T>;
    using MG = QqMagic<T>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr int RING_MIN = S::RED_BYTES;  // the ring is reused for the partial sums
    constexpr float kFold = BITS == 4 ? MG::kVal : 17.0f * MG::kVal;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int ns = a.ns;
    const int ring = ns * S::STAGE_BYTES > RING_MIN ? ns * S::STAGE_BYTES : RING_MIN;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring);
    uint64_t* empty = full + QQ_MAX_STAGES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // units [u0, u0 + nu): a CTA holds FR or FR - 1 of them (host-chosen grid)
    const int u0 = int((long long)blockIdx.x * a.units / gridDim.x);
    const int nu = int((long long)(blockIdx.x + 1) * a.units / gridDim.x) - u0;
    if (nu < 1 || nu > FR || nu < FR - 1) {  // the weight boxes hold 16 FR or 16 (FR - 1) rows: nothing else fits
        if (threadIdx.x == 0) record_status(LQ_DEV_BOUNDS);
        return;
    }
    const int row0 = 16 * u0;
    // this CTA's K slice: stages [c0, c0 + total) of the cluster's units
    const int ks = a.ks;
    const int krank = ks > 1 ? int(cluster_ctarank()) : 0;
    const int c0 = (a.nchunk * krank) / ks;
    const int total = (a.nchunk * (krank + 1)) / ks - c0;
    const int mv = a.M < S::MTOK ? a.M : S::MTOK;  // real token rows

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; ++s) {
            mbar_init(&full[s], 1 + 32);  // lane 0's expect_tx arrive + 32 cp.async arrivals
            mbar_init(&empty[s], QQ_CW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    bool ok = true;

    if (warp == QQ_CW) {
        // ------------------------------ producer warp ------------------------------
        const uint64_t pol_w = policy_evict_first();
        const CUtensorMap* tmw[2] = {nu == FR ? &tm0 : &tm1, nu == FR ? &tm2 : &tm3};
        if (lane == 0) {
            prefetch_tmap(tmw[0]);
            if (NMAT == 2) prefetch_tmap(tmw[1]);
        }
        const uint32_t smem_base = smem_u32(smem);
        const int vb = a.sb_vec;
        const int units = 16 / vb;
        auto load = [&](int c, int s) {
            uint8_t* st = smem + s * S::STAGE_BYTES;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], NMAT * nu * S::W_FRAG);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
                    tma_load_3d(st + m * S::W_MAT, tmw[m], &full[s], 0, row0, S::SEGS * c, pol_w);
            }
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const uint32_t sdst = smem_base + s * S::STAGE_BYTES + S::SB_OFF + m * 2 * S::SB_MAT;
                for (int r = lane; r < nu * 16; r += 32) {
                    const int grow = row0 + r;
                    for (int u = 0; u < units; ++u) {
                        const int gcol = 8 * c + u * (vb >> 1);
                        const bool valid = grow < a.N && gcol < a.kg;
                        const size_t off = valid ? (size_t(grow) * a.kg + gcol) * 2 : 0;
                        const uint32_t d = sdst + r * 16 + u * vb;
                        cp_async(d, reinterpret_cast<const uint8_t*>(a.s[m]) + off, vb, valid);
                        cp_async(d + S::SB_MAT, reinterpret_cast<const uint8_t*>(a.b[m]) + off, vb, valid);
                    }
                }
            }
            cp_async_arrive(&full[s]);
        };
        const int pre = total < ns ? total : ns;
        for (int i = 0; i < pre; ++i) load(c0 + i, i);  // (weights and scales only: nothing here waits for the
                                                        // previous kernel)
        if (lane == 0) grid_dep_launch();
        for (int i = pre; i < total; ++i) {
            const int s = i % ns;
            ok = mbar_wait(&empty[s], ((i / ns) - 1) & 1);
            if (!ok) break;
            load(c0 + i, s);
        }
        __syncwarp();
        if (ks == 1) return;
        grid_dep_wait();  // (before the cluster's output stores)
    } else {

    // ------------------------------ consumer warps ------------------------------
    grid_dep_wait();  // x may be the previous kernel's output (and before any output store of this kernel)
    const int g = lane >> 2, t = lane & 3;
    const uint32_t smem_base = smem_u32(smem);
    float acc[NMAT][FR][MT][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int f = 0; f < FR; ++f)
#pragma unroll
            for (int q = 0; q < MT; ++q)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[m][f][q][e] = 0.0f;

    // The row of a fragment this lane reads (and r + 8): 4-bit lanes read 8 bytes of row g; 8-bit lanes read 16 bytes
    // of row (g >> 1) | ((g & 1) << 2), so the two rows a quarter-warp reads at once sit in different halves of the
    // 128-byte swizzle atom (no bank conflicts); the MMA's row g then holds that weight row.
    const int r_lo = BITS == 4 ? g : ((g >> 1) | ((g & 1) << 2));
    // this lane's bytes of a row inside group w of a stage (128-byte swizzle: 16-byte chunk c of row r sits at
    // c ^ (r & 7)); a matrix's box is [segment][16 nu rows][128 bytes], fragment f's rows at 2048 f of each segment
    const uint32_t w_off = BITS == 4
                               ? (warp >> 2) * (nu * 2048) + r_lo * 128 + (((2 * (warp & 3) + (t >> 1)) ^ r_lo) << 4) +
                                     8 * (t & 1)
                               : (warp >> 1) * (nu * 2048) + r_lo * 128 + (((4 * (warp & 1) + t) ^ r_lo) << 4);
    // x of stage i's group for this lane: values 16t .. 16t + 15 of tokens g + 8 mt (zero past M and past K), loaded
    // straight into registers ahead of its use. Token columns past M keep whatever their registers held: an MMA's
    // output column n depends on its input column n only (the x sums too), and those columns are never stored. Stages
    // past K are skipped whole.
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(a.x);
    auto fetch_x = [&](int i, uint4 (&u)[MT][2]) {
        const int gi = 8 * (c0 + i) + warp;
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
        if (ok && 8 * (c0 + i) + warp < a.kg) {
            const uint32_t st = smem_base + s * S::STAGE_BYTES;
            // x fragments of group w permuted to the code order of a k16 step, and the group's x sums in the
            // accumulator layout (sx[mt][e] = sum(x) of token column 2t + (e & 1); rows are alike, entries 2 and 3 go
            // unused). 4-bit: step s takes codes (p, p + 4) of word s / 2 (p = 2 (s & 1), + 1), i.e. x words
            // (s / 2 * 4 + s % 2, + 2); 8-bit: step s takes word s's bytes (0, 2) and (1, 3), i.e. x words (2s, 2s + 1).
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
                if constexpr (SXA) {
                    // this lane's 16 values of token g + 8 mt, then the quad's 64, then moved to columns 2t, 2t + 1
                    float sum = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) sum += TR::to_f32(xw[j] & 0xFFFFu) + TR::to_f32(xw[j] >> 16);
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
            // All fragments run without a branch (one straight block). A CTA holding nu = FR - 1 units computes one
            // extra fragment a matrix from stale bytes of its own stage: every address stays inside the stage's
            // weight boxes and tables, and its partial sums land in reduction rows the final sum never reads.
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const uint32_t sb = st + S::SB_OFF + m * 2 * S::SB_MAT + 2 * warp;  // group w's scale of row r: sb + 16 r
#pragma unroll
                for (int f = 0; f < FR; ++f) {
                    const uint32_t fb = st + m * S::W_MAT + f * 2048 + w_off;
                    // rows r_lo and r_lo + 8: s and b - fold * s in fp32
                    const int ra = 16 * f + r_lo, rb = ra + 8;
                    const float sa = TR::to_f32(lds_u16(sb + ra * 16)), sbb = TR::to_f32(lds_u16(sb + rb * 16));
                    const float ca = fmaf(-kFold, sa, TR::to_f32(lds_u16(sb + S::SB_MAT + ra * 16)));
                    const float cb = fmaf(-kFold, sbb, TR::to_f32(lds_u16(sb + S::SB_MAT + rb * 16)));
                    float part[MT][4];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) part[mt][e] = 0.0f;
                    if constexpr (BITS == 4) {
                        const uint2 wa = qq_lds64(fb), wb = qq_lds64(fb + 8 * 128);
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
                    } else {
                        // 16 codes a row: word s holds the codes of step s, bytes (0, 2) and (1, 3) the MMA's k pairs
                        const uint4 wa = qq_lds128(fb), wb = qq_lds128(fb + 8 * 128);
                        const uint32_t va4[4] = {wa.x, wa.y, wa.z, wa.w}, vb4[4] = {wb.x, wb.y, wb.z, wb.w};
                        float hi[MT][4];
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int e = 0; e < 4; ++e) hi[mt][e] = 0.0f;
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
                            for (int mt = 0; mt < MT; ++mt) {
                                qq_mma<T>(part[mt], l0, l1, l2, l3, xb[mt][step][0], xb[mt][step][1]);
                                qq_mma<T>(hi[mt], h0, h1, h2, h3, xb[mt][step][0], xb[mt][step][1]);
                            }
                        }
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int e = 0; e < 4; ++e) part[mt][e] = fmaf(16.0f, hi[mt][e], part[mt][e]);
                    }
                    // y += s * acc + (b - fold s) * sum(x), rows r_lo (a) and r_lo + 8 (b)
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
            if (S::DX == 2) {
                xn[mt][0] = xnn[mt][0];
                xn[mt][1] = xnn[mt][1];
            }
        }
    }

    // ---- the eight warps' partial sums, added through shared memory (the ring is free: every stage was consumed) ----
    named_barrier(1, 32 * QQ_CW);
    float* red = reinterpret_cast<float*>(smem);  // [warp][token][NMAT * FR * 16 rows + pad]
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int f = 0; f < FR; ++f)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int row = (m * FR + f) * 16 + r_lo + 8 * (e >> 1), tok = 8 * mt + 2 * t + (e & 1);
                    red[(warp * S::MTOK + tok) * S::RRP + row] = acc[m][f][mt][e];
                }
    named_barrier(1, 32 * QQ_CW);
    auto sum_warps = [&](int tok, int row) {
        float p[QQ_CW];  // the eight partial sums loaded together, then added as a tree
#pragma unroll
        for (int w = 0; w < QQ_CW; ++w) p[w] = red[(w * S::MTOK + tok) * S::RRP + row];
        return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
    };
    const int R = nu * 16;
    if (ks == 1) {
        for (int idx = threadIdx.x; idx < R * mv; idx += 32 * QQ_CW) {
            const int tok = idx / R, row = idx - tok * R;
            const int n = row0 + row;
            if (n >= a.N) continue;
            float v;
            if constexpr (NMAT == 2)
                v = qq_swiglu<T>(sum_warps(tok, row), sum_warps(tok, FR * 16 + row));
            else
                v = sum_warps(tok, row);
            if (ok) qq_store(a, tok, n, v, kBF16);
        }
        return;
    }
    // K slices: this CTA's sums [matrix][token][FR * 16 rows] after the warps' table, for the cluster to add
    float* part = red + S::RED_BYTES / 4;
    for (int idx = threadIdx.x; idx < NMAT * mv * R; idx += 32 * QQ_CW) {
        const int m = idx / (mv * R), rem = idx - m * (mv * R), tok = rem / R, row = rem - tok * R;
        part[(m * S::MTOK + tok) * (FR * 16) + row] = ok ? sum_warps(tok, m * FR * 16 + row) : 0.0f;
    }
    }  // (consumer warps)

    // ------------------ the K slices added over the cluster (distributed shared memory) ------------------
    cluster_sync();
    const uint32_t part_local = smem_u32(smem) + S::RED_BYTES;
    uint32_t peer[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) peer[q] = map_peer(part_local, q < ks ? q : 0);
    const int R = nu * 16;
    for (int idx = krank * QQ_THREADS + int(threadIdx.x); idx < R * mv; idx += ks * QQ_THREADS) {
        const int tok = idx / R, row = idx - tok * R;  // consecutive threads: consecutive output columns
        const int n = row0 + row;
        if (n >= a.N) continue;
        // every slice's partial requested before any is added (one round of remote latency); slices in rank order
        float v[8], u[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            v[q] = q < ks ? ld_dsmem_f(peer[q] + 4 * (tok * (FR * 16) + row)) : 0.0f;
            if constexpr (NMAT == 2) u[q] = q < ks ? ld_dsmem_f(peer[q] + 4 * ((S::MTOK + tok) * (FR * 16) + row)) : 0.0f;
        }
        float g0 = 0.0f, u0s = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            g0 += v[q];
            if constexpr (NMAT == 2) u0s += u[q];
        }
        if constexpr (NMAT == 2) g0 = qq_swiglu<T>(g0, u0s);
        if (ok) qq_store(a, tok, n, g0, kBF16);
    }
    cluster_sync();  // the slices keep their shared memory until every CTA of the cluster has read it
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------

template <typename T, int BITS, int MT, int FR, int NMAT, bool SXA>
static int qmvq_launch_t(const uint32_t* const* w, QqArgs a, int ns_req, int nctas, cudaStream_t st) {
    using S = QqShape<BITS, MT, FR, NMAT>;
    const DeviceInfo& di = device_info();
    const int K = a.K;
    // stages: half an SM's shared memory for the two-CTA footprint (so the next call's CTA can start beside a running
    // one), else the whole SM
    const size_t fixed = 2 * QQ_MAX_STAGES * 8 + 1024;
    const size_t budget = QqFoot<BITS, NMAT>::kHalf ? di.smem_per_sm / 2 - 1024 : di.smem_optin;
    int ns = budget > fixed ? int((budget - fixed) / S::STAGE_BYTES) : 0;
    if (ns > QQ_MAX_STAGES) ns = QQ_MAX_STAGES;
    if (ns > a.nchunk) ns = a.nchunk;
    if (ns_req > 0 && ns_req < ns) ns = ns_req;
    if (ns < 1) return LQ_E_SHAPE;
    a.ns = ns;
    size_t ring = size_t(ns) * S::STAGE_BYTES;
    const size_t red_need = size_t(S::RED_BYTES) + (a.ks > 1 ? size_t(S::PART_BYTES) : 0);
    if (ring < red_need) ring = red_need;
    const size_t smem = ring + fixed;
    if (smem > di.smem_optin) return LQ_E_SHAPE;

    // weight boxes of 16 FR rows (CTAs holding FR units) and 16 (FR - 1) rows (the others) for each matrix; S::SEGS
    // 128-byte segments a stage
    CUtensorMap tw[4];
    for (int m = 0; m < 2; ++m)
        for (int h = 0; h < 2; ++h) {
            const int rows = 16 * (h == 0 || FR == 1 ? FR : FR - 1);
            const uint64_t dims[3] = {32, uint64_t(a.N), uint64_t(K) * BITS / 1024};
            const uint64_t str[2] = {uint64_t(K) * BITS / 8, 128};
            const uint32_t box[3] = {32, uint32_t(rows), uint32_t(S::SEGS)};
            const int rc = make_tmap(&tw[2 * m + h], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, w[m < NMAT ? m : 0], dims, str,
                                     box, CU_TENSOR_MAP_SWIZZLE_128B);
            if (rc) return rc;
        }
    const int kg = a.kg;
    uintptr_t sb_addr = 0;
    for (int m = 0; m < NMAT; ++m)
        sb_addr |= reinterpret_cast<uintptr_t>(a.s[m]) | reinterpret_cast<uintptr_t>(a.b[m]);
    a.sb_vec = (kg % 8 == 0 && sb_addr % 16 == 0) ? 16 : (kg % 4 == 0 && sb_addr % 8 == 0) ? 8 : 4;

    auto kern = qmvq_kernel<T, BITS, MT, FR, NMAT, SXA>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return LQ_E_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nctas, a.ks, 1);
    cfg.blockDim = dim3(QQ_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int na = 1;
    if (a.ks > 1) {  // the K slices of a unit range form one cluster along y
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1;
        attr[1].val.clusterDim.y = a.ks;
        attr[1].val.clusterDim.z = 1;
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    e = cudaLaunchKernelEx(&cfg, kern, tw[0], tw[1], tw[2], tw[3], a);
    return e == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

template <typename T, int BITS, int MT, int NMAT, bool SXA>
static int qmvq_dispatch_fr(int FR, const uint32_t* const* w, const QqArgs& a, int ns, int nctas, cudaStream_t st) {
    switch (FR) {
        case 1: return qmvq_launch_t<T, BITS, MT, 1, NMAT, SXA>(w, a, ns, nctas, st);
        case 2: return qmvq_launch_t<T, BITS, MT, 2, NMAT, SXA>(w, a, ns, nctas, st);
        case 3: return qmvq_launch_t<T, BITS, MT, 3, NMAT, SXA>(w, a, ns, nctas, st);
        case 4: return qmvq_launch_t<T, BITS, MT, 4, NMAT, SXA>(w, a, ns, nctas, st);
        case 5:
            if constexpr (QqFoot<BITS, NMAT>::kMaxFr >= 5) return qmvq_launch_t<T, BITS, MT, 5, NMAT, SXA>(w, a, ns, nctas, st);
            return LQ_E_SHAPE;
        case 6:
            if constexpr (QqFoot<BITS, NMAT>::kMaxFr >= 6) return qmvq_launch_t<T, BITS, MT, 6, NMAT, SXA>(w, a, ns, nctas, st);
            return LQ_E_SHAPE;
        default: return LQ_E_SHAPE;
    }
}

// x sums by adds are built for the 4-bit single-matrix kernels only (the all-ones MMA elsewhere)
template <typename T, int BITS, int MT, int NMAT>
static int qmvq_dispatch_sx(bool sxa, int FR, const uint32_t* const* w, const QqArgs& a, int ns, int nctas,
                            cudaStream_t st) {
    if constexpr (BITS == 4 && NMAT == 1)
        if (sxa) return qmvq_dispatch_fr<T, BITS, MT, NMAT, true>(FR, w, a, ns, nctas, st);
    return qmvq_dispatch_fr<T, BITS, MT, NMAT, false>(FR, w, a, ns, nctas, st);
}

template <typename T, int NMAT>
static int qmvq_dispatch(int bits, int M, bool sxa, int FR, const uint32_t* const* w, const QqArgs& a, int ns,
                         int nctas, cudaStream_t st) {
    if (bits == 4)
        return M <= 8 ? qmvq_dispatch_sx<T, 4, 1, NMAT>(sxa, FR, w, a, ns, nctas, st)
                      : qmvq_dispatch_sx<T, 4, 2, NMAT>(sxa, FR, w, a, ns, nctas, st);
    return M <= 8 ? qmvq_dispatch_sx<T, 8, 1, NMAT>(sxa, FR, w, a, ns, nctas, st)
                  : qmvq_dispatch_sx<T, 8, 2, NMAT>(sxa, FR, w, a, ns, nctas, st);
}

bool qmvq_shape_ok(int M, int K, int bits) {
    return (bits == 4 || bits == 8) && M >= 1 && M <= 16 && K >= 256 && K % 256 == 0;
}

// The grid and fragment count of a call: CTAs of at most fr units each (0 = spread over every SM); every CTA then
// holds FR or FR - 1 units with FR = ceil(units / nctas), the two weight-box heights the kernel is given. With
// ks K slices (clusters of ks CTAs along y) the unit CTAs are fewer: about sms / ks of them.
static int qmvq_grid(int units, int fr_req, int max_fr, int ks, int* nctas) {
    const int sms = device_info().sm_count;
    const int slots = sms / ks > 0 ? sms / ks : 1;
    int fr = fr_req;
    if (fr == 0) {
        fr = (units + slots - 1) / slots;
        if (fr > max_fr) fr = max_fr;
    }
    int n = (units + fr - 1) / fr;
    if (fr_req == 0 && n < slots) n = units < slots ? units : slots;
    *nctas = n;
    return (units + n - 1) / n;
}

// K slices for the library's choice: the fewest stage-fragments a CTA (units a CTA x stages a slice) with the grid
// within one CTA an SM (clusters of at most 8); a tie keeps fewer slices. Long-K matrices with few rows gain: the
// 2560 x 9728 down projection goes from 2 units x 19 stages a CTA to 6 x 4.
static int qmvq_choose_ks(int units, int nchunk, int max_fr) {
    const int sms = device_info().sm_count;
    int best_ks = 1;
    long best = -1;
    for (int ks = 1; ks <= 8 && ks <= nchunk; ++ks) {
        const int slots = sms / ks;
        const int fr = (units + slots - 1) / slots;
        if (fr > max_fr) continue;
        const long work = long(fr) * ((nchunk + ks - 1) / ks);
        if (best < 0 || work < best) {
            best = work;
            best_ks = ks;
        }
    }
    return best_ks;
}

static int qmvq_common(int nmat, const void* x, const uint32_t* const* w, const void* const* s, const void* const* b,
                       int nout, void* const* outs, const int* seg_end, const int* ldo, int M, int N, int K, int bits,
                       int dtype, const int* p, cudaStream_t st) {
    if (!qmvq_shape_ok(M, K, bits) || N < 1) return LQ_E_SHAPE;
    QqArgs a = {};
    a.M = M;
    a.N = N;
    a.K = K;
    a.kg = K / 64;
    a.nchunk = (K + 511) / 512;
    a.units = (N + 15) / 16;
    a.x = x;
    for (int m = 0; m < nmat; ++m) {
        a.s[m] = s[m];
        a.b[m] = b[m];
    }
    for (int i = 0; i < nout; ++i) {
        a.out[i] = outs[i];
        a.seg_end[i] = seg_end[i];
        a.ldo[i] = ldo[i];
    }
    a.nseg_out = nout;
    const int fr_req = p ? p[0] : 0;
    const int ns = p ? p[1] : 0;
    const int ks_req = p ? p[2] : 0;
    const int sxm = p ? p[3] : 0;
    const int max_fr = (bits == 4 && nmat == 1) ? QqFoot<4, 1>::kMaxFr : QqFoot<8, 1>::kMaxFr;
    if (fr_req < 0 || fr_req > max_fr || ns < 0 || ks_req < 0 || ks_req > 8 || sxm < 0 || sxm > 2) return LQ_E_ARG;
    a.ks = ks_req > 0 ? ks_req : (fr_req > 0 ? 1 : qmvq_choose_ks(a.units, a.nchunk, max_fr));
    if (a.ks > a.nchunk) a.ks = a.nchunk;
    int nctas = 0;
    const int FR = qmvq_grid(a.units, fr_req, max_fr, a.ks, &nctas);
    if (FR > max_fr) return LQ_E_SHAPE;
    const bool bf16 = dtype == LQ_BF16, sxa = sxm == 2;
    if (nmat == 1)
        return bf16 ? qmvq_dispatch<__nv_bfloat16, 1>(bits, M, sxa, FR, w, a, ns, nctas, st)
                    : qmvq_dispatch<__half, 1>(bits, M, sxa, FR, w, a, ns, nctas, st);
    return bf16 ? qmvq_dispatch<__nv_bfloat16, 2>(bits, M, sxa, FR, w, a, ns, nctas, st)
                : qmvq_dispatch<__half, 2>(bits, M, sxa, FR, w, a, ns, nctas, st);
}

// p = {FR (max units a CTA, 0 = spread over every SM), NS (stages, 0 = choose), KS (K slices reduced over a cluster,
// 1-8, 0 = choose), SX (group x sums: 0 = choose, 1 = by an all-ones MMA, 2 = by fp32 adds and shuffles, 4-bit only)}.
int qmvq_run(const void* x, const uint32_t* w, const void* s, const void* b, int nout, void* const* outs,
             const int* seg_end, const int* ldo, int M, int N, int K, int bits, int dtype, const int* p,
             cudaStream_t st) {
    const uint32_t* ws[2] = {w, w};
    const void* ss[2] = {s, s};
    const void* bs[2] = {b, b};
    return qmvq_common(1, x, ws, ss, bs, nout, outs, seg_end, ldo, M, N, K, bits, dtype, p, st);
}

// h (M, I) = swiglu(x . gate^T, x . up^T) with the rounding points of locals/moe.py:284-289.
int qmvq_glu_run(const void* x, const uint32_t* w_gate, const void* s_gate, const void* b_gate, const uint32_t* w_up,
                 const void* s_up, const void* b_up, void* h, int M, int I, int K, int bits, int dtype, const int* p,
                 cudaStream_t st) {
    const uint32_t* ws[2] = {w_gate, w_up};
    const void* ss[2] = {s_gate, s_up};
    const void* bs[2] = {b_gate, b_up};
    void* outs[1] = {h};
    const int seg_end[1] = {I}, ldo[1] = {I};
    return qmvq_common(2, x, ws, ss, bs, 1, outs, seg_end, ldo, M, I, K, bits, dtype, p, st);
}

}  // namespace lq
