// One token's whole routed MoE layer in ONE launch (decode at batch 1): router logits and top-k, every routed slot's
// gate/up projections with SwiGLU, its down projection, and the weighted combine of the k slots. The unfused form is
// locals/moe.py:86-165 (routing) and locals/moe.py:243-349 (the per-slot decode experts and the combine); the
// library's unfused kernels are lq_moe_route, lq_moe_experts and lq_moe_down_combine.
//
// Grid (CS, C, k), clusters of CS = 8 CTAs along x, 512 threads (16 warps); slot j = blockIdx.z, K slice
// c = blockIdx.y of C, cluster rank t = blockIdx.x. At config 4 (E 64, k 4, D 2048, I 768, 4-bit) C = 4: 128 CTAs.
//   * Routing, in every cluster: CTA t stages the router rows of experts [t EC, (t + 1) EC) (EC = ceil(E / CS))
//     BEFORE waiting for the previous kernel (they do not depend on it), computes their float32 logits with the
//     library's one router dot product (moe_route.cuh) and stores them into every peer's shared memory; after a
//     cluster barrier every CTA runs the softmax / sigmoid top-k of lq_moe_route on all E logits: every CTA knows
//     the k experts and weights, bit-identical to lq_moe_route's. CTA (0, 0, 0) writes them out.
//   * Weights: with e = inds[j], the CTA copies (cp.async, all in flight together) gate and up rows
//     [c I/C + t R, + R) (R = I / (C CS)) and down rows [t D/CS, + D/CS) restricted to the K slice
//     [c I/C, (c + 1) I/C) into shared memory -- about 83 KB a CTA at config 4, so the layer's whole weight stream
//     (10.6 MB) is requested at once.
//   * Gate/up: mma.sync m16n8k16 with the 4-bit codes entering the tensor core as magic + q (one lop3 per two codes)
//     and each 64-group's scale and bias folded after its four MMAs: y += s acc + (b - magic s) sum_group(x). The
//     MMA's k order is a permutation of the group's 64 positions, applied to x (fragments built once) and to the
//     codes alike. The 16 warps split K and their partial sums are added in warp order; h = swiglu with the
//     activation-dtype rounding points of locals/moe.py:284-289.
//   * Down: each CTA stores its R values of h into every peer's copy of the cluster's h slice (I/C values); warp w
//     computes row tiles w, w + 16, ... of the CTA's D/CS rows over the whole K slice and stores float32 partial sums.
//   * Combine: the last CTA to finish row block t (a per-block atomic counter: no CTA waits for another) adds each
//     slot's C partials in slice order, rounds the slot's output to the activation dtype and sums w_j y_j in slot
//     order in float32 (locals/moe.py:339-348), stores y and resets the counter to zero for the next launch.
// The only waits are the cluster's own hardware barriers and cp.async completion.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"
#include "lq_status.cuh"
#include "moe_route.cuh"

namespace lq {

constexpr int MD_CS = 8;  // CTAs a cluster (portable cluster size)
constexpr int MD_WARPS = 16;
constexpr int MD_THREADS = 32 * MD_WARPS;
constexpr int MD_RT_MAX = 4;                       // gate/up row tiles of 16 a CTA (R <= 64)
constexpr size_t MD_ROUTER_STAGE_MAX = 64 * 1024;  // router rows staged in shared memory up to this size
constexpr int MD_MAX_E = 1024;
constexpr int MD_MAX_K = 32;

struct MdArgs {
    const void* x;   // (1, D) activation dtype
    const void* rw;  // router (E, D), fp16 or bf16
    int x_dt, rw_dt;
    const uint32_t* w[3];  // gate (E, I, D/8), up (E, I, D/8), down (E, D, I/8) packed 4-bit codes
    const void* s[3];      // scales (E, rows, K/64), activation dtype
    const void* b[3];      // biases
    void* y;               // (1, D)
    uint32_t* inds;        // optional (k) outputs: the routed experts and their weights
    float* wts;
    float* part;    // workspace: (k C, D) float32 partial sums
    uint32_t* cnt;  // workspace: CS row-block counters, zero between launches
    int E, k, D, I, mode, C, R, staged;
};

// Shared-memory layout (byte offsets), the same on host and device.
struct MdLayout {
    int gs, ds;     // gate/up row stride (padded) and down row stride (the TMA box's dense rows), bytes
    int DR, KS, gq;  // down rows a CTA, the K slice, its 64-groups
    int RT;          // gate/up row tiles of 16
    size_t o_bar, o_rw, o_x, o_xf, o_sx, o_lg, o_sel, o_gu, o_gusb, o_dw, o_dsb, o_red, o_hs, o_hf, o_hsx,
        o_flag, total;
};

__host__ __device__ inline size_t md_up16(size_t v) { return (v + 15) / 16 * 16; }

// A gate/up row stride of `bytes` (a multiple of 32) padded so that rows g = 0..3 start 8 banks apart: the 64-bit
// loads of the A fragments (lane (g, c) reads words 2c, 2c + 1 of row g) are conflict-free.
__host__ __device__ inline int md_stride(int bytes) {
    const int w = bytes / 4;
    return 4 * (w + ((w % 16) == 0 ? 8 : 0));
}

__host__ __device__ inline MdLayout md_layout(int E, int k, int D, int I, int C, int R, int staged) {
    MdLayout L = {};
    const int EC = (E + MD_CS - 1) / MD_CS;
    L.KS = I / C;
    L.gq = L.KS / 64;
    L.DR = D / MD_CS;
    L.RT = (R + 15) / 16;
    L.gs = md_stride(D / 2);
    L.ds = L.KS / 2;
    size_t o = 0;
    L.o_dw = o;  // first: the TMA destination (128-byte aligned)
    o += md_up16(size_t(L.DR) * L.ds);
    L.o_bar = o;  // [0]: the down tile and scales, [1 + t]: gate/up row tile t (tile 0 also the scale blocks)
    o += 8 * (1 + MD_RT_MAX) + 8;
    L.o_rw = o;
    o += staged ? md_up16(size_t(EC) * D * 2) : 0;
    L.o_x = o;
    o += md_up16(size_t(D) * 2);
    L.o_xf = o;
    o += size_t(D / 64) * 128;
    L.o_sx = o;
    o += md_up16(size_t(D / 64) * 4);
    L.o_lg = o;  // every expert's logit (each CTA's own written into every peer)
    o += md_up16(size_t(E) * 4);
    L.o_sel = o;
    o += md_up16(size_t(k) * 8);
    L.o_gu = o;  // the gate/up rows; the last CTA of a row block stages the slices' partial sums here
    o += size_t(2) * R * L.gs > size_t(k) * C * L.DR * 4 ? size_t(2) * R * L.gs : size_t(k) * C * L.DR * 4;
    L.o_gusb = o;  // 4 planes (gate s, gate b, up s, up b) of R rows x D/64 values
    o += size_t(4) * R * (D / 64) * 2;
    L.o_dsb = o;   // 2 planes (s, b) of DR whole rows x I/64 values
    o += size_t(2) * L.DR * (I / 64) * 2;
    L.o_red = o;
    o += size_t(MD_WARPS) * 2 * L.RT * 16 * 4;
    L.o_hs = o;
    o += md_up16(size_t(L.KS) * 2);
    L.o_hf = o;
    o += size_t(L.gq) * 128;
    L.o_hsx = o;
    o += md_up16(size_t(L.gq) * 4);
    L.o_flag = o;
    o += 16;
    L.total = o;
    return L;
}

template <typename T>
struct MdMagic;
template <>
struct MdMagic<__nv_bfloat16> {
    static constexpr uint32_t kCode2 = 0x43004300u;  // bf16x2 (128, 128): 128 + q is exact
    static constexpr float kVal = 128.0f;
};
template <>
struct MdMagic<__half> {
    static constexpr uint32_t kCode2 = 0x64006400u;  // fp16x2 (1024, 1024): 1024 + q is exact
    static constexpr float kVal = 1024.0f;
};

template <typename T>
__device__ __forceinline__ float md_round(float v) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return __bfloat162float(__float2bfloat16_rn(v));
    else
        return __half2float(__float2half_rn(v));
}

// silu(g) * u with the rounding points of locals/moe.py:284-289 (the same as the library's GLU epilogues)
template <typename T>
__device__ __forceinline__ float md_swiglu(float g, float u) {
    const float gt = md_round<T>(g), ut = md_round<T>(u);
    const float sig = md_round<T>(1.0f / (1.0f + expf(-gt)));
    return md_round<T>(gt * sig) * ut;
}

__device__ __forceinline__ uint2 md_lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// stores into a cluster peer's shared memory (addr from mapa); ordered before the peer's reads by the next
// cluster barrier (release / acquire)
__device__ __forceinline__ void md_st_dsmem_f(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void md_st_dsmem_u16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ void md_mma(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
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

// B fragments of a vector v (n 64-groups, activation-dtype bits in shared memory) and its float32 group sums. For
// group G and lane class c (lane & 3) the 8 words at frag[(4 G + c) 8 ...] are (b0, b1) of the group's MMAs m = 0..3:
// MMA m takes, in lane c's k columns (2c, 2c+1 | 2c+8, 2c+9), the positions p + (0, 4 | 1, 5) with
// p = 16 c + 8 (m >> 1) + 2 (m & 1) -- the nibbles (n, n + 4 | n + 1, n + 5), n = 2 (m & 1), of code word 2c + (m >> 1).
__device__ __forceinline__ void md_frags(const uint16_t* v, int groups, uint32_t* frag, float* gsum, int tid,
                                         int nthreads, int dt) {
    for (int it = tid; it < groups * 4; it += nthreads) {
        const int G = it >> 2, c = it & 3;
        const uint32_t* u = reinterpret_cast<const uint32_t*>(v + 64 * G + 16 * c);
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = u[i];
        uint32_t* f = frag + (4 * G + c) * 8;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int a = 4 * (m >> 1) + (m & 1);
            f[2 * m] = prmt(w[a], w[a + 2], 0x5410u);
            f[2 * m + 1] = prmt(w[a], w[a + 2], 0x7632u);
        }
    }
    for (int G = tid; G < groups; G += nthreads) {
        float s = 0.0f;
        for (int i = 0; i < 64; i += 8) {
            float f8[8];
            unpack8(*reinterpret_cast<const uint4*>(v + 64 * G + i), dt, f8);
#pragma unroll
            for (int q = 0; q < 8; ++q) s += f8[q];
        }
        gsum[G] = s;
    }
}

// One 64-group of a 16-row tile: four MMAs over the rows' code words (va: row g, vb: row g + 8; .x = word 2c,
// .y = word 2c + 1) against the group's B fragments xa (MMAs 0, 1) and xb (MMAs 2, 3); returns the raw sums of rows
// g (acc[0]) and g + 8 (acc[2]) (acc[1], acc[3] are not set).
template <typename T>
__device__ __forceinline__ void md_group(float* acc, uint2 va, uint2 vb, uint4 xa, uint4 xb) {
    constexpr uint32_t M2 = MdMagic<T>::kCode2;
    float p0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, p1[4] = {0.0f, 0.0f, 0.0f, 0.0f}, p2[4] = {0.0f, 0.0f, 0.0f, 0.0f},
          p3[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four independent MMAs (no accumulation chain), added after
    md_mma<T>(p0, lop3_and_or(va.x, 0x000F000Fu, M2), lop3_and_or(vb.x, 0x000F000Fu, M2),
              lop3_and_or(va.x >> 4, 0x000F000Fu, M2), lop3_and_or(vb.x >> 4, 0x000F000Fu, M2), xa.x, xa.y);
    md_mma<T>(p1, lop3_and_or(va.x >> 8, 0x000F000Fu, M2), lop3_and_or(vb.x >> 8, 0x000F000Fu, M2),
              lop3_and_or(va.x >> 12, 0x000F000Fu, M2), lop3_and_or(vb.x >> 12, 0x000F000Fu, M2), xa.z, xa.w);
    md_mma<T>(p2, lop3_and_or(va.y, 0x000F000Fu, M2), lop3_and_or(vb.y, 0x000F000Fu, M2),
              lop3_and_or(va.y >> 4, 0x000F000Fu, M2), lop3_and_or(vb.y >> 4, 0x000F000Fu, M2), xb.x, xb.y);
    md_mma<T>(p3, lop3_and_or(va.y >> 8, 0x000F000Fu, M2), lop3_and_or(vb.y >> 8, 0x000F000Fu, M2),
              lop3_and_or(va.y >> 12, 0x000F000Fu, M2), lop3_and_or(vb.y >> 12, 0x000F000Fu, M2), xb.z, xb.w);
    acc[0] = (p0[0] + p1[0]) + (p2[0] + p3[0]);
    acc[2] = (p0[2] + p1[2]) + (p2[2] + p3[2]);
}

// One bulk copy (no multicast) of `bytes` (a multiple of 16; both addresses 16-byte aligned) into this CTA's shared
// memory, completing on `bar`.
__device__ __forceinline__ void md_bulk(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

template <typename T>
__global__ void __launch_bounds__(MD_THREADS, 1)
    moe_decode_kernel(const __grid_constant__ CUtensorMap tm_down, const MdArgs a) {
    extern __shared__ __align__(1024) uint8_t sm[];
    constexpr float kVal = MdMagic<T>::kVal;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const int t = int(cluster_ctarank());
    const int cs = blockIdx.y, j = blockIdx.z;
    const int D = a.D, I = a.I, R = a.R, E = a.E, k = a.k;
    const MdLayout L = md_layout(E, k, D, I, a.C, R, a.staged);
    const int EC = (E + MD_CS - 1) / MD_CS, e0 = t * EC;
    const int ne = E - e0 < EC ? (E - e0 > 0 ? E - e0 : 0) : EC;
    const int dt = std::is_same<T, __nv_bfloat16>::value ? LQ_BF16 : LQ_F16;

    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.o_bar);  // [0]: down, [1 + t]: gate/up row tile t
    if (tid == 0) {
        for (int i = 0; i <= MD_RT_MAX; ++i) mbar_init(&bar[i], 1);
        fence_barrier_init();
        prefetch_tmap(&tm_down);
    }
    // every CTA of the cluster has started before any CTA stores into a peer's shared memory (waited on below)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

    // ---- routing: this CTA's router rows (independent of the previous kernel), then x and the logits ----
    const uint16_t* rrows = reinterpret_cast<const uint16_t*>(a.rw) + size_t(e0) * D;
    uint16_t* rws = reinterpret_cast<uint16_t*>(sm + L.o_rw);
    if (a.staged) {
        for (int i = tid; i < ne * D / 8; i += MD_THREADS) cp_async(smem_u32(rws + 8 * i), rrows + 8 * i, 16, true);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    grid_dep_wait();  // x may be the previous kernel's output; the workspace counters are free from here on
    grid_dep_launch();
    uint16_t* xs = reinterpret_cast<uint16_t*>(sm + L.o_x);
    for (int i = tid; i < D / 8; i += MD_THREADS)
        reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(a.x)[i];
    if (a.staged) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    float* lg = reinterpret_cast<float*>(sm + L.o_lg);
    const uint16_t* rsrc = a.staged ? rws : rrows;
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    for (int el = warp; el < ne; el += MD_WARPS) {
        const float v = router_dot(xs, a.x_dt, rsrc + size_t(el) * D, a.rw_dt, D, lane);  // (in every lane)
        if (lane < MD_CS) md_st_dsmem_f(map_peer(smem_u32(lg + e0 + el), uint32_t(lane)), v);  // lane p: into peer p
    }
    cluster_sync();  // every expert's logit is in every CTA's shared memory
    uint32_t* sel_i = reinterpret_cast<uint32_t*>(sm + L.o_sel);
    float* sel_w = reinterpret_cast<float*>(sm + L.o_sel) + k;
    uint32_t* xf = reinterpret_cast<uint32_t*>(sm + L.o_xf);
    float* sx = reinterpret_cast<float*>(sm + L.o_sx);
    if (warp == 0) {
        score_and_select([&](int e) { return lg[e]; }, E, k, a.mode, lane, sel_i, sel_w);
    } else {
        md_frags(xs, D / 64, xf, sx, tid - 32, MD_THREADS - 32, dt);
    }
    __syncthreads();
    if (blockIdx.x == 0 && cs == 0 && j == 0 && tid < k && a.inds) {
        a.inds[tid] = sel_i[tid];
        a.wts[tid] = sel_w[tid];
    }
    const int e = int(sel_i[j]);  // < E: the top-k never returns an index outside [0, E)

    // ---- every weight byte of this CTA in flight at once (warp 0), in the order they are used: gate/up row tile 0
    // with the gate/up scale blocks (bar[1]), the other row tiles (bar[1 + t]), then the down tile (one TMA box a 256
    // rows) and its whole scale rows (bar[0]) ----
    const int G = D / 64, GI = I / 64;
    const int r0 = cs * L.KS + t * R;  // first gate/up row
    const int DR = L.DR, gq = L.gq, RT = L.RT;
    const uint32_t gu = smem_u32(sm + L.o_gu), gusb = smem_u32(sm + L.o_gusb);
    const uint32_t dw = smem_u32(sm + L.o_dw), dsb = smem_u32(sm + L.o_dsb);
    const uint32_t gu_plane = uint32_t(R * G * 2), d_plane = uint32_t(DR * GI * 2);
    if (warp == 0) {
        if (lane == 0) {
            for (int tl = 0; tl < RT; ++tl) {
                const int rows = R - 16 * tl < 16 ? R - 16 * tl : 16;
                mbar_arrive_expect_tx(&bar[1 + tl], uint32_t(rows * D) + (tl == 0 ? 4 * gu_plane : 0u));
            }
            mbar_arrive_expect_tx(&bar[0], uint32_t(DR * L.ds) + 2 * d_plane);
        }
        __syncwarp();
        if (lane < 4) {  // the R rows' scales / biases are one contiguous block a matrix
            const int mat = lane >> 1;
            const void* base = (lane & 1) ? a.b[mat] : a.s[mat];
            md_bulk(gusb + uint32_t(lane) * gu_plane,
                    reinterpret_cast<const uint8_t*>(base) + (size_t(e) * I + r0) * size_t(G) * 2, gu_plane, &bar[1]);
        }
        for (int tl = 0; tl < RT; ++tl) {  // lanes 0-15: gate rows of the tile, 16-31: up rows
            const int mat = lane >> 4, r = 16 * tl + (lane & 15);
            if (r < R)
                md_bulk(gu + uint32_t((mat * R + r) * L.gs), a.w[mat] + (size_t(e) * I + r0 + r) * size_t(D / 8),
                        uint32_t(D / 2), &bar[1 + tl]);
        }
        if (lane == 0) {
            const int box = DR < 256 ? DR : 256;
            const uint64_t pol = policy_evict_first();
            for (int r = 0; r < DR; r += box)
                tma_load_2d(sm + L.o_dw + size_t(r) * L.ds, &tm_down, &bar[0], cs * (L.KS / 8),
                            e * D + t * DR + r, pol);
        } else if (lane < 3) {  // the row block's whole down scale / bias rows (every K slice: one contiguous block)
            const void* base = lane == 2 ? a.b[2] : a.s[2];
            md_bulk(dsb + uint32_t(lane - 1) * d_plane,
                    reinterpret_cast<const uint8_t*>(base) + (size_t(e) * D + size_t(t) * DR) * size_t(GI) * 2, d_plane,
                    &bar[0]);
        }
    }

    // ---- gate / up: warps split the 64-groups, rows in tiles of 16 ----
    // shared-memory addresses of each lane's rows (g and g + 8 of every tile; rows past R repeat row R - 1 and
    // their sums are never read) and of their scale windows (the biases sit one plane later)
    const int gpw = (G + MD_WARPS - 1) / MD_WARPS;
    uint32_t wrow[2][MD_RT_MAX][2], srow[2][MD_RT_MAX][2];
#pragma unroll
    for (int mat = 0; mat < 2; ++mat)
#pragma unroll
        for (int tl = 0; tl < MD_RT_MAX; ++tl)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = min(16 * tl + g + 8 * h, R - 1);
                wrow[mat][tl][h] = gu + uint32_t((mat * R + r) * L.gs + 8 * c);
                srow[mat][tl][h] = gusb + uint32_t(2 * mat) * gu_plane + uint32_t(r * G * 2);
            }
    float yacc[2][MD_RT_MAX][2];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int tl = 0; tl < MD_RT_MAX; ++tl) yacc[m][tl][0] = yacc[m][tl][1] = 0.0f;
    const uint32_t xfa = smem_u32(xf) + uint32_t(c * 32);
#pragma unroll
    for (int tl = 0; tl < MD_RT_MAX; ++tl) {  // each row tile as soon as its rows have landed
        if (tl >= RT) break;
        mbar_wait(&bar[1 + tl], 0);  // (a timeout is recorded; the kernel still runs to its end and every barrier)
        for (int gi = 0; gi < gpw; ++gi) {
            const int q = warp * gpw + gi;
            if (q >= G) break;
            const uint4 xa = lds128(xfa + uint32_t(q * 128)), xb = lds128(xfa + uint32_t(q * 128 + 16));
            const float sq = sx[q];
#pragma unroll
            for (int mat = 0; mat < 2; ++mat) {
                const uint2 va = md_lds64(wrow[mat][tl][0] + uint32_t(32 * q));
                const uint2 vb = md_lds64(wrow[mat][tl][1] + uint32_t(32 * q));
                float acc[4];
                md_group<T>(acc, va, vb, xa, xb);
                const uint32_t qa = srow[mat][tl][0] + 2u * q, qb = srow[mat][tl][1] + 2u * q;
                const float sa = F16Traits<T>::to_f32(lds_u16(qa)), ba = F16Traits<T>::to_f32(lds_u16(qa + gu_plane));
                const float sb = F16Traits<T>::to_f32(lds_u16(qb)), bb = F16Traits<T>::to_f32(lds_u16(qb + gu_plane));
                yacc[mat][tl][0] = fmaf(sa, acc[0], fmaf(fmaf(-kVal, sa, ba), sq, yacc[mat][tl][0]));
                yacc[mat][tl][1] = fmaf(sb, acc[2], fmaf(fmaf(-kVal, sb, bb), sq, yacc[mat][tl][1]));
            }
        }
    }
    float* red = reinterpret_cast<float*>(sm + L.o_red);  // [warp][mat][RT * 16 rows]
    const int RR = RT * 16;
    if (c == 0) {
#pragma unroll
        for (int mat = 0; mat < 2; ++mat)
#pragma unroll
            for (int tl = 0; tl < MD_RT_MAX; ++tl) {
                if (tl >= RT) break;
                red[(warp * 2 + mat) * RR + 16 * tl + g] = yacc[mat][tl][0];
                red[(warp * 2 + mat) * RR + 16 * tl + g + 8] = yacc[mat][tl][1];
            }
    }
    __syncthreads();
    // ---- the cluster's h slice: each CTA writes its R values into every peer's copy of the slice ----
    uint16_t* hs = reinterpret_cast<uint16_t*>(sm + L.o_hs);
    for (int r = tid; r < R; r += MD_THREADS) {
        float gs = 0.0f, us = 0.0f;
        for (int w = 0; w < MD_WARPS; ++w) {
            gs += red[(w * 2) * RR + r];
            us += red[(w * 2 + 1) * RR + r];
        }
        const uint16_t hv = F16Traits<T>::from_f32(md_swiglu<T>(gs, us));
        const uint32_t dst = smem_u32(hs + t * R + r);
#pragma unroll
        for (int p = 0; p < MD_CS; ++p) md_st_dsmem_u16(map_peer(dst, uint32_t(p)), hv);
    }
    cluster_sync();  // the whole slice in every CTA; no shared-memory access crosses CTAs after this
    uint32_t* hf = reinterpret_cast<uint32_t*>(sm + L.o_hf);
    float* hsx = reinterpret_cast<float*>(sm + L.o_hsx);
    md_frags(hs, gq, hf, hsx, tid, MD_THREADS, dt);
    __syncthreads();
    mbar_wait(&bar[0], 0);

    // ---- down: warp w takes row tiles w, w + NW, ... over the whole K slice ----
    const uint32_t hfa = smem_u32(hf) + uint32_t(c * 32);
    float* part = a.part + size_t(j * a.C + cs) * D + size_t(t) * DR;
    for (int tl = warp; tl < DR / 16; tl += MD_WARPS) {
        const int ra = 16 * tl + g, rb = ra + 8;
        const uint32_t wa = dw + uint32_t(ra * L.ds + 8 * c), wb = dw + uint32_t(rb * L.ds + 8 * c);
        const uint32_t sa0 = dsb + uint32_t((ra * GI + cs * gq) * 2), sb0 = dsb + uint32_t((rb * GI + cs * gq) * 2);
        float ya = 0.0f, yb = 0.0f;
        for (int q = 0; q < gq; ++q) {
            const uint4 xa = lds128(hfa + uint32_t(q * 128)), xb = lds128(hfa + uint32_t(q * 128 + 16));
            const uint2 va = md_lds64(wa + uint32_t(32 * q)), vb = md_lds64(wb + uint32_t(32 * q));
            float acc[4];
            md_group<T>(acc, va, vb, xa, xb);
            const uint32_t qa = sa0 + 2u * q, qb = sb0 + 2u * q;
            const float sa = F16Traits<T>::to_f32(lds_u16(qa)), ba = F16Traits<T>::to_f32(lds_u16(qa + d_plane));
            const float sb = F16Traits<T>::to_f32(lds_u16(qb)), bb = F16Traits<T>::to_f32(lds_u16(qb + d_plane));
            const float hq = hsx[q];
            ya = fmaf(sa, acc[0], fmaf(fmaf(-kVal, sa, ba), hq, ya));
            yb = fmaf(sb, acc[2], fmaf(fmaf(-kVal, sb, bb), hq, yb));
        }
        if (c == 0) {
            __stcg(part + ra, ya);
            __stcg(part + rb, yb);
        }
    }

    // ---- combine: the last CTA of row block t adds every slot's slices ----
    __syncthreads();  // every partial store of the CTA before thread 0's fence (cumulative) and count
    int* flag = reinterpret_cast<int*>(sm + L.o_flag);
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.cnt + t, 1u);
        const int last = prev == unsigned(k * a.C - 1);
        if (last) __threadfence();
        *flag = last;
    }
    __syncthreads();
    if (*flag) {
        // every slice's row block staged in shared memory (the gate/up rows are no longer read), the loads of a
        // thread all in flight together, then the sums in slice and slot order
        float* stg = reinterpret_cast<float*>(sm + L.o_gu);  // [k C][DR]
        const int KC = k * a.C;
        const float* pb = a.part + size_t(t) * DR;
        for (int i0 = tid; i0 < KC * DR; i0 += 8 * MD_THREADS) {  // eight loads in flight a thread
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = i0 + u * MD_THREADS;
                const int sl = i / DR, rr = i - sl * DR;
                v[u] = i < KC * DR ? __ldcg(pb + size_t(sl) * D + rr) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i0 + u * MD_THREADS < KC * DR) stg[i0 + u * MD_THREADS] = v[u];
        }
        __syncthreads();
        for (int rr = tid; rr < DR; rr += MD_THREADS) {
            float y = 0.0f;
            for (int sl = 0; sl < k; ++sl) {
                float v = 0.0f;
                for (int c2 = 0; c2 < a.C; ++c2) v += stg[(sl * a.C + c2) * DR + rr];
                y = fmaf(md_round<T>(v), sel_w[sl], y);  // as the stand-alone combine kernel sums the slots
            }
            reinterpret_cast<uint16_t*>(a.y)[t * DR + rr] = F16Traits<T>::from_f32(y);
        }
        if (tid == 0) atomicExch(a.cnt + t, 0u);
    }
}

// ------------------------------------------------------------------------------------------------

struct MdPlan {
    int C, R, staged;
    size_t smem, work;
};

// Clusters of the kernel resident at once with `smem` bytes a CTA on the current device (cached per device and
// shared-memory size).
static int md_max_clusters(size_t smem) {
    static std::mutex mu;
    static size_t seen_smem[32];
    static int seen_dev[32], seen_n[32];
    static int nseen = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < nseen; ++i)
        if (seen_smem[i] == smem && seen_dev[i] == dev) return seen_n[i];
    int n = 0;
    // (the limit is a property of the current device; every launch sets it again for its own device)
    const bool ok = cudaFuncSetAttribute(moe_decode_kernel<__nv_bfloat16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) == cudaSuccess;
    if (ok) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(MD_CS, 1, 1);
        cfg.blockDim = dim3(MD_THREADS, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = MD_CS;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, moe_decode_kernel<__nv_bfloat16>, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    if (nseen < 32) {
        seen_smem[nseen] = smem;
        seen_dev[nseen] = dev;
        seen_n[nseen++] = n;
    }
    return n;
}

// The plan of a shape: the K slices C (the largest whose k C clusters are resident at once, else the smallest that
// fits shared memory), R gate/up rows a CTA, router staging, shared memory and workspace bytes. False when the shape
// is outside the kernel.
static bool md_plan(int E, int k, int D, int I, MdPlan* p) {
    if (E < 1 || E > MD_MAX_E || k < 1 || k > MD_MAX_K || k > E) return false;
    if (D < 128 || D % 128 || I < 64 || I % 64) return false;
    if (D / MD_CS > 256 && (D / MD_CS) % 256) return false;  // the down tile in whole TMA boxes
    const DeviceInfo& di = device_info();
    const int EC = (E + MD_CS - 1) / MD_CS;
    const int staged = size_t(EC) * D * 2 <= MD_ROUTER_STAGE_MAX ? 1 : 0;
    int best = 0;
    MdPlan cand = {};
    for (int C = I / 64; C >= 1; --C) {
        if (I % (64 * C) || I % (C * MD_CS)) continue;
        const int R = I / (C * MD_CS);
        if (R > 16 * MD_RT_MAX || I / C > 2048) continue;  // (a TMA box is at most 256 words wide)
        const size_t smem = md_layout(E, k, D, I, C, R, staged).total;
        if (smem > di.smem_optin) continue;
        const int clusters = md_max_clusters(smem);
        if (clusters < 1) continue;
        if (k * C <= clusters) {  // one wave: the largest such C
            cand = {C, R, staged, smem, 0};
            best = 2;
            break;
        }
        cand = {C, R, staged, smem, 0};  // several waves: keep the smallest C seen
        best = 1;
    }
    if (!best) return false;
    cand.work = 64 + size_t(k) * cand.C * D * 4;
    *p = cand;
    return true;
}

size_t moe_decode_workspace_bytes(int E, int k, int D, int I) {
    MdPlan p;
    return md_plan(E, k, D, I, &p) ? p.work : 0;
}

bool moe_decode_ok(int E, int k, int D, int I) {
    MdPlan p;
    return md_plan(E, k, D, I, &p);
}

template <typename T>
static int md_launch(const CUtensorMap& tm, const MdArgs& a, const MdPlan& p, cudaStream_t st) {
    // set on every launch: the limit belongs to the device current at the call (as the other families do)
    if (cudaFuncSetAttribute(moe_decode_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(p.smem)) !=
        cudaSuccess)
        return LQ_E_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(MD_CS, unsigned(p.C), unsigned(a.k));
    cfg.blockDim = dim3(MD_THREADS, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = MD_CS;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cuda_status(cudaLaunchKernelEx(&cfg, moe_decode_kernel<T>, tm, a));
}

int moe_decode_run(const void* x, int x_dt, const void* rw, int rw_dt, int E, int k, int mode, const uint32_t* const* w,
                   const void* const* s, const void* const* b, int D, int I, void* y, uint32_t* inds, float* wts,
                   void* work, size_t work_bytes, cudaStream_t st) {
    MdPlan p;
    if (!md_plan(E, k, D, I, &p)) return LQ_E_SHAPE;
    if (work_bytes < p.work) return LQ_E_ARG;
    MdArgs a = {};
    a.x = x;
    a.rw = rw;
    a.x_dt = x_dt;
    a.rw_dt = rw_dt;
    for (int i = 0; i < 3; ++i) {
        a.w[i] = w[i];
        a.s[i] = s[i];
        a.b[i] = b[i];
    }
    a.y = y;
    a.inds = inds;
    a.wts = wts;
    a.cnt = reinterpret_cast<uint32_t*>(work);
    a.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(work) + 64);
    a.E = E;
    a.k = k;
    a.D = D;
    a.I = I;
    a.mode = mode;
    a.C = p.C;
    a.R = p.R;
    a.staged = p.staged;
    // the down stack as a 2-D map of 32-bit words (E D rows of I / 8), box (K slice, up to 256 rows)
    const int DR = D / MD_CS;
    const uint64_t dims[2] = {uint64_t(I / 8), uint64_t(E) * D};
    const uint64_t strides[1] = {uint64_t(I / 2)};
    const uint32_t box[2] = {uint32_t(I / p.C / 8), uint32_t(DR < 256 ? DR : 256)};
    CUtensorMap tm;
    const int rc = make_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, w[2], dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    return x_dt == LQ_BF16 ? md_launch<__nv_bfloat16>(tm, a, p, st) : md_launch<__half>(tm, a, p, st);
}

}  // namespace lq
