// Routed mixture-of-experts helpers: router logits, top-k routing, the expert grouping (counting
// sort + pair-order gather) and the weighted combine. The expert projections themselves run on the
// qmv kernel family in grouped mode (qmv.cu).
//
//  router_logits : float32 logits = float(x) . float(w)^T, one warp per (token, expert), 16-byte loads
//                  (locals/moe.py:86-139: "exactly as x.astype(f32) @ W.astype(f32).T").
//  route_topk    : one warp per token; softmax (or sigmoid, locals/moe.py:36-82) over E experts held
//                  E/32 per lane, k rounds of a warp argmax with ties to the lower index, renormalise.
//  group         : one CTA; per-expert counts in shared memory, segments of used experts in ascending
//                  expert order, a stable order (pair ids ascending within an expert) and its inverse
//                  (locals/moe_kernel.py:28-66 with a deterministic order).
//  gather_rows   : xs[j] = x[order[j] / k], the tokens laid out in pair order for the grouped kernel.
//  combine       : y[t] = sum_r w[t, r] * ys[pos[t*k + r]] in float32, slots in order (locals/moe.py:339-348).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lq_host.h"
#include "lq_ptx.cuh"
#include "lq_status.cuh"
#include "moe_route.cuh"

namespace lq {

// Launch with programmatic dependent launch: the kernel may start while the previous kernel on the stream
// finishes; it calls grid_dep_wait() before reading anything that kernel wrote.
template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
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
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
}

// grid: T * ceil(E / 4) blocks of 128 threads (4 warps = 4 experts of one token)
__global__ void router_logits_kernel(const void* x, int x_dt, const void* w, int w_dt, float* logits, int T, int E,
                                     int D) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int eb = (E + 3) / 4;
    const int t = blockIdx.x / eb;
    const int e = (blockIdx.x % eb) * 4 + warp;
    if (t >= T || e >= E) return;
    const float acc = router_dot(reinterpret_cast<const uint16_t*>(x) + size_t(t) * D, x_dt,
                                 reinterpret_cast<const uint16_t*>(w) + size_t(e) * D, w_dt, D, lane);
    if (lane == 0) logits[size_t(t) * E + e] = acc;
}

// one warp per token; 4 tokens per block
__global__ void route_topk_kernel(const float* logits, int T, int E, int k, int mode, uint32_t* inds,
                                  float* weights) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 4 + warp;
    if (t >= T) return;
    const float* l = logits + size_t(t) * E;
    score_and_select([&](int e) { return l[e]; }, E, k, mode, lane, inds + size_t(t) * k, weights + size_t(t) * k);
}

// One CTA of 1024 threads. order/starts/experts/nseg as lq_moe_group; pos = inverse of order (optional).
constexpr int GROUP_STAGE = 8192;  // routed pairs staged in shared memory per ranking pass

// Stable counting sort of the routed (token, slot) pairs by expert (moe_kernel.group's order): a shared-memory
// histogram, a one-warp scan that emits the segments, then a one-warp pass over the pairs in order, 32 at a
// time: __match_any_sync finds the lanes of the same expert, a pair's rank is the expert's running count
// plus its rank among those lanes.
// The expert a pair is grouped under: its own id, or with a range (range > 0) its id inside [lo, lo + range) and
// `range` -- the padding bucket, which the grouped expert kernels skip -- for every expert outside it (the local
// experts of one rank of an expert-parallel layer).
__device__ __forceinline__ uint32_t grp_key(uint32_t e, int lo, int range) {
    if (range <= 0) return e;
    const uint32_t d = e - uint32_t(lo);
    return d < uint32_t(range) ? d : uint32_t(range);
}

__global__ void group_kernel(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts,
                             int32_t* nseg, int32_t* pos, int lo, int range) {
    grid_dep_wait();
    grid_dep_launch();
    extern __shared__ int32_t sh[];
    int32_t* cnt = sh;                                   // E counts
    int32_t* run = sh + E;                               // E running positions
    uint32_t* staged = reinterpret_cast<uint32_t*>(sh + 2 * E);  // GROUP_STAGE expert ids
    const int lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const uint32_t e = grp_key(inds[p], lo, range);
        if (e < uint32_t(E))
            atomicAdd(&cnt[e], 1);
        else
            record_status(LQ_DEV_BOUNDS);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        int at = 0, s = 0;
        for (int c = 0; c < E; c += 32) {
            const int e = c + lane;
            const int v = e < E ? cnt[e] : 0;
            int incl = v;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int t = __shfl_up_sync(0xFFFFFFFFu, incl, d);
                if (lane >= d) incl += t;
            }
            const unsigned nz = __ballot_sync(0xFFFFFFFFu, v > 0);
            if (e < E) run[e] = at + incl - v;
            if (v > 0) {
                const int si = s + __popc(nz & ((1u << lane) - 1u));
                starts[si] = at + incl - v;
                experts[si] = e;
            }
            at += __shfl_sync(0xFFFFFFFFu, incl, 31);
            s += __popc(nz);
        }
        if (lane == 0) {
            starts[s] = at;
            nseg[0] = s;
        }
    }
    for (int p0 = 0; p0 < P; p0 += GROUP_STAGE) {
        const int n = P - p0 < GROUP_STAGE ? P - p0 : GROUP_STAGE;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) staged[i] = grp_key(inds[p0 + i], lo, range);
        __syncthreads();
        if (threadIdx.x < 32) {
            for (int c = 0; c < n; c += 32) {
                const int i = c + lane;
                const uint32_t e = i < n ? staged[i] : 0xFFFFFFFFu;
                const bool valid = e < uint32_t(E);
                const unsigned peers = __match_any_sync(0xFFFFFFFFu, valid ? e : 0xFFFFFFFFu);
                const int rank = __popc(peers & ((1u << lane) - 1u));
                const int j = valid ? run[e] + rank : 0;
                __syncwarp();
                if (valid && rank == 0) run[e] += __popc(peers);
                __syncwarp();
                if (valid) {
                    order[j] = p0 + i;
                    if (pos) pos[p0 + i] = j;
                }
            }
        }
    }
}

// The same grouping with every warp at work (E <= GROUP_PAR_MAX_E): warp w owns the contiguous pairs
// [w CH, (w + 1) CH) and counts them per expert in its own row of a (32, E) table; a column scan turns the table into
// each warp's first slot in every expert's segment; the segments are laid out as in group_kernel; then each warp
// places its pairs in pair order (a match over each 32 pairs ranks equal experts by lane). Pair p of expert e lands
// after every earlier pair of e, exactly as in group_kernel: the same order, starts, experts and pos.
constexpr int GROUP_PAR_MAX_E = 1024;

__global__ void __launch_bounds__(1024) group_par_kernel(const uint32_t* inds, int P, int E, int32_t* order,
                                                         int32_t* starts, int32_t* experts, int32_t* nseg,
                                                         int32_t* pos, int lo, int range) {
    grid_dep_wait();
    grid_dep_launch();
    extern __shared__ int32_t sh[];
    int32_t* hist = sh;            // [32][E]: counts, then each warp's running slot
    int32_t* cnt = sh + 32 * E;    // E totals
    int32_t* run = cnt + E;        // E segment starts
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int CH = (P + 31) / 32;
    const int p0 = warp * CH, p1 = p0 + CH < P ? p0 + CH : P;
    for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int c = p0; c < p1; c += 32) {
        const int p = c + lane;
        const uint32_t e = p < p1 ? grp_key(inds[p], lo, range) : 0xFFFFFFFFu;
        if (p < p1 && e >= uint32_t(E)) record_status(LQ_DEV_BOUNDS);
        const bool valid = p < p1 && e < uint32_t(E);
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, valid ? e : 0xFFFFFFFFu);
        if (valid && (peers & ((1u << lane) - 1u)) == 0) hist[warp * E + int(e)] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {  // each warp's offset inside the expert's segment
        int acc = 0;
        for (int w = 0; w < 32; ++w) {
            const int v = hist[w * E + e];
            hist[w * E + e] = acc;
            acc += v;
        }
        cnt[e] = acc;
    }
    __syncthreads();
    if (warp == 0) {
        int at = 0, sgi = 0;
        for (int c = 0; c < E; c += 32) {
            const int e = c + lane;
            const int v = e < E ? cnt[e] : 0;
            int incl = v;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int t = __shfl_up_sync(0xFFFFFFFFu, incl, d);
                if (lane >= d) incl += t;
            }
            const unsigned nz = __ballot_sync(0xFFFFFFFFu, v > 0);
            if (e < E) run[e] = at + incl - v;
            if (v > 0) {
                const int si = sgi + __popc(nz & ((1u << lane) - 1u));
                starts[si] = at + incl - v;
                experts[si] = e;
            }
            at += __shfl_sync(0xFFFFFFFFu, incl, 31);
            sgi += __popc(nz);
        }
        if (lane == 0) {
            starts[sgi] = at;
            nseg[0] = sgi;
        }
    }
    __syncthreads();
    for (int c = p0; c < p1; c += 32) {
        const int p = c + lane;
        const uint32_t e = p < p1 ? grp_key(inds[p], lo, range) : 0xFFFFFFFFu;
        const bool valid = p < p1 && e < uint32_t(E);
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, valid ? e : 0xFFFFFFFFu);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const int j = valid ? run[e] + hist[warp * E + int(e)] + rank : 0;
        __syncwarp();
        if (valid && rank == 0) hist[warp * E + int(e)] += __popc(peers);
        __syncwarp();
        if (valid) {
            order[j] = p;
            if (pos) pos[p] = j;
        }
    }
}

// xs[j] = x[order[j] / k]: one warp per row, 16-byte copies
__global__ void gather_rows_kernel(const uint16_t* x, const int32_t* order, int P, int k, int D, uint16_t* xs) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= P) return;
    const int tok = order[warp] / k;
    const uint4* src = reinterpret_cast<const uint4*>(x + size_t(tok) * D);
    uint4* dst = reinterpret_cast<uint4*>(xs + size_t(warp) * D);
    for (int i = lane; i < D / 8; i += 32) dst[i] = src[i];
}

// y[t, d] = sum_r w[t, r] * ys[row(t, r), d]; row = pos[t*k + r] if pos, else t*k + r
__global__ void combine_kernel(const uint16_t* ys, const float* w, const int32_t* pos, uint16_t* y, int T, int k, int D,
                               int dt) {
    grid_dep_wait();
    grid_dep_launch();
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(T) * D) return;
    const int t = int(i / D), d = int(i % D);
    float acc = 0.0f;
    for (int r = 0; r < k; ++r) {
        const int slot = t * k + r;
        const int row = pos ? pos[slot] : slot;
        const uint16_t h = ys[size_t(row) * D + d];
        float v;
        if (dt == LQ_BF16) {
            v = __uint_as_float(uint32_t(h) << 16);
        } else {
            v = __half2float(*reinterpret_cast<const __half*>(&h));
        }
        acc = fmaf(v, w[slot], acc);
    }
    if (dt == LQ_BF16) {
        __nv_bfloat16 b = __float2bfloat16_rn(acc);
        y[i] = *reinterpret_cast<uint16_t*>(&b);
    } else {
        __half hh = __float2half_rn(acc);
        y[i] = *reinterpret_cast<uint16_t*>(&hh);
    }
}

// Router logits and top-k, the experts split over a cluster of RC_CL CTAs and the tokens in tiles of TT (grid
// (ceil(T / TT), RC_CL), cluster (1, RC_CL, 1), 256 threads; TT = ceil(T / 16) up to RC_TT, so up to 16 tokens run
// one token a cluster). Each CTA stages its E / RC_CL experts' router rows in
// shared memory BEFORE waiting for the previous kernel (they do not depend on it; at config 4 a CTA's 8 rows are
// 32 KB, so the weights are read by eight SMs at once instead of one), computes the float32 dot products of its
// experts with the tile's tokens (16-byte loads, one warp an expert for all the tile's tokens), and keeps the logits
// in shared memory.
// After a cluster barrier warp t of CTA 0 reads token t's E logits from the eight CTAs (distributed shared memory)
// and picks the top k exactly as route_topk_kernel does. logits_out may be null.
constexpr int ROUTE_MAX_E = 1024;
constexpr int RC_CL = 8;
constexpr int RC_TT = 8;  // the largest token tile
constexpr size_t RC_STAGE_MAX = 64 * 1024;

__global__ void __launch_bounds__(256) router_topk_kernel(const void* x, int x_dt, const void* w, int w_dt, int T,
                                                          int E, int D, int k, int mode, int staged, int TT,
                                                          uint32_t* inds, float* weights, float* logits_out) {
    extern __shared__ __align__(16) uint8_t rsm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = int(cluster_ctarank());
    const int EC = (E + RC_CL - 1) / RC_CL;
    const int e0 = rank * EC;
    const int ne = E - e0 < EC ? (E - e0 > 0 ? E - e0 : 0) : EC;
    float* lg = reinterpret_cast<float*>(rsm);  // [TT][EC]
    const size_t lg_bytes = (size_t(TT) * EC * 4 + 15) / 16 * 16;
    const uint16_t* wrows = reinterpret_cast<const uint16_t*>(w) + size_t(e0) * D;
    uint16_t* wsm = reinterpret_cast<uint16_t*>(rsm + lg_bytes);
    const size_t wbytes = (staged & 1) ? (size_t(EC) * D * 2 + 15) / 16 * 16 : 0;
    uint16_t* xsm = reinterpret_cast<uint16_t*>(rsm + lg_bytes + wbytes);  // the tile's tokens (staged & 2)
    if (staged & 1) {  // this CTA's router rows (independent of the previous kernel)
        const int n16 = ne * D / 8;
        for (int i = threadIdx.x; i < n16; i += blockDim.x) cp_async(smem_u32(wsm + 8 * i), wrows + 8 * i, 16, true);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    grid_dep_wait();
    grid_dep_launch();
    const int t0 = blockIdx.x * TT;
    const int tt = T - t0 < TT ? T - t0 : TT;
    const uint16_t* xtile = reinterpret_cast<const uint16_t*>(x) + size_t(t0) * D;
    if (staged & 2) {  // the tile's tokens, every 16-byte load in flight at once
        const int n16 = tt * D / 8;
        for (int i = threadIdx.x; i < n16; i += blockDim.x) cp_async(smem_u32(xsm + 8 * i), xtile + 8 * i, 16, true);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (staged) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const uint16_t* wsrc = (staged & 1) ? wsm : wrows;
    const uint16_t* xsrc = (staged & 2) ? xsm : xtile;
    // warp w: expert w (w + 8, ...) for every token of the tile at once, each router piece loaded once for all of
    // them; every logit keeps router_dot's order (lane-strided pieces in order, then the same butterfly)
    if (tt == 1) {  // (one token: the plain one-warp dot, the same order)
        for (int el = warp; el < ne; el += 8) {
            const float v = router_dot(xsrc, x_dt, wsrc + size_t(el) * D, w_dt, D, lane);
            if (lane == 0) {
                lg[el] = v;
                if (logits_out) logits_out[size_t(t0) * E + e0 + el] = v;
            }
        }
    }
    for (int el = warp; tt > 1 && el < ne; el += 8) {
        const uint4* wr = reinterpret_cast<const uint4*>(wsrc + size_t(el) * D);
        float acc[RC_TT];
#pragma unroll
        for (int t = 0; t < RC_TT; ++t) acc[t] = 0.0f;
        for (int i = lane; i < D / 8; i += 32) {
            float wf[8];
            unpack8(wr[i], w_dt, wf);
#pragma unroll
            for (int t = 0; t < RC_TT; ++t)
                if (t < tt) {
                    float xf[8];
                    unpack8(reinterpret_cast<const uint4*>(xsrc + size_t(t) * D)[i], x_dt, xf);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[t] = fmaf(xf[j], wf[j], acc[t]);
                }
        }
#pragma unroll
        for (int t = 0; t < RC_TT; ++t)
            if (t < tt) {
                float v = acc[t];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == t) {
                    lg[t * EC + el] = v;
                    if (logits_out) logits_out[size_t(t0 + t) * E + e0 + el] = v;
                }
            }
    }
    cluster_sync();  // every CTA's logits are visible to the cluster
    if (rank == 0 && warp < tt) {
        const uint32_t base = smem_u32(lg + warp * EC);
        auto get = [&](int e) {
            const int owner = e / EC;
            return ld_dsmem_f(map_peer(base + 4u * uint32_t(e - owner * EC), uint32_t(owner)));
        };
        const int t = t0 + warp;
        score_and_select(get, E, k, mode, lane, inds + size_t(t) * k, weights + size_t(t) * k);
    }
    cluster_sync();  // peers keep their shared memory until CTA 0 has read it
}

// More than 64 tokens: a CTA takes TT tokens and all E <= 8 EW experts (no cluster); warp w takes experts
// [w EW, (w + 1) EW) and keeps TT x EW sums a lane, each x piece loaded once for EW experts and each router piece once
// for TT tokens. Every logit keeps router_dot's order (lane-strided pieces in order with fmaf, then the same butterfly),
// so the choice is bit-identical to the cluster kernel's and to the fused one-token layer's. Warp t then picks token
// t's top k from the CTA's logits in shared memory.
template <int TT, int EW>
__global__ void __launch_bounds__(256) router_tile_kernel(const void* x, int x_dt, const void* w, int w_dt, int T,
                                                          int E, int D, int k, int mode, uint32_t* inds,
                                                          float* weights, float* logits_out) {
    __shared__ float lg[TT][8 * EW];
    grid_dep_wait();
    grid_dep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * TT;
    const int tt = T - t0 < TT ? T - t0 : TT;
    const int e0 = warp * EW;
    const uint4* xr[TT];
    const uint4* wr[EW];
#pragma unroll
    for (int t = 0; t < TT; ++t)
        xr[t] = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + size_t(t0 + (t < tt ? t : 0)) * D);
#pragma unroll
    for (int e = 0; e < EW; ++e)
        wr[e] = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w) +
                                               size_t(e0 + e < E ? e0 + e : 0) * D);
    float acc[TT][EW];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int e = 0; e < EW; ++e) acc[t][e] = 0.0f;
    if (e0 < E) {
#pragma unroll 2
        for (int i = lane; i < D / 8; i += 32) {
            float xf[TT][8];
#pragma unroll
            for (int t = 0; t < TT; ++t) unpack8(xr[t][i], x_dt, xf[t]);
#pragma unroll
            for (int e = 0; e < EW; ++e) {
                float wf[8];
                unpack8(wr[e][i], w_dt, wf);
#pragma unroll
                for (int t = 0; t < TT; ++t)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[t][e] = fmaf(xf[t][j], wf[j], acc[t][e]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int e = 0; e < EW; ++e) {
            float v = acc[t][e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == ((t * EW + e) & 31) && t < tt && e0 + e < E) {
                lg[t][e0 + e] = v;
                if (logits_out) logits_out[size_t(t0 + t) * E + e0 + e] = v;
            }
        }
    __syncthreads();
    if (warp < tt)
        score_and_select([&](int e) { return lg[warp][e]; }, E, k, mode, lane, inds + size_t(t0 + warp) * k,
                         weights + size_t(t0 + warp) * k);
}

template <int TT, int EW>
static int router_tile_launch(const void* x, int x_dt, const void* w, int w_dt, int T, int E, int D, int k, int mode,
                              uint32_t* inds, float* weights, float* logits, cudaStream_t st) {
    return launch_pdl(router_tile_kernel<TT, EW>, dim3(unsigned((T + TT - 1) / TT)), dim3(256), 0, st, x, x_dt, w,
                      w_dt, T, E, D, k, mode, inds, weights, logits);
}

int router_topk_run(const void* x, int x_dt, const void* w, int w_dt, int T, int E, int D, int k, int mode,
                    uint32_t* inds, float* weights, float* logits, cudaStream_t st) {
    // measured on B200 at E 64, D 2048: the cluster kernel 4.8 / 7.6 us at 16 / 64 tokens (22.9 at 512), the tiled
    // kernel 10.5 us at 64 and at 512 tokens
    if (T > 64 && E <= 128) {  // (four tokens a CTA: one wave for up to 592 tokens)
        if (E <= 32) return router_tile_launch<4, 4>(x, x_dt, w, w_dt, T, E, D, k, mode, inds, weights, logits, st);
        if (E <= 64) return router_tile_launch<4, 8>(x, x_dt, w, w_dt, T, E, D, k, mode, inds, weights, logits, st);
        return router_tile_launch<4, 16>(x, x_dt, w, w_dt, T, E, D, k, mode, inds, weights, logits, st);
    }
    const int EC = (E + RC_CL - 1) / RC_CL;
    const int TT = T <= 16 ? 1 : ((T + 15) / 16 < RC_TT ? (T + 15) / 16 : RC_TT);
    const size_t lg_bytes = (size_t(TT) * EC * 4 + 15) / 16 * 16;
    const size_t wbytes = (size_t(EC) * D * 2 + 15) / 16 * 16;
    const size_t xbytes = size_t(TT) * D * 2;
    // bit 0: router rows staged in shared memory; bit 1: the tile's tokens too (x is 16-byte aligned, D % 8 == 0)
    const int staged = ((wbytes <= RC_STAGE_MAX && (reinterpret_cast<uintptr_t>(w) % 16) == 0) ? 1 : 0) |
                       (xbytes <= RC_STAGE_MAX ? 2 : 0);
    const size_t smem = lg_bytes + ((staged & 1) ? wbytes : 0) + ((staged & 2) ? xbytes : 0);
    if (smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(router_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return LQ_E_CUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((T + TT - 1) / TT, RC_CL, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = RC_CL;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cuda_status(cudaLaunchKernelEx(&cfg, router_topk_kernel, x, x_dt, w, w_dt, T, E, D, k, mode, staged, TT,
                                          inds, weights, logits));
}

int router_logits_run(const void* x, int x_dt, const void* w, int w_dt, float* logits, int T, int E, int D,
                      cudaStream_t st) {
    const int blocks = T * ((E + 3) / 4);
    return launch_pdl(router_logits_kernel, dim3(blocks), dim3(128), 0, st, x, x_dt, w, w_dt, logits, T, E, D);
}

int route_topk_run(const float* logits, int T, int E, int k, int mode, uint32_t* inds, float* weights,
                   cudaStream_t st) {
    return launch_pdl(route_topk_kernel, dim3((T + 3) / 4), dim3(128), 0, st, logits, T, E, k, mode, inds, weights);
}

static int group_impl(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts,
                      int32_t* nseg, int32_t* pos, cudaStream_t st, int lo, int range) {
    if (E <= GROUP_PAR_MAX_E && P > 256) {  // (up to 256 pairs the one-warp placement is as fast)
        const size_t smem = size_t(34) * E * sizeof(int32_t);
        if (smem > 48 * 1024) {
            const cudaError_t e =
                cudaFuncSetAttribute(group_par_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            if (e != cudaSuccess) return LQ_E_CUDA;
        }
        return launch_pdl(group_par_kernel, dim3(1), dim3(1024), smem, st, inds, P, E, order, starts, experts, nseg,
                          pos, lo, range);
    }
    const size_t smem = size_t(2) * E * sizeof(int32_t) + size_t(GROUP_STAGE) * sizeof(uint32_t);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return LQ_E_CUDA;
    }
    return launch_pdl(group_kernel, dim3(1), dim3(1024), smem, st, inds, P, E, order, starts, experts, nseg, pos, lo,
                      range);
}

int group_run(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts, int32_t* nseg,
              int32_t* pos, cudaStream_t st) {
    return group_impl(inds, P, E, order, starts, experts, nseg, pos, st, 0, 0);
}

// The grouping of the pairs routed to experts [lo, lo + range) only (local ids 0 .. range - 1); every other pair goes
// to the padding bucket `range`, which sorts last.
int group_range_run(const uint32_t* inds, int P, int lo, int range, int32_t* order, int32_t* starts, int32_t* experts,
                    int32_t* nseg, int32_t* pos, cudaStream_t st) {
    return group_impl(inds, P, range + 1, order, starts, experts, nseg, pos, st, lo, range);
}

int gather_rows_run(const void* x, const int32_t* order, int P, int k, int D, void* xs, cudaStream_t st) {
    const int threads = 256;
    const int blocks = (P * 32 + threads - 1) / threads;
    return launch_pdl(gather_rows_kernel, dim3(blocks), dim3(threads), 0, st, reinterpret_cast<const uint16_t*>(x),
                      order, P, k, D, reinterpret_cast<uint16_t*>(xs));
}

int combine_run(const void* ys, const float* w, const int32_t* pos, void* y, int T, int k, int D, int dt,
                cudaStream_t st) {
    const size_t n = size_t(T) * D;
    const int threads = 256;
    return launch_pdl(combine_kernel, dim3(unsigned((n + threads - 1) / threads)), dim3(threads), 0, st,
                      reinterpret_cast<const uint16_t*>(ys), w, pos, reinterpret_cast<uint16_t*>(y), T, k, D, dt);
}

}  // namespace lq
