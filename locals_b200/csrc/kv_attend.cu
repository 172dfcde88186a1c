// Decode attention over an 8-bit key/value cache: one query a (row, head) against positions start[b] .. n-1 of
// a cache held as MLX affine 8-bit groups of 64, with the head's sink logit in the softmax denominator
// (locals/qkv.py:1-17 and attend, qkv.py:213-249; the reference's two passes _PASS1 / _PASS2).
//
// Cache layout, read in place as the reference's cache keeps it: words uint32 (B, KVH, cap, 32) — four codes a
// word, low byte first — and scales / biases (B, KVH, cap, 2) in the activation dtype; q and out (B, H, 128).
//
// kv_attend_kernel: one CTA a (block of keys, kv head, row), four warps; each warp walks 16-key chunks of the block
// through its own 4-deep cp.async ring (rows outside [start, n) are zero-filled, never read). The G query heads
// that share the kv head are the M rows of an m16n8k16 f16 MMA, so every key is read and unpacked once for all
// of them (the reference's reason for its simdgroup-matrix pass):
//   * scores: the codes enter the MMA as they are (1024 + q is exact in fp16: one prmt a pair) against the
//     queries scaled by a power of two into fp16 range; the per-key group scale and bias are applied to the fp32
//     accumulators afterwards, score = sum_g s_g (C_g - 1024 Qsum_g) + b_g Qsum_g, so keys are never rounded;
//   * values: dequantized to fp16 (v = s q + b, one rounding) into the MMA's B operand, the probabilities
//     (<= 1, relative to the running maximum) its A operand;
//   * a running softmax a head in base 2 (scores pre-multiplied by scale * log2 e), merged across the four warps
//     in shared memory into one part a (head, block).
// Dims are permuted inside each MMA (a dot product does not mind; the output is stored un-permuted) so that a lane
// reads whole 16-byte (keys) and 8-byte (values) pieces, and key rows are permuted within a chunk (p(x) =
// x ^ ((x & 1) << 2)) so that those reads, with the XOR swizzle of the ring, are free of bank conflicts.
// kv_join_kernel joins a head's parts with its sink (skipped when one block covers the keys).
// HBM-bound: 272 bytes a key and kv head (128 + 128 code bytes, 16 bytes of scales and biases).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

#include "lq_host.h"
#include "lq_ptx.cuh"
#include "lq_status.cuh"

namespace lq {

constexpr int KVA_HD = 128;
constexpr int KVA_NW = 4;      // warps a CTA
constexpr int KVA_STAGES = 4;  // ring depth a warp
constexpr int KVA_KEYS = 16;   // keys a warp step
constexpr int KVA_MAX_G = 16;  // query heads a kv head (the MMA's M)
constexpr int KVA_CODES = KVA_KEYS * KVA_HD;                       // 2048 bytes of codes a chunk (keys or values)
constexpr int KVA_STAGE_BYTES = 2 * KVA_CODES + 4 * KVA_KEYS * 4;  // + ks, kb, vs, vb: 4352
constexpr int KVA_SMEM = KVA_NW * KVA_STAGES * KVA_STAGE_BYTES;    // 69632
constexpr int KVA_MIN_BLOCK = 256;                                 // keys a CTA at least (4 chunks a warp)
constexpr int KVA_CTAS_PER_SM = 3;
constexpr float KVA_LOG2E = 1.4426950408889634f;

struct KvaArgs {
    const uint16_t* q;
    const uint32_t* kq;
    const uint32_t* ks;  // one word = a row's two 16-bit group values (group 0 low)
    const uint32_t* kb;
    const uint32_t* vq;
    const uint32_t* vs;
    const uint32_t* vb;
    const int32_t* start;  // may be null: every row from 0
    const float* sinks;    // may be null: no sink
    float scale_log2;      // scale * log2(e)
    int n, H, KVH, G, cap, nsplit, block;
    float* part_ml;  // (B * H * nsplit) x {m, l}, base 2
    float* part_o;   // (B * H * nsplit) x 128
    uint16_t* out;
};

static_assert(KVA_NW * 32 == KVA_HD, "the merge gives one thread a dim");
static_assert(KVA_NW * (2 * KVA_MAX_G + KVA_MAX_G * KVA_HD) * 4 <= KVA_SMEM, "the merge reuses the rings");

__device__ __forceinline__ int kva_perm(int x) { return x ^ ((x & 1) << 2); }

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t h2_sub_fma(uint32_t v, uint32_t s2, uint32_t b2) {
    const uint32_t m = 0x64006400u;  // (v - 1024) * s + b on fp16 pairs: v - 1024 is the code, exactly
    __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&v), *reinterpret_cast<const __half2*>(&m));
    __half2 r = __hfma2(q, *reinterpret_cast<const __half2*>(&s2), *reinterpret_cast<const __half2*>(&b2));
    return *reinterpret_cast<uint32_t*>(&r);
}

// Two rows' 16-bit values of group g as an fp16 pair (row a low).
template <typename T>
__device__ __forceinline__ uint32_t kva_pair_f16(uint32_t wa, uint32_t wb, int g) {
    if constexpr (std::is_same<T, __half>::value) {
        return prmt(wa, wb, g ? 0x7632u : 0x5410u);
    } else {
        const float fa = __uint_as_float(g ? (wa & 0xffff0000u) : (wa << 16));
        const float fb = __uint_as_float(g ? (wb & 0xffff0000u) : (wb << 16));
        return cvt_f16x2(fb, fa);
    }
}

template <typename T>
__device__ __forceinline__ float kva_f32(uint32_t w, int g) {
    return F16Traits<T>::to_f32(g ? (w >> 16) : (w & 0xffffu));
}

// The head's softmax parts (m, l, O) combined with its sink into T(O / L); 0 where nothing was attended.
template <typename T>
__device__ __forceinline__ uint16_t kva_finish(float m, float l, float o, float sink) {
    const float M = fmaxf(m, sink);
    if (M == -INFINITY) return F16Traits<T>::from_f32(0.0f);
    const float w = m == -INFINITY ? 0.0f : exp2f(m - M);
    const float L = l * w + (sink == -INFINITY ? 0.0f : exp2f(sink - M));
    return F16Traits<T>::from_f32(L > 0.0f ? o * w / L : 0.0f);
}

template <typename T, bool HI>
__global__ void __launch_bounds__(KVA_NW * 32, KVA_CTAS_PER_SM) kv_attend_kernel(const KvaArgs a) {
    extern __shared__ __align__(128) uint8_t kva_smem[];
    grid_dep_wait();
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, c = lane & 3;
    const int lo = a.start ? max(a.start[b], 0) : 0, hi = a.n;
    const int c_lo = max(split * a.block, lo), c_hi = min((split + 1) * a.block, hi);
    const int q0 = c_lo / KVA_KEYS, q1 = c_hi > c_lo ? (c_hi + KVA_KEYS - 1) / KVA_KEYS : q0;
    const size_t rowbase = (size_t(b) * a.KVH + kvh) * a.cap;

    // ---- the queries of the G heads: fp16 A fragments scaled by 2^-E, the group sums of what the MMA sees ----
    constexpr int NH = HI ? 2 : 1;
    uint32_t qa[NH][2][4][2];  // [half][group][k-tile][lo/hi reg]
    float qs[NH][2], fq[NH];
#pragma unroll
    for (int hf = 0; hf < NH; ++hf) {
        const int hh = gid + 8 * hf;
        float x[2][16];
        float mx = 0.0f;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            if (hh < a.G) {
                const uint4* src = reinterpret_cast<const uint4*>(
                    a.q + (size_t(b) * a.H + size_t(kvh) * a.G + hh) * KVA_HD + 64 * g + 16 * c);
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const uint4 v = src[u];
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        x[g][8 * u + 2 * i] = F16Traits<T>::to_f32(w[i] & 0xffffu);
                        x[g][8 * u + 2 * i + 1] = F16Traits<T>::to_f32(w[i] >> 16);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) x[g][i] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(x[g][i]));
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        // 2^-E with E the exponent of the head's largest |q| (clamped): scaled values lie below 2 in magnitude
        int E = mx > 0.0f ? int((__float_as_uint(mx) >> 23) & 0xff) - 127 : 0;
        E = min(max(E, -100), 100);
        const float f = __uint_as_float(uint32_t(127 - E) << 23);
        fq[hf] = a.scale_log2 * __uint_as_float(uint32_t(127 + E) << 23);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            float sum = 0.0f;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const __half h0 = __float2half_rn(x[g][4 * t] * f), h1 = __float2half_rn(x[g][4 * t + 1] * f);
                const __half h2 = __float2half_rn(x[g][4 * t + 2] * f), h3 = __float2half_rn(x[g][4 * t + 3] * f);
                sum += (__half2float(h0) + __half2float(h1)) + (__half2float(h2) + __half2float(h3));
                qa[hf][g][t][0] = uint32_t(__half_as_ushort(h0)) | (uint32_t(__half_as_ushort(h1)) << 16);
                qa[hf][g][t][1] = uint32_t(__half_as_ushort(h2)) | (uint32_t(__half_as_ushort(h3)) << 16);
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            qs[hf][g] = sum;
        }
    }

    // ---- the warp's chunks: q0 + warp, q0 + warp + NW, ... ----
    const int nq = q1 - q0 > warp ? (q1 - q0 - warp + KVA_NW - 1) / KVA_NW : 0;
    const uint32_t ring = smem_u32(kva_smem) + warp * KVA_STAGES * KVA_STAGE_BYTES;
    auto issue = [&](int qi, int st) {
        const uint32_t sb = ring + st * KVA_STAGE_BYTES;
        const int pos0 = qi * KVA_KEYS;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = lane + 32 * j, r = e >> 3, piece = e & 7;
            const int pos = pos0 + r;
            const bool ok = pos >= lo && pos < hi;
            const size_t row = rowbase + (ok ? pos : 0);
            const uint32_t off = r * KVA_HD + ((piece ^ (r & 7)) << 4);
            cp_async(sb + off, a.kq + row * 32 + piece * 4, 16, ok);
            cp_async(sb + KVA_CODES + off, a.vq + row * 32 + piece * 4, 16, ok);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int e = lane + 32 * j, arr = e >> 4, r = e & 15;
            const int pos = pos0 + r;
            const bool ok = pos >= lo && pos < hi;
            const size_t row = rowbase + (ok ? pos : 0);
            const uint32_t* src = arr == 0 ? a.ks : arr == 1 ? a.kb : arr == 2 ? a.vs : a.vb;
            cp_async(sb + 2 * KVA_CODES + arr * 64 + r * 4, src + row, 4, ok);
        }
    };

    float o[16][4];
#pragma unroll
    for (int t = 0; t < 16; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[t][i] = 0.0f;
    float m[NH], l[NH];
#pragma unroll
    for (int hf = 0; hf < NH; ++hf) m[hf] = -INFINITY, l[hf] = 0.0f;

#pragma unroll
    for (int i = 0; i < KVA_STAGES - 1; ++i) {
        if (i < nq) issue(q0 + warp + i * KVA_NW, i);
        cp_async_commit();
    }
    const int ra = 2 * c, rb = kva_perm(2 * c + 1);  // the value rows of this lane's keys 2c, 2c + 1 (+8)
    for (int i = 0; i < nq; ++i) {
        const int nx = i + KVA_STAGES - 1;
        if (nx < nq) issue(q0 + warp + nx * KVA_NW, nx % KVA_STAGES);
        cp_async_commit();
        cp_async_wait<KVA_STAGES - 1>();
        __syncwarp();
        const uint32_t sb = ring + (i % KVA_STAGES) * KVA_STAGE_BYTES;
        const int pos0 = (q0 + warp + i * KVA_NW) * KVA_KEYS;

        // scores: S^T tiles [heads x 8 keys] per (key tile nt, group g)
        float sc[2][2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const int r = kva_perm(gid) + 8 * nt;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
#pragma unroll
                for (int u = 0; u < 4; ++u) sc[nt][g][u] = 0.0f;
                const uint4 w = lds128(sb + r * KVA_HD + (((4 * g + c) ^ (r & 7)) << 4));
                const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t b0 = prmt(wv[t], 0x64646464u, 0x4140u), b1 = prmt(wv[t], 0x64646464u, 0x4342u);
                    mma_16816<__half>(sc[nt][g], qa[0][g][t][0], HI ? qa[NH - 1][g][t][0] : 0u, qa[0][g][t][1],
                                      HI ? qa[NH - 1][g][t][1] : 0u, b0, b1);
                }
            }
        }
        float s[NH][2][2];  // [half][nt][j]: this lane's keys 8 nt + 2c + j
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int r = kva_perm(2 * c + j) + 8 * nt;
                const uint32_t ksw = lds32(sb + 2 * KVA_CODES + r * 4), kbw = lds32(sb + 2 * KVA_CODES + 64 + r * 4);
                const float k0 = kva_f32<T>(ksw, 0), k1 = kva_f32<T>(ksw, 1);
                const float c0 = kva_f32<T>(kbw, 0) - 1024.0f * k0, c1 = kva_f32<T>(kbw, 1) - 1024.0f * k1;
                const int pos = pos0 + r;
                const bool ok = pos >= lo && pos < hi;
#pragma unroll
                for (int hf = 0; hf < NH; ++hf) {
                    const float v = k0 * sc[nt][0][2 * hf + j] + k1 * sc[nt][1][2 * hf + j] + c0 * qs[hf][0] +
                                    c1 * qs[hf][1];
                    s[hf][nt][j] = ok ? v * fq[hf] : -INFINITY;
                }
            }
        // running softmax a head (the head's four lanes agree on m)
        float corr[NH];
        uint32_t pa[NH][2];
#pragma unroll
        for (int hf = 0; hf < NH; ++hf) {
            float mx = fmaxf(fmaxf(s[hf][0][0], s[hf][0][1]), fmaxf(s[hf][1][0], s[hf][1][1]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(m[hf], mx);
            float p[2][2];
            if (mn == -INFINITY) {
                corr[hf] = 1.0f;
                p[0][0] = p[0][1] = p[1][0] = p[1][1] = 0.0f;
            } else {
                corr[hf] = exp2f(m[hf] - mn);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int j = 0; j < 2; ++j) p[nt][j] = exp2f(s[hf][nt][j] - mn);
            }
            l[hf] = l[hf] * corr[hf] + ((p[0][0] + p[0][1]) + (p[1][0] + p[1][1]));
            m[hf] = mn;
            pa[hf][0] = cvt_f16x2(p[0][1], p[0][0]);
            pa[hf][1] = cvt_f16x2(p[1][1], p[1][0]);
        }
        bool rescale = corr[0] != 1.0f;
        if constexpr (HI) rescale = rescale || corr[NH - 1] != 1.0f;
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                o[t][0] *= corr[0];
                o[t][1] *= corr[0];
                o[t][2] *= corr[NH - 1];
                o[t][3] *= corr[NH - 1];
            }
        }

        // values: rows of keys 2c, 2c + 1 (b0) and 2c + 8, 2c + 9 (b1), dims 64 gg + 8 gid + i of n-tile 8 gg + i
        const uint32_t vsa = lds32(sb + 2 * KVA_CODES + 128 + ra * 4), vsb = lds32(sb + 2 * KVA_CODES + 128 + rb * 4);
        const uint32_t vsc = lds32(sb + 2 * KVA_CODES + 128 + (ra + 8) * 4);
        const uint32_t vsd = lds32(sb + 2 * KVA_CODES + 128 + (rb + 8) * 4);
        const uint32_t vba = lds32(sb + 2 * KVA_CODES + 192 + ra * 4), vbb = lds32(sb + 2 * KVA_CODES + 192 + rb * 4);
        const uint32_t vbc = lds32(sb + 2 * KVA_CODES + 192 + (ra + 8) * 4);
        const uint32_t vbd = lds32(sb + 2 * KVA_CODES + 192 + (rb + 8) * 4);
#pragma unroll
        for (int gg = 0; gg < 2; ++gg) {
            const uint32_t piece = (4 * gg + (gid >> 1)), half8 = (gid & 1) << 3;
            const uint2 A = lds64(sb + KVA_CODES + ra * KVA_HD + ((piece ^ (ra & 7)) << 4) + half8);
            const uint2 Bv = lds64(sb + KVA_CODES + rb * KVA_HD + ((piece ^ (rb & 7)) << 4) + half8);
            const uint2 C = lds64(sb + KVA_CODES + (ra + 8) * KVA_HD + ((piece ^ (ra & 7)) << 4) + half8);
            const uint2 D = lds64(sb + KVA_CODES + (rb + 8) * KVA_HD + ((piece ^ (rb & 7)) << 4) + half8);
            const uint32_t sab = kva_pair_f16<T>(vsa, vsb, gg), bab = kva_pair_f16<T>(vba, vbb, gg);
            const uint32_t scd = kva_pair_f16<T>(vsc, vsd, gg), bcd = kva_pair_f16<T>(vbc, vbd, gg);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t by = i & 3;
                const uint32_t sel = by | (by << 4) | ((4 + by) << 8) | ((4 + by) << 12);
                const uint32_t xa = prmt(i < 4 ? A.x : A.y, i < 4 ? Bv.x : Bv.y, sel);
                const uint32_t xc = prmt(i < 4 ? C.x : C.y, i < 4 ? D.x : D.y, sel);
                const uint32_t b0 = h2_sub_fma(lop3_and_or(xa, 0x00ff00ffu, 0x64006400u), sab, bab);
                const uint32_t b1 = h2_sub_fma(lop3_and_or(xc, 0x00ff00ffu, 0x64006400u), scd, bcd);
                mma_16816<__half>(o[8 * gg + i], pa[0][0], HI ? pa[NH - 1][0] : 0u, pa[0][1],
                                  HI ? pa[NH - 1][1] : 0u, b0, b1);
            }
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    grid_dep_launch();

    // ---- merge the four warps' softmax states into one part a head ----
#pragma unroll
    for (int hf = 0; hf < NH; ++hf) {
        l[hf] += __shfl_xor_sync(0xffffffffu, l[hf], 1);
        l[hf] += __shfl_xor_sync(0xffffffffu, l[hf], 2);
    }
    __syncthreads();  // every warp is done with its ring
    float* cm = reinterpret_cast<float*>(kva_smem);  // [NW][16]
    float* cl = cm + KVA_NW * KVA_MAX_G;             // [NW][16]
    float* co = cl + KVA_NW * KVA_MAX_G;             // [NW][16][128]
#pragma unroll
    for (int hf = 0; hf < NH; ++hf) {
        const int hh = gid + 8 * hf;
        if (c == 0) {
            cm[warp * KVA_MAX_G + hh] = m[hf];
            cl[warp * KVA_MAX_G + hh] = l[hf];
        }
#pragma unroll
        for (int t = 0; t < 16; ++t)
#pragma unroll
            for (int j = 0; j < 2; ++j)
                co[(warp * KVA_MAX_G + hh) * KVA_HD + 64 * (t >> 3) + 8 * (2 * c + j) + (t & 7)] = o[t][2 * hf + j];
    }
    __syncthreads();
    const int d = threadIdx.x;
    for (int hh = 0; hh < a.G; ++hh) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < KVA_NW; ++w) M = fmaxf(M, cm[w * KVA_MAX_G + hh]);
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < KVA_NW; ++w) {
                const float mw = cm[w * KVA_MAX_G + hh];
                const float sw = mw == -INFINITY ? 0.0f : exp2f(mw - M);
                L += cl[w * KVA_MAX_G + hh] * sw;
                O += co[(w * KVA_MAX_G + hh) * KVA_HD + d] * sw;
            }
        }
        const int head = kvh * a.G + hh;
        const size_t bh = size_t(b) * a.H + head;
        if (a.nsplit == 1) {
            const float sink = a.sinks ? a.sinks[head] * KVA_LOG2E : -INFINITY;
            a.out[bh * KVA_HD + d] = kva_finish<T>(M, L, O, sink);
        } else {
            const size_t part = bh * a.nsplit + split;
            if (d == 0) {
                a.part_ml[2 * part] = M;
                a.part_ml[2 * part + 1] = L;
            }
            a.part_o[part * KVA_HD + d] = O;
        }
    }
}

// One CTA a (row, head), one thread a dim: the head's parts joined with its sink.
template <typename T>
__global__ void __launch_bounds__(KVA_HD) kv_join_kernel(const KvaArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const size_t bh = blockIdx.x;
    const int d = threadIdx.x, head = int(bh % a.H);
    const float* ml = a.part_ml + bh * a.nsplit * 2;
    const float* po = a.part_o + bh * a.nsplit * KVA_HD;
    float M = -INFINITY;
    for (int j = 0; j < a.nsplit; ++j) M = fmaxf(M, ml[2 * j]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
        for (int j = 0; j < a.nsplit; ++j) {
            const float mj = ml[2 * j];
            if (mj == -INFINITY) continue;
            const float w = exp2f(mj - M);
            L += ml[2 * j + 1] * w;
            O += po[size_t(j) * KVA_HD + d] * w;
        }
    }
    const float sink = a.sinks ? a.sinks[head] * KVA_LOG2E : -INFINITY;
    a.out[bh * KVA_HD + d] = kva_finish<T>(M, L, O, sink);
}

// ---- host ----------------------------------------------------------------------------------------

// Blocks a (row, kv head): enough CTAs for KVA_CTAS_PER_SM a SM, at least KVA_MIN_BLOCK keys a block.
void kv_attend_splits(int B, int KVH, int n, int sms, int* nsplit, int* block) {
    const int groups = B * KVH;
    const int want = (sms * KVA_CTAS_PER_SM + groups - 1) / groups;
    int ns = max(1, min(want, (n + KVA_MIN_BLOCK - 1) / KVA_MIN_BLOCK));
    int blk = ((max(n, 1) + ns - 1) / ns + KVA_NW * KVA_KEYS - 1) / (KVA_NW * KVA_KEYS) * (KVA_NW * KVA_KEYS);
    ns = max(1, (n + blk - 1) / blk);
    *nsplit = ns;
    *block = blk;
}

size_t kv_attend_workspace_bytes(int B, int H, int KVH, int n, int sms) {
    int ns, blk;
    kv_attend_splits(B, KVH, n, sms, &ns, &blk);
    return ns == 1 ? 0 : size_t(B) * H * ns * (2 + KVA_HD) * sizeof(float);
}

bool kv_attend_shape_ok(int B, int H, int KVH, int n, int cap, int head_dim) {
    // B and KVH are the attend kernel's grid z and y (at most 65535 each)
    if (B < 1 || B > 65535 || H < 1 || KVH < 1 || KVH > 65535 || H % KVH || head_dim != KVA_HD) return false;
    const int G = H / KVH;
    return G <= KVA_MAX_G && n >= 0 && n <= cap && cap >= 1;
}

template <typename K>
static int kva_launch(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, const KvaArgs& a) {
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
    return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? LQ_OK : LQ_E_CUDA;
}

template <typename T, bool HI>
static int kva_run_t(const KvaArgs& a, int B, cudaStream_t st) {
    // The shared-memory limit is an attribute of the function on the CURRENT device: set it on every call (a
    // cheap host call), so a process that attends on several GPUs sets it on each and no host flag is shared.
    if (cudaFuncSetAttribute(kv_attend_kernel<T, HI>, cudaFuncAttributeMaxDynamicSharedMemorySize, KVA_SMEM) !=
        cudaSuccess)
        return LQ_E_CUDA;
    int rc = kva_launch(kv_attend_kernel<T, HI>, dim3(a.nsplit, a.KVH, B), dim3(KVA_NW * 32), KVA_SMEM, st, a);
    if (rc || a.nsplit == 1) return rc;
    return kva_launch(kv_join_kernel<T>, dim3(B * a.H), dim3(KVA_HD), 0, st, a);
}

int kv_attend_run(const void* q, const uint32_t* kq, const void* ks, const void* kb, const uint32_t* vq,
                  const void* vs, const void* vb, const int32_t* start, int n, const float* sinks, float scale, int B,
                  int H, int KVH, int cap, int dtype, void* workspace, size_t workspace_bytes, void* out,
                  cudaStream_t st) {
    KvaArgs a = {};
    a.q = static_cast<const uint16_t*>(q);
    a.kq = kq;
    a.ks = static_cast<const uint32_t*>(ks);
    a.kb = static_cast<const uint32_t*>(kb);
    a.vq = vq;
    a.vs = static_cast<const uint32_t*>(vs);
    a.vb = static_cast<const uint32_t*>(vb);
    a.start = start;
    a.sinks = sinks;
    a.scale_log2 = scale * KVA_LOG2E;
    a.n = n;
    a.H = H;
    a.KVH = KVH;
    a.G = H / KVH;
    a.cap = cap;
    kv_attend_splits(B, KVH, n, device_info().sm_count, &a.nsplit, &a.block);
    if (a.nsplit > 1) {
        const size_t need = size_t(B) * H * a.nsplit * (2 + KVA_HD) * sizeof(float);
        if (!workspace || workspace_bytes < need) return LQ_E_ARG;
        a.part_ml = static_cast<float*>(workspace);
        a.part_o = a.part_ml + size_t(B) * H * a.nsplit * 2;
    }
    a.out = static_cast<uint16_t*>(out);
    const bool hi = a.G > 8;
    if (dtype == LQ_BF16)
        return hi ? kva_run_t<__nv_bfloat16, true>(a, B, st) : kva_run_t<__nv_bfloat16, false>(a, B, st);
    return hi ? kva_run_t<__half, true>(a, B, st) : kva_run_t<__half, false>(a, B, st);
}

}  // namespace lq
