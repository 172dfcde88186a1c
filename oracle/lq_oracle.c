/*
 * CPU oracle for the MLX affine group-quantized matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load this library, and
 * only as the checker (or as the timed CPU restatement).  The product path
 * (locals_b200) never calls it.
 *
 * Each function restates the arithmetic of the reference (Generated-Computers/
 * Locals, which computes through MLX 0.32.3 and its own Metal kernels):
 *
 *   lqo_quantize      MLX mx.quantize(w, group_size, bits) (affine mode), the
 *                     call the reference makes in tests/test_kernel_patching.py:163
 *                     and tests/test_nax_kernel.py:16.  MLX itself is not in the
 *                     reference tree (uv.lock:376-377 pins mlx 0.32.3); this is a
 *                     restatement of its published affine algorithm: per group,
 *                     scale = (max - min) / (2^bits - 1), signed towards the
 *                     larger-magnitude edge, the edge made exact (q0 = rint(edge /
 *                     scale), scale = edge / q0, bias = edge), codes =
 *                     clip(rint((w - bias) / scale), 0, 2^bits - 1).
 *                     PARITY UNPINNED: no MLX in this environment to compare to.
 *   lqo_unpack        bit order of locals/kernels.py:31-35,63-64 and
 *                     locals/qmv_multi.py:47-54: code i of word j is K index
 *                     (32/bits)*j + i at bits bits*i (low bits first).
 *   lqo_dequantize    w = scale * q + bias (locals/kernels.py:64,77).
 *   lqo_qmm           y = sum_g scale_g * sum_{k in g} q_k x_k + bias_g * sum_{k in g} x_k
 *                     with float32 accumulation, the factoring of
 *                     locals/qmv_multi.py:57-75 and locals/qmv_frag.py:356-359.
 *   lqo_router        float32 x @ W^T of 16-bit x and W (locals/moe.py:86-89,134-139).
 *   lqo_topk_softmax  softmax over experts in float32, the k largest (ties to the
 *                     lower index), renormalised to sum 1 (the routing of a softmax MoE block;
 *                     tie rule of locals/moe.py:32-35,51-61, renormalisation of
 *                     locals/moe.py:63-70).
 *   lqo_topk_sigmoid  locals/moe.py:36-82 (sigmoid scores, NaN -> 0, ties to the
 *                     lower index, renormalised).
 *   lqo_group         counting sort of expert ids (locals/moe_kernel.py:28-66),
 *                     made stable (pairs of one expert in ascending pair id).
 *   lqo_swiglu        silu(g) * u with the rounding points of locals/moe.py:284-289.
 *   lqo_combine       sum_k w_k * y_k in float32, slots in their order
 *                     (locals/moe.py:339-348).
 *   lqo_add_rms / lqo_combine_norm   locals/norm_kernel.py:16-85, locals/moe.py:353-389.
 *   lqo_kv_attend     decode attention over an 8-bit key/value cache with sinks and left
 *                     padding (locals/qkv.py:30-249): keys and values dequantized in float32
 *                     (qkv.py:50-53), scores scale * q.k, softmax over the keys start[b] .. n-1
 *                     and the head's sink (qkv.py:_PASS2), in double here.
 *
 * Build: oracle/build.py (gcc -O2 -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define LQO_F16 0
#define LQO_BF16 1
#define LQO_F32 2

/* ---- 16-bit float rounding (round to nearest even), written from the IEEE formats ---- */

static float bits_to_float(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint32_t float_to_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

uint16_t lqo_f32_to_bf16(float f) {
    uint32_t u = float_to_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

float lqo_bf16_to_f32(uint16_t h) { return bits_to_float((uint32_t)h << 16); }

uint16_t lqo_f32_to_f16(float f) {
    uint32_t u = float_to_bits(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520: inf */
    if (a < 0x38800000u) {                                   /* below the smallest normal 2^-14 */
        /* subnormal: value / 2^-24 rounded to an integer, ties to even */
        float v = bits_to_float(a) * 16777216.0f;            /* exact: power of two */
        float r = rintf(v);
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t mant = a & 0x7fffffu;
    int32_t exp = (int32_t)(a >> 23) - 127 + 15;
    uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
    uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h += 1u; /* carry may bump the exponent: correct */
    return (uint16_t)(sign | h);
}

float lqo_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    if (exp == 0) {
        float v = (float)mant * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (exp == 31) return bits_to_float(sign | 0x7f800000u | (mant << 13));
    return bits_to_float(sign | ((exp - 15 + 127) << 23) | (mant << 13));
}

float lqo_round1(float v, int dtype) {
    if (dtype == LQO_BF16) return lqo_bf16_to_f32(lqo_f32_to_bf16(v));
    if (dtype == LQO_F16) return lqo_f16_to_f32(lqo_f32_to_f16(v));
    return v;
}

void lqo_round(float* a, int64_t n, int dtype) {
    for (int64_t i = 0; i < n; i++) a[i] = lqo_round1(a[i], dtype);
}

/* ---- format ---- */

void lqo_quantize(const float* w, int64_t N, int64_t K, int bits, int group, uint32_t* wq, float* scales,
                  float* biases) {
    const float n_bins = (float)((1 << bits) - 1);
    const float eps = 1e-7f;
    const int per_word = 32 / bits;
    const int64_t words = K / per_word;
    const int64_t ng = K / group;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++) {
        for (int64_t g = 0; g < ng; g++) {
            const float* wg = w + n * K + g * group;
            float w_min = INFINITY, w_max = -INFINITY;
            for (int j = 0; j < group; j++) {
                w_max = fmaxf(w_max, wg[j]);
                w_min = fminf(w_min, wg[j]);
            }
            int mask = fabsf(w_min) > fabsf(w_max);
            float scale = fmaxf((w_max - w_min) / n_bins, eps);
            scale = mask ? scale : -scale;
            float edge = mask ? w_min : w_max;
            float q0 = rintf(edge / scale);
            float bias = 0.0f;
            if (q0 != 0.0f) {
                scale = edge / q0;
                bias = edge;
            }
            scales[n * ng + g] = scale;
            biases[n * ng + g] = bias;
            for (int j = 0; j < group; j++) {
                float q = rintf((wg[j] - bias) / scale);
                q = fminf(fmaxf(q, 0.0f), n_bins);
                int64_t k = g * group + j;
                int64_t word = n * words + k / per_word;
                int sh = (int)(k % per_word) * bits;
                if (sh == 0) wq[word] = 0;
                wq[word] |= ((uint32_t)q) << sh;
            }
        }
    }
}

void lqo_unpack(const uint32_t* wq, int64_t N, int64_t K, int bits, uint8_t* codes) {
    const int per_word = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int64_t words = K / per_word;
    for (int64_t n = 0; n < N; n++)
        for (int64_t k = 0; k < K; k++)
            codes[n * K + k] = (uint8_t)((wq[n * words + k / per_word] >> ((k % per_word) * bits)) & mask);
}

void lqo_dequantize(const uint32_t* wq, const float* s, const float* b, int64_t N, int64_t K, int bits, int group,
                    float* w) {
    const int per_word = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int64_t words = K / per_word, ng = K / group;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++)
        for (int64_t k = 0; k < K; k++) {
            uint32_t q = (wq[n * words + k / per_word] >> ((k % per_word) * bits)) & mask;
            w[n * K + k] = s[n * ng + k / group] * (float)q + b[n * ng + k / group];
        }
}

/* y (M, N) = x (M, K) . dequant(W)^T, float32 accumulation per group (MLX qmv factoring). */
void lqo_qmm(const float* x, int64_t M, int64_t K, const uint32_t* wq, const float* s, const float* b, int64_t N,
             int bits, int group, float* y, int nthreads) {
    const int per_word = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int64_t words = K / per_word, ng = K / group;
    float* xsum = (float*)malloc(sizeof(float) * (size_t)(M * ng));
    for (int64_t m = 0; m < M; m++)
        for (int64_t g = 0; g < ng; g++) {
            float t = 0.0f;
            for (int j = 0; j < group; j++) t += x[m * K + g * group + j];
            xsum[m * ng + g] = t;
        }
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel
    {
        float* q = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            const uint32_t* row = wq + n * words;
            for (int64_t k = 0; k < K; k++) q[k] = (float)((row[k / per_word] >> ((k % per_word) * bits)) & mask);
            for (int64_t m = 0; m < M; m++) {
                const float* xm = x + m * K;
                float acc = 0.0f;
                for (int64_t g = 0; g < ng; g++) {
                    float d = 0.0f;
                    const float* qg = q + g * group;
                    const float* xg = xm + g * group;
                    for (int j = 0; j < group; j++) d += qg[j] * xg[j];
                    acc += s[n * ng + g] * d + b[n * ng + g] * xsum[m * ng + g];
                }
                y[m * N + n] = acc;
            }
        }
        free(q);
    }
    free(xsum);
}

/* ---- MoE ---- */

void lqo_router(const float* x, const float* w, int64_t T, int64_t E, int64_t D, float* logits) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t t = 0; t < T; t++)
        for (int64_t e = 0; e < E; e++) {
            float acc = 0.0f;
            for (int64_t d = 0; d < D; d++) acc += x[t * D + d] * w[e * D + d];
            logits[t * E + e] = acc;
        }
}

/* k rounds of "largest remaining score, ties to the lower index". scores with NaN are never picked
   before a number; the result always names k distinct experts. */
static void topk_pick(const float* sc, int E, int k, uint32_t* inds, float* picked) {
    unsigned char used[4096];
    memset(used, 0, (size_t)E);
    for (int r = 0; r < k; r++) {
        int best = -1;
        float bv = 0.0f;
        for (int e = 0; e < E; e++) {
            if (used[e]) continue;
            float v = sc[e];
            if (best < 0 || (!isnan(v) && (isnan(bv) || v > bv))) {
                best = e;
                bv = v;
            }
        }
        used[best] = 1;
        inds[r] = (uint32_t)best;
        picked[r] = bv;
    }
}

void lqo_topk_softmax(const float* logits, int64_t T, int E, int k, uint32_t* inds, float* weights) {
    for (int64_t t = 0; t < T; t++) {
        const float* l = logits + t * E;
        float mx = -INFINITY;
        for (int e = 0; e < E; e++) mx = fmaxf(mx, l[e]);
        float p[4096];
        float tot = 0.0f;
        for (int e = 0; e < E; e++) {
            p[e] = expf(l[e] - mx);
            tot += p[e];
        }
        for (int e = 0; e < E; e++) p[e] = p[e] / tot;
        float picked[64];
        topk_pick(p, E, k, inds + t * k, picked);
        float s = 0.0f;
        for (int r = 0; r < k; r++) s += picked[r];
        for (int r = 0; r < k; r++) weights[t * k + r] = picked[r] / s;
    }
}

void lqo_topk_sigmoid(const float* logits, int64_t T, int E, int k, uint32_t* inds, float* weights) {
    for (int64_t t = 0; t < T; t++) {
        float p[4096];
        for (int e = 0; e < E; e++) {
            float v = 1.0f / (1.0f + expf(-logits[t * E + e]));
            p[e] = isnan(v) ? 0.0f : v;
        }
        float picked[64];
        topk_pick(p, E, k, inds + t * k, picked);
        float s = 0.0f;
        for (int r = 0; r < k; r++) s += picked[r];
        for (int r = 0; r < k; r++) weights[t * k + r] = picked[r] / s;
    }
}

void lqo_group(const uint32_t* inds, int64_t P, int E, int32_t* order, int32_t* starts, int32_t* experts,
               int32_t* nseg) {
    int32_t* cnt = (int32_t*)calloc((size_t)E, sizeof(int32_t));
    int32_t* base = (int32_t*)calloc((size_t)E, sizeof(int32_t));
    for (int64_t p = 0; p < P; p++) cnt[inds[p]]++;
    int32_t at = 0, s = 0;
    for (int e = 0; e < E; e++) {
        base[e] = at;
        if (cnt[e] > 0) {
            starts[s] = at;
            experts[s] = e;
            s++;
        }
        at += cnt[e];
    }
    starts[s] = at;
    *nseg = s;
    for (int64_t p = 0; p < P; p++) order[base[inds[p]]++] = (int32_t)p;
    free(cnt);
    free(base);
}

void lqo_swiglu(const float* g, const float* u, int64_t n, int dtype, float* h) {
    for (int64_t i = 0; i < n; i++) {
        float gt = lqo_round1(g[i], dtype), ut = lqo_round1(u[i], dtype);
        float sig = lqo_round1(1.0f / (1.0f + expf(-gt)), dtype);
        float act = lqo_round1(gt * sig, dtype);
        h[i] = lqo_round1(act * ut, dtype);
    }
}

void lqo_combine(const float* ys, const float* w, int64_t T, int k, int64_t D, float* y) {
    for (int64_t t = 0; t < T; t++)
        for (int64_t d = 0; d < D; d++) {
            float acc = 0.0f;
            for (int r = 0; r < k; r++) acc += ys[(t * k + r) * D + d] * w[t * k + r];
            y[t * D + d] = acc;
        }
}

/* Residual add + RMS norm (locals/norm_kernel.py:16-85): h = round(x + r); n = round(w * round(h * inv)) with
 * inv = 1 / sqrt(sum(h^2) / D + eps), the sum of squares in float32. Inputs hold values already in dtype. */
void lqo_add_rms(const float* x, const float* r, const float* w, int64_t rows, int64_t D, float eps, int dtype,
                 float* h, float* n) {
    for (int64_t t = 0; t < rows; t++) {
        float sq = 0.0f;
        for (int64_t d = 0; d < D; d++) {
            const float v = lqo_round1(x[t * D + d] + r[t * D + d], dtype);
            h[t * D + d] = v;
            sq += v * v;
        }
        const float inv = 1.0f / sqrtf(sq / (float)D + eps);
        for (int64_t d = 0; d < D; d++)
            n[t * D + d] = lqo_round1(w[d] * lqo_round1(h[t * D + d] * inv, dtype), dtype);
    }
}

/* The MoE combine with the shared expert, the layer's residual add and the next norm (locals/moe.py:353-389):
 * y = round(sum_k weights[t,k] * ys[t*k+k]) (float32, slots in order); if shared: y = round(y + shared);
 * y = round(res + y); n as lqo_add_rms with nw. ys rows in slot order (row t*k + r); shared may be NULL. */
void lqo_combine_norm(const float* ys, const float* w, const float* shared, const float* res, const float* nw,
                      int64_t T, int k, int64_t D, float eps, int dtype, float* y, float* n) {
    for (int64_t t = 0; t < T; t++) {
        float sq = 0.0f;
        for (int64_t d = 0; d < D; d++) {
            float acc = 0.0f;
            for (int r = 0; r < k; r++) acc += ys[(t * k + r) * D + d] * w[t * k + r];
            float v = lqo_round1(acc, dtype);
            if (shared) v = lqo_round1(v + shared[t * D + d], dtype);
            v = lqo_round1(res[t * D + d] + v, dtype);
            y[t * D + d] = v;
            sq += v * v;
        }
        const float inv = 1.0f / sqrtf(sq / (float)D + eps);
        for (int64_t d = 0; d < D; d++)
            n[t * D + d] = lqo_round1(nw[d] * lqo_round1(y[t * D + d] * inv, dtype), dtype);
    }
}

/* Decode attention over an 8-bit key/value cache (locals/qkv.py:30-249). q (B, H, HD) float; kq, vq uint32
 * (B, KVH, cap, HD/4), four codes a word, low byte first; ks, kb, vs, vb (B, KVH, cap, HD/64) float. Query head
 * h reads kv head h / (H / KVH). For row b the keys max(start[b], 0) .. n-1 (start NULL: from 0); element d of
 * a key is the float32 s * code + b of its group (qkv.py:50-53); score = scale * sum_d q_d k_d; out = sum p v /
 * (sum p + exp(sink - M)) with p = exp(score - M), M the largest of the scores and the sink (sinks NULL: no
 * sink; qkv.py:_PASS2); 0 where nothing is attended. Double accumulation, out (B, H, HD) float. */
void lqo_kv_attend(const float* q, const uint32_t* kq, const float* ks, const float* kb, const uint32_t* vq,
                   const float* vs, const float* vb, const int32_t* start, int64_t n, const float* sinks, float scale,
                   int64_t B, int64_t H, int64_t KVH, int64_t cap, int64_t HD, float* out) {
    const int64_t G = H / KVH, WPR = HD / 4, GPR = HD / 64;
#pragma omp parallel for schedule(dynamic)
    for (int64_t bh = 0; bh < B * H; bh++) {
        const int64_t b = bh / H, h = bh % H, kh = h / G;
        const int64_t lo = start ? (start[b] > 0 ? start[b] : 0) : 0;
        const float* qr = q + bh * HD;
        const int64_t row0 = (b * KVH + kh) * cap;
        const int64_t cnt = n > lo ? n - lo : 0;
        double* sc = (double*)malloc((size_t)(cnt > 0 ? cnt : 1) * sizeof(double));
        double* o = (double*)calloc((size_t)HD, sizeof(double));
        double M = sinks ? (double)sinks[h] : -INFINITY;
        for (int64_t t = 0; t < cnt; t++) {
            const int64_t r = row0 + lo + t;
            double acc = 0.0;
            for (int64_t d = 0; d < HD; d++) {
                const uint32_t code = (kq[r * WPR + d / 4] >> (8 * (d % 4))) & 0xffu;
                const float k = ks[r * GPR + d / 64] * (float)code + kb[r * GPR + d / 64];
                acc += (double)qr[d] * (double)k;
            }
            sc[t] = acc * (double)scale;
            if (sc[t] > M) M = sc[t];
        }
        double L = (sinks && M > -INFINITY) ? exp((double)sinks[h] - M) : 0.0;
        for (int64_t t = 0; t < cnt; t++) {
            const int64_t r = row0 + lo + t;
            const double p = exp(sc[t] - M);
            L += p;
            for (int64_t d = 0; d < HD; d++) {
                const uint32_t code = (vq[r * WPR + d / 4] >> (8 * (d % 4))) & 0xffu;
                const float v = vs[r * GPR + d / 64] * (float)code + vb[r * GPR + d / 64];
                o[d] += p * (double)v;
            }
        }
        for (int64_t d = 0; d < HD; d++) out[bh * HD + d] = L > 0.0 ? (float)(o[d] / L) : 0.0f;
        free(sc);
        free(o);
    }
}
