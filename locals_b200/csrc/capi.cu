// The C ABI (include/lq.h): argument checks, then dispatch to the kernel families. Never aborts;
// every failure is an LQ_E_* code.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/lq.h"
#include "lq_host.h"
#include "qmv.h"

namespace lq {
int quantize_run(const void* w, int w_dt, int N, int K, int bits, int group, uint32_t* wq, void* s, void* b,
                 int sb_dt, cudaStream_t st);
int dequantize_run(const uint32_t* wq, const void* s, const void* b, int N, int K, int bits, int group, int dt,
                   void* out, cudaStream_t st);
int router_logits_run(const void* x, int x_dt, const void* w, int w_dt, float* logits, int T, int E, int D,
                      cudaStream_t st);
int route_topk_run(const float* logits, int T, int E, int k, int mode, uint32_t* inds, float* weights,
                   cudaStream_t st);
int group_run(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts, int32_t* nseg,
              int32_t* pos, cudaStream_t st);
int gather_rows_run(const void* x, const int32_t* order, int P, int k, int D, void* xs, cudaStream_t st);
int combine_run(const void* ys, const float* w, const int32_t* pos, void* y, int T, int k, int D, int dt,
                cudaStream_t st);
int router_topk_run(const void* x, int x_dt, const void* w, int w_dt, int T, int E, int D, int k, int mode,
                    uint32_t* inds, float* weights, float* logits, cudaStream_t st);
int tc_run(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K, int bits,
           int dtype, const int* p, cudaStream_t st);
bool tc_shape_ok(int M, int N, int K, int bits);
bool tcv_shape_ok(int M, int K, int bits);
int tcv_run(const void* x, int M, const QmvMats& mats, int nmat, int N, int K, int nout, void* const* outs,
            const int* seg_end, const int* ldo, int bits, int dtype, const int* p, cudaStream_t st);
int tcv_run_grouped(const void* xs, int P, const QmvMats& mats, int nmat, int N, int K, void* out,
                    const int32_t* starts, const int32_t* experts, const int32_t* nseg, int E, int bits, int dtype,
                    const int* p, cudaStream_t st);
bool tcvp_shape_ok(int M, int K, int bits);
int tcvp_run(const void* x, int M, const QmvMats& mats, int nmat, int N, int K, int nout, void* const* outs,
             const int* seg_end, const int* ldo, int bits, int dtype, int ntok, cudaStream_t st);
int tcvp_run_grouped(const void* xs, int P, const QmvMats& mats, int nmat, int N, int K, void* out,
                     const int32_t* starts, const int32_t* experts, const int32_t* nseg, int E, int bits, int dtype,
                     int ntok, cudaStream_t st);
bool norm_shape_ok(int D);
size_t qmm_dense_workspace_bytes(int N, int K);
int qmm_dense_gather_run(const void* x, const uint32_t* w, const void* s, const void* b, void* const* dst, int ndst,
                         int col_off, int ldo, int M, int N, int K, int bits, int dtype, void* workspace, const int* p,
                         cudaStream_t st);
bool qmm_dense_shape_ok(int M, int N, int K, int bits);
int qmm_dense_run(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K,
                  int bits, int dtype, void* workspace, const int* p, cudaStream_t st);
bool qmvg_shape_ok(int M, int K, int bits);
int qmvg_run(const void* x, const uint32_t* w, const void* s, const void* b, int nout, void* const* outs,
             const int* seg_end, const int* ldo, int M, int N, int K, int dtype, const int* p, cudaStream_t st);
bool qmvq_shape_ok(int M, int K, int bits);
int qmvq_run(const void* x, const uint32_t* w, const void* s, const void* b, int nout, void* const* outs,
             const int* seg_end, const int* ldo, int M, int N, int K, int bits, int dtype, const int* p,
             cudaStream_t st);
int qmvq_glu_run(const void* x, const uint32_t* w_gate, const void* s_gate, const void* b_gate, const uint32_t* w_up,
                 const void* s_up, const void* b_up, void* h, int M, int I, int K, int bits, int dtype, const int* p,
                 cudaStream_t st);
bool qmvqg_shape_ok(int max_rows, int N, int K, int bits);
int qmvqg_run(const void* x, const int32_t* gather, int gather_k, const int32_t* starts, const int32_t* experts,
              const int32_t* nseg, int P, int max_rows, int glu, const uint32_t* w0, const void* s0, const void* b0,
              const uint32_t* w1, const void* s1, const void* b1, void* out, int E, int N, int K, int bits, int dtype,
              cudaStream_t st);
bool qmvg_moe_ok(int mode, int k, int rows_e, int K, int sms);
int qmvg_moe_run(int mode, const void* x, const int32_t* experts, const int32_t* pos, const float* wts,
                 const uint32_t* w0, const void* s0, const void* b0, const uint32_t* w1, const void* s1, const void* b1,
                 void* out, int k, int E, int rows_e, int K, int dtype, cudaStream_t st);
bool moe_decode_ok(int E, int k, int D, int I);
size_t moe_decode_workspace_bytes(int E, int k, int D, int I);
int moe_decode_run(const void* x, int x_dt, const void* rw, int rw_dt, int E, int k, int mode, const uint32_t* const* w,
                   const void* const* s, const void* const* b, int D, int I, void* y, uint32_t* inds, float* wts,
                   void* work, size_t work_bytes, cudaStream_t st);
size_t peer_sync_bytes();
int peer_scatter_rows_run(const void* src, const int32_t* idx, const int32_t* starts, const int32_t* experts,
                          const int32_t* nseg, int bucket, int rows_max, int row_bytes, int dst_rows,
                          void* const* dst, int G, int rank, void* const* sync, cudaStream_t st);
int group_range_run(const uint32_t* inds, int P, int lo, int range, int32_t* order, int32_t* starts, int32_t* experts,
                    int32_t* nseg, int32_t* pos, cudaStream_t st);
int peer_gather_run(const void* src, int M, int n, int col_off, int ldo, int elem_bytes, void* const* dst, int G,
                    int rank, void* const* sync, cudaStream_t st);
bool kv_attend_shape_ok(int B, int H, int KVH, int n, int cap, int head_dim);
size_t kv_attend_workspace_bytes(int B, int H, int KVH, int n, int sms);
int kv_attend_run(const void* q, const uint32_t* kq, const void* ks, const void* kb, const uint32_t* vq,
                  const void* vs, const void* vb, const int32_t* start, int n, const float* sinks, float scale, int B,
                  int H, int KVH, int cap, int dtype, void* workspace, size_t workspace_bytes, void* out,
                  cudaStream_t st);
int add_rms_run(const void* x, const void* r, const void* w, void* h, void* n, int rows, int D, float eps, int dtype,
                cudaStream_t st);
int combine_norm_run(const void* ys, const float* wts, const int32_t* pos, const void* shared, const void* res,
                     const void* nw, void* y, void* n, int T, int K, int D, float eps, int dtype, cudaStream_t st);
int scatter_rows_run(const void* src, const int32_t* idx, int R, int row_bytes, void* dst, int dst_rows,
                     cudaStream_t st);
}  // namespace lq

using namespace lq;


static int check_common(const void* x, const uint32_t* w, const void* s, const void* b, int M, int N, int K, int bits,
                        int group_size, int dtype) {
    if (!x || !w || !s || !b) return LQ_E_ARG;
    if (!is16(dtype)) return LQ_E_UNSUPPORTED;
    if (bits != 4 && bits != 8) return LQ_E_UNSUPPORTED;
    if (group_size != 64) return LQ_E_UNSUPPORTED;
    if (M < 1 || N < 1 || K < 64 || K % 64) return LQ_E_SHAPE;
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(s, 4) || !aligned(b, 4)) return LQ_E_ALIGN;
    return check_device();
}

// Decode family for the library's own pick: the tensor-core family (tcv) once the weights of one call
// are large enough to keep the GPU streaming or the token tile is wide, else the mma.sync family (qmv),
// whose two CTAs per SM let one call's weights load while the previous call still runs. Measured on
// B200: qmv wins the 8 MB fused QKV projection up to 32 tokens; tcv wins the 25-50 MB 8-bit MLP
// projections from 16 tokens and everything from 33 tokens.
static bool prefer_tcv(int M, double weight_bytes, int K, int bits) {
    if (!tcv_shape_ok(M, K, bits)) return false;
    return M > 32 || (M > 8 && weight_bytes >= 24.0e6);
}

static QmvMats one_matrix(const uint32_t* w, const void* s, const void* b, int rows) {
    QmvMats m = {};
    m.w[0] = m.w[1] = w;
    m.s[0] = m.s[1] = s;
    m.b[0] = m.b[1] = b;
    m.rows_total[0] = m.rows_total[1] = rows;
    return m;
}

static int qmm_common(const void* x, const uint32_t* w, const void* s, const void* b, int nout, void* const* outs,
                      const int* widths, int M, int N, int K, int bits, int group_size, int dtype, const lq_cfg* cfg,
                      void* stream) {
    int rc = check_common(x, w, s, b, M, N, K, bits, group_size, dtype);
    if (rc) return rc;
    if (nout < 1 || nout > 3 || !outs) return LQ_E_ARG;
    QmvArgs a = {};
    a.M = M;
    a.N = N;
    a.K = K;
    int acc = 0;
    for (int i = 0; i < nout; ++i) {
        if (!outs[i] || widths[i] < 1) return LQ_E_ARG;
        acc += widths[i];
        a.out[i] = outs[i];
        a.seg_end[i] = acc;
        a.ldo[i] = widths[i];
    }
    if (acc != N) return LQ_E_SHAPE;
    a.nseg_out = nout;
    const int fam = cfg ? cfg->family : LQ_FAM_AUTO;
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (fam == LQ_FAM_TC || (fam == LQ_FAM_AUTO && M > 64 && nout == 1 && tc_shape_ok(M, N, K, bits))) {
        if (nout != 1) return LQ_E_UNSUPPORTED;
        if (!tc_shape_ok(M, N, K, bits)) return LQ_E_SHAPE;
        return finish(tc_run(x, w, s, b, outs[0], M, N, K, bits, dtype, cfg ? cfg->p : nullptr, st));
    }
    if (fam == LQ_FAM_QMVQ) {
        if (!qmvq_shape_ok(M, K, bits)) return LQ_E_SHAPE;
        return finish(qmvq_run(x, w, s, b, nout, outs, a.seg_end, a.ldo, M, N, K, bits, dtype, cfg->p, st));
    }
    if (fam == LQ_FAM_QMVG) {
        if (!qmvg_shape_ok(M, K, bits)) return LQ_E_SHAPE;
        return finish(qmvg_run(x, w, s, b, nout, outs, a.seg_end, a.ldo, M, N, K, dtype, cfg->p, st));
    }
    const QmvMats mats = one_matrix(w, s, b, N);
    if (fam == LQ_FAM_TCV) {
        if (cfg->p[3] == 1) {  // persistent form
            if (!tcvp_shape_ok(M, K, bits)) return LQ_E_SHAPE;
            return finish(tcvp_run(x, M, mats, 1, N, K, nout, outs, a.seg_end, a.ldo, bits, dtype, cfg->p[0], st));
        }
        if (!tcv_shape_ok(M, K, bits)) return LQ_E_SHAPE;
        return finish(tcv_run(x, M, mats, 1, N, K, nout, outs, a.seg_end, a.ldo, bits, dtype, cfg->p, st));
    }
    if (fam == LQ_FAM_AUTO && prefer_tcv(M, double(N) * K * bits / 8, K, bits)) {
        rc = tcv_run(x, M, mats, 1, N, K, nout, outs, a.seg_end, a.ldo, bits, dtype, nullptr, st);
        if (rc != LQ_E_SHAPE) return finish(rc);
    }
    // Few tokens of a 4-bit matrix: the folded group-per-warp family (codes fed raw to the MMA, scale and bias applied
    // per group in fp32) where it was measured fastest on B200 (CUDA graphs of weight copies larger than L2, us a
    // call, qmvq / qmvg / qmv): the fused QKV projection 6144 x 2560 at 1, 8 and 16 tokens (4.87 / 5.43 / 6.04,
    // 5.05 / 5.74 / 5.98, 6.86 / 7.10 / 7.04), and up to 8 tokens for K <= 4096 (4096 x 4096: 6.01 / 6.64 / 6.89 at
    // M=1; 9728 x 2560: 7.59 / 8.35 / 8.80 at M=1); qmv for the rest (2560 x 9728 at M=1: 10.63 against 12.67;
    // 4096 x 4096 at M=16: 7.57 against 7.95)
    const bool qmvq_auto = bits == 4 && qmvq_shape_ok(M, K, bits) && (M <= 8 ? K <= 4096 : (K <= 2560 && N <= 8192));
    if (fam == LQ_FAM_AUTO && qmvq_auto) {
        const int p[4] = {0, 0, 0, 0};
        rc = qmvq_run(x, w, s, b, nout, outs, a.seg_end, a.ldo, M, N, K, bits, dtype, p, st);
        if (rc != LQ_E_SHAPE) return finish(rc);
    }
    if (!qmv_shape_ok(K, bits)) {
        // a 4-bit K that is a multiple of 128 but not of 256: the tensor-core family
        if (fam != LQ_FAM_AUTO || !tcv_shape_ok(M, K, bits)) return LQ_E_SHAPE;
        return finish(tcv_run(x, M, mats, 1, N, K, nout, outs, a.seg_end, a.ldo, bits, dtype, nullptr, st));
    }
    return finish(qmv_run(x, M, mats, 1, a, bits, dtype, (cfg && fam == LQ_FAM_QMV) ? cfg->p : nullptr, M, 1, st));
}

extern "C" {

int lq_version(void) { return 100; }

const char* lq_strerror(int code) {
    switch (code) {
        case LQ_OK: return "ok";
        case LQ_E_ARG: return "bad argument";
        case LQ_E_SHAPE: return "unsupported shape";
        case LQ_E_ALIGN: return "misaligned pointer or stride";
        case LQ_E_UNSUPPORTED: return "unsupported bits/group/dtype";
        case LQ_E_CUDA: return "CUDA error";
        case LQ_E_DEVICE: return "not an sm_100 device";
        case LQ_E_SCRATCH: return "shape needs more than the 4 MiB static scratch buffer";
        default: return "unknown";
    }
}

const char* lq_last_cuda_error(void) { return last_cuda_error(); }

unsigned int lq_device_status(int clear) { return read_status(clear != 0); }

int lq_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N, int K,
           int bits, int group_size, int dtype, const lq_cfg* cfg, void* stream) {
    void* outs[1] = {y};
    const int widths[1] = {N};
    return qmm_common(x, w, scales, biases, 1, outs, widths, M, N, K, bits, group_size, dtype, cfg, stream);
}

int lq_qmm_split(const void* x, const uint32_t* w, const void* scales, const void* biases, int nout, void* const* outs,
                 const int* widths, int M, int N, int K, int bits, int group_size, int dtype, const lq_cfg* cfg,
                 void* stream) {
    if (!widths) return LQ_E_ARG;
    return qmm_common(x, w, scales, biases, nout, outs, widths, M, N, K, bits, group_size, dtype, cfg, stream);
}

int lq_qmm_glu(const void* x, const uint32_t* w_gate, const void* s_gate, const void* b_gate, const uint32_t* w_up,
               const void* s_up, const void* b_up, void* h, int M, int I, int K, int bits, int group_size, int dtype,
               const lq_cfg* cfg, void* stream) {
    int rc = check_common(x, w_gate, s_gate, b_gate, M, I, K, bits, group_size, dtype);
    if (rc) return rc;
    if (!w_up || !s_up || !b_up || !h) return LQ_E_ARG;
    if (!aligned(w_up, 16) || !aligned(s_up, 4) || !aligned(b_up, 4)) return LQ_E_ALIGN;
    QmvArgs a = {};
    a.M = M;
    a.N = I;
    a.K = K;
    a.out[0] = h;
    a.seg_end[0] = I;
    a.ldo[0] = I;
    a.nseg_out = 1;
    QmvMats m = {};
    m.w[0] = w_gate;
    m.s[0] = s_gate;
    m.b[0] = b_gate;
    m.w[1] = w_up;
    m.s[1] = s_up;
    m.b[1] = b_up;
    m.rows_total[0] = m.rows_total[1] = I;
    const int fam = cfg ? cfg->family : LQ_FAM_AUTO;
    void* outs[1] = {h};
    if (fam == LQ_FAM_QMVQ) {
        if (!qmvq_shape_ok(M, K, bits)) return LQ_E_SHAPE;
        return finish(qmvq_glu_run(x, w_gate, s_gate, b_gate, w_up, s_up, b_up, h, M, I, K, bits, dtype, cfg->p,
                                   reinterpret_cast<cudaStream_t>(stream)));
    }
    if (fam == LQ_FAM_TCV) {
        if (cfg->p[3] == 1) {
            if (!tcvp_shape_ok(M, K, bits)) return LQ_E_SHAPE;
            return finish(tcvp_run(x, M, m, 2, I, K, 1, outs, a.seg_end, a.ldo, bits, dtype, cfg->p[0],
                                   reinterpret_cast<cudaStream_t>(stream)));
        }
        if (!tcv_shape_ok(M, K, bits)) return LQ_E_SHAPE;
        return finish(tcv_run(x, M, m, 2, I, K, 1, outs, a.seg_end, a.ldo, bits, dtype, cfg->p,
                              reinterpret_cast<cudaStream_t>(stream)));
    }
    // up to 16 tokens: gate and up in one folded kernel over every SM (B200, us a call on 9728 x 2560 pairs, qmvq
    // against the previous choice: 8-bit 15.2 / 25.2 (qmv) at M=1, 21.1 / 24.0 (tcv) at M=16; 4-bit 11.5 / 14.6 at
    // M=1, 14.5 / 22.1 at M=16)
    if (fam == LQ_FAM_AUTO && qmvq_shape_ok(M, K, bits)) {
        rc = qmvq_glu_run(x, w_gate, s_gate, b_gate, w_up, s_up, b_up, h, M, I, K, bits, dtype, nullptr,
                          reinterpret_cast<cudaStream_t>(stream));
        if (rc != LQ_E_SHAPE) return finish(rc);
    }
    if (fam == LQ_FAM_AUTO && prefer_tcv(M, 2.0 * I * K * bits / 8, K, bits)) {
        rc = tcv_run(x, M, m, 2, I, K, 1, outs, a.seg_end, a.ldo, bits, dtype, nullptr,
                     reinterpret_cast<cudaStream_t>(stream));
        if (rc != LQ_E_SHAPE) return finish(rc);
    }
    if (!qmv_shape_ok(K, bits)) return LQ_E_SHAPE;
    return finish(qmv_run(x, M, m, 2, a, bits, dtype, (cfg && fam == LQ_FAM_QMV) ? cfg->p : nullptr, M, 1,
                          reinterpret_cast<cudaStream_t>(stream)));
}

int lq_quantize(const void* w, int w_dtype, int N, int K, int bits, int group_size, uint32_t* wq, void* scales,
                void* biases, int sb_dtype, void* stream) {
    if (!w || !wq || !scales || !biases) return LQ_E_ARG;
    if (bits < 2 || bits > 8 || (32 % bits) != 0) return LQ_E_UNSUPPORTED;
    if (group_size < 32 / bits || group_size % (32 / bits) || K % group_size || N < 1 || K < 1) return LQ_E_SHAPE;
    if (w_dtype != LQ_F32 && !is16(w_dtype)) return LQ_E_ARG;
    if (sb_dtype != LQ_F32 && !is16(sb_dtype)) return LQ_E_ARG;
    int rc = check_device();
    if (rc) return rc;
    return finish(quantize_run(w, w_dtype, N, K, bits, group_size, wq, scales, biases, sb_dtype,
                               reinterpret_cast<cudaStream_t>(stream)));
}

int lq_dequantize(const uint32_t* wq, const void* scales, const void* biases, int N, int K, int bits, int group_size,
                  int dtype, void* w_out, void* stream) {
    if (!wq || !scales || !biases || !w_out) return LQ_E_ARG;
    if (bits < 2 || bits > 8 || (32 % bits) != 0) return LQ_E_UNSUPPORTED;
    if (group_size < 32 / bits || K % group_size || N < 1 || K < 1) return LQ_E_SHAPE;
    if (dtype != LQ_F32 && !is16(dtype)) return LQ_E_ARG;
    int rc = check_device();
    if (rc) return rc;
    return finish(dequantize_run(wq, scales, biases, N, K, bits, group_size, dtype, w_out,
                                 reinterpret_cast<cudaStream_t>(stream)));
}

int lq_router_logits(const void* x, int x_dtype, const void* w, int w_dtype, float* logits, int T, int E, int D,
                     void* stream) {
    if (!x || !w || !logits) return LQ_E_ARG;
    if (!is16(x_dtype) || !is16(w_dtype)) return LQ_E_UNSUPPORTED;
    if (T < 1 || E < 1 || D < 8 || D % 8) return LQ_E_SHAPE;
    if (!aligned(x, 16) || !aligned(w, 16)) return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    return finish(router_logits_run(x, x_dtype, w, w_dtype, logits, T, E, D, reinterpret_cast<cudaStream_t>(stream)));
}

int lq_route_topk(const float* logits, int T, int E, int k, int mode, uint32_t* inds, float* weights, void* stream) {
    if (!logits || !inds || !weights) return LQ_E_ARG;
    if (mode != 0 && mode != 1) return LQ_E_ARG;
    if (T < 1 || E < 1 || E > 1024 || k < 1 || k > 32 || k > E) return LQ_E_SHAPE;
    int rc = check_device();
    if (rc) return rc;
    return finish(route_topk_run(logits, T, E, k, mode, inds, weights, reinterpret_cast<cudaStream_t>(stream)));
}

int lq_moe_route(const void* x, int x_dtype, const void* w, int w_dtype, int T, int E, int D, int k, int mode,
                 uint32_t* inds, float* weights, float* logits, void* stream) {
    if (!x || !w || !inds || !weights) return LQ_E_ARG;
    if (!is16(x_dtype) || !is16(w_dtype)) return LQ_E_UNSUPPORTED;
    if (mode != 0 && mode != 1) return LQ_E_ARG;
    if (T < 1 || E < 1 || E > 1024 || k < 1 || k > 32 || k > E || D < 8 || D % 8) return LQ_E_SHAPE;
    if (!aligned(x, 16) || !aligned(w, 16)) return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    return finish(router_topk_run(x, x_dtype, w, w_dtype, T, E, D, k, mode, inds, weights, logits,
                                  reinterpret_cast<cudaStream_t>(stream)));
}

int lq_moe_group(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts, int32_t* nseg,
                 int32_t* pos, void* stream) {
    if (!inds || !order || !starts || !experts || !nseg) return LQ_E_ARG;
    if (P < 1 || E < 1 || E > 8192) return LQ_E_SHAPE;
    int rc = check_device();
    if (rc) return rc;
    return finish(group_run(inds, P, E, order, starts, experts, nseg, pos, reinterpret_cast<cudaStream_t>(stream)));
}

int lq_moe_gather(const void* x, const int32_t* order, int P, int k, int D, void* xs, void* stream) {
    if (!x || !order || !xs) return LQ_E_ARG;
    if (P < 1 || k < 1 || D < 8 || D % 8) return LQ_E_SHAPE;
    if (!aligned(x, 16) || !aligned(xs, 16)) return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    return finish(gather_rows_run(x, order, P, k, D, xs, reinterpret_cast<cudaStream_t>(stream)));
}

int lq_moe_experts(const void* xs, const int32_t* starts, const int32_t* experts, const int32_t* nseg, int P,
                   int max_rows, int glu, const uint32_t* w0, const void* s0, const void* b0, const uint32_t* w1,
                   const void* s1, const void* b1, void* out, int E, int N, int K, int bits, int group_size, int dtype,
                   const int32_t* gather_order, int gather_k, void* stream) {
    int rc = check_common(xs, w0, s0, b0, P, N, K, bits, group_size, dtype);
    if (rc) return rc;
    if (!starts || !experts || !nseg || !out) return LQ_E_ARG;
    if (glu && (!w1 || !s1 || !b1)) return LQ_E_ARG;
    if (glu && (!aligned(w1, 16) || !aligned(s1, 4) || !aligned(b1, 4))) return LQ_E_ALIGN;
    if (E < 1 || max_rows < 1) return LQ_E_SHAPE;
    if (!qmv_shape_ok(K, bits) && (gather_order || !tcv_shape_ok(P, K, bits))) return LQ_E_SHAPE;
    if (int64_t(E) * N > INT32_MAX) return LQ_E_SHAPE;
    QmvArgs a = {};
    a.M = P;
    a.N = N;
    a.K = K;
    a.out[0] = out;
    a.seg_end[0] = N;
    a.ldo[0] = N;
    a.nseg_out = 1;
    a.grouped = 1;
    a.starts = starts;
    a.experts = experts;
    a.nseg = nseg;
    a.n_experts = E;
    QmvMats m = {};
    m.w[0] = w0;
    m.s[0] = s0;
    m.b[0] = b0;
    m.w[1] = glu ? w1 : w0;
    m.s[1] = glu ? s1 : s0;
    m.b[1] = glu ? b1 : b0;
    m.rows_total[0] = m.rows_total[1] = E * N;
    if (gather_order && gather_k < 1) return LQ_E_ARG;
    // one token (P == k pairs, its experts distinct, so every segment holds one pair): the gate/up projections of
    // the k experts run as one fragment-spread 4-bit decode launch over all SMs (qmvg's MoE mode)
    if (glu && gather_order && P == gather_k && bits == 4 &&
        qmvg_moe_ok(1, gather_k, N, K, device_info().sm_count)) {
        rc = qmvg_moe_run(1, xs, experts, nullptr, nullptr, w0, s0, b0, w1, s1, b1, out, gather_k, E, N, K, dtype,
                          reinterpret_cast<cudaStream_t>(stream));
        if (rc != LQ_E_SHAPE) return finish(rc);
    }
    // up to 16 rows a segment (decode batches): the grouped folded kernel, every SM walking (segment, fragment
    // chunk) items with one ring of weight stages running on across them
    if (P < 1024 && qmvqg_shape_ok(max_rows, N, K, bits)) {
        rc = qmvqg_run(xs, gather_order, gather_k, starts, experts, nseg, P, max_rows, glu, w0, s0, b0, w1, s1, b1,
                       out, E, N, K, bits, dtype, reinterpret_cast<cudaStream_t>(stream));
        if (rc != LQ_E_SHAPE) return finish(rc);
    }
    // from 1024 routed rows (about 16 per expert at 64 experts) the expert GEMMs run on the tensor-core
    // family, persistent when K allows (pre-gathered rows only); below that the mma.sync family's grouped
    // mode measured faster on B200
    // K the mma.sync family does not take (a 4-bit K that is a multiple of 128 but not of 256, e.g. an expert
    // intermediate of 384): the tensor-core family at any row count
    if (!gather_order && (P >= 1024 || !qmv_shape_ok(K, bits))) {
        const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        // persistent (one CTA per SM walks the expert tiles) for the gate/up pair and long rows; a single matrix
        // with short rows (the down projection, K = the expert intermediate) on the non-persistent tiles, measured
        // on B200 at config 4 with 2048 routed rows: gate/up 93.5 us persistent vs 105.9, down (K 768) 44.0 vs 51.2
        if (tcvp_shape_ok(P, K, bits) && (glu || K > 1024)) {
            rc = tcvp_run_grouped(xs, P, m, glu ? 2 : 1, N, K, out, starts, experts, nseg, E, bits, dtype, 0, st);
            if (rc != LQ_E_SHAPE) return finish(rc);
        }
        if (tcv_shape_ok(P, K, bits)) {
            rc = tcv_run_grouped(xs, P, m, glu ? 2 : 1, N, K, out, starts, experts, nseg, E, bits, dtype, nullptr, st);
            if (rc != LQ_E_SHAPE) return finish(rc);
        }
    }
    a.gather = gather_order;
    a.gather_k = gather_k;
    const int nseg_grid = (E + 1) < P ? (E + 1) : P;  // (one more for a padding bucket, expert id E)
    return finish(qmv_run(xs, gather_order ? 1 : P, m, glu ? 2 : 1, a, bits, dtype, nullptr, max_rows, nseg_grid,
                          reinterpret_cast<cudaStream_t>(stream)));
}

int lq_moe_down_combine(const void* h, const int32_t* experts, const int32_t* pos, const float* weights,
                        const uint32_t* w, const void* s, const void* b, void* y, int k, int E, int N, int K, int bits,
                        int group_size, int dtype, void* stream) {
    int rc = check_common(h, w, s, b, k, N, K, bits, group_size, dtype);
    if (rc) return rc;
    if (!experts || !weights || !y) return LQ_E_ARG;
    if (E < 1 || int64_t(E) * N > INT32_MAX) return LQ_E_SHAPE;
    if (bits != 4 || !qmvg_moe_ok(2, k, N, K, device_info().sm_count)) return LQ_E_SHAPE;
    if (!aligned(y, 2) || !aligned(weights, 4) || !aligned(experts, 4) || !aligned(pos, 4)) return LQ_E_ALIGN;
    return finish(qmvg_moe_run(2, h, experts, pos, weights, w, s, b, nullptr, nullptr, nullptr, y, k, E, N, K, dtype,
                               reinterpret_cast<cudaStream_t>(stream)));
}

size_t lq_moe_decode_workspace(int E, int k, int D, int I) {
    if (check_device() != LQ_OK) return 0;
    return moe_decode_workspace_bytes(E, k, D, I);
}

int lq_moe_decode(const void* x, const void* router_w, int router_dtype, int E, int k, int mode, const uint32_t* wg,
                  const void* sg, const void* bg, const uint32_t* wu, const void* su, const void* bu,
                  const uint32_t* wd, const void* sd, const void* bd, int D, int I, int bits, int group_size,
                  int dtype, void* y, uint32_t* inds, float* weights, void* workspace, size_t workspace_bytes,
                  void* stream) {
    int rc = check_common(x, wg, sg, bg, 1, I, D, bits, group_size, dtype);
    if (rc) return rc;
    rc = check_common(x, wu, su, bu, 1, I, D, bits, group_size, dtype);
    if (rc) return rc;
    rc = check_common(x, wd, sd, bd, 1, D, I, bits, group_size, dtype);
    if (rc) return rc;
    if (!router_w || !y || !workspace || (inds == nullptr) != (weights == nullptr)) return LQ_E_ARG;
    if (!is16(router_dtype)) return LQ_E_UNSUPPORTED;
    if (mode != 0 && mode != 1) return LQ_E_ARG;
    if (bits != 4 || !moe_decode_ok(E, k, D, I)) return LQ_E_SHAPE;
    if (!aligned(router_w, 16) || !aligned(y, 2) || !aligned(inds, 4) || !aligned(weights, 4) ||
        !aligned(workspace, 16) || !aligned(sg, 16) || !aligned(bg, 16) || !aligned(su, 16) || !aligned(bu, 16) ||
        !aligned(sd, 16) || !aligned(bd, 16))
        return LQ_E_ALIGN;
    const uint32_t* w[3] = {wg, wu, wd};
    const void* s[3] = {sg, su, sd};
    const void* b[3] = {bg, bu, bd};
    return finish(moe_decode_run(x, dtype, router_w, router_dtype, E, k, mode, w, s, b, D, I, y, inds, weights,
                                 workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream)));
}

size_t lq_peer_sync_bytes(void) { return peer_sync_bytes(); }

int lq_peer_scatter_rows(const void* src, const int32_t* idx, const int32_t* starts, const int32_t* experts,
                         const int32_t* nseg, int bucket, int rows_max, int row_bytes, int dst_rows, void* const* dst,
                         int G, int rank, void* const* sync, void* stream) {
    if (!src || !idx || !starts || !experts || !nseg || !dst || !sync) return LQ_E_ARG;
    int rc = check_device();
    if (rc) return rc;
    return finish(peer_scatter_rows_run(src, idx, starts, experts, nseg, bucket, rows_max, row_bytes, dst_rows, dst,
                                        G, rank, sync, reinterpret_cast<cudaStream_t>(stream)));
}

int lq_moe_group_range(const uint32_t* inds, int P, int lo, int range, int32_t* order, int32_t* starts,
                       int32_t* experts, int32_t* nseg, int32_t* pos, void* stream) {
    if (!inds || !order || !starts || !experts || !nseg) return LQ_E_ARG;
    if (P < 1 || lo < 0 || range < 1 || range > 8191) return LQ_E_SHAPE;
    int rc = check_device();
    if (rc) return rc;
    return finish(group_range_run(inds, P, lo, range, order, starts, experts, nseg, pos,
                                  reinterpret_cast<cudaStream_t>(stream)));
}

int lq_peer_gather_cols(const void* src, int M, int n, int col_off, int ldo, int elem_bytes, void* const* dst, int G,
                        int rank, void* const* sync, void* stream) {
    if (!src || !dst || !sync) return LQ_E_ARG;
    int rc = check_device();
    if (rc) return rc;
    return finish(peer_gather_run(src, M, n, col_off, ldo, elem_bytes, dst, G, rank, sync,
                                  reinterpret_cast<cudaStream_t>(stream)));
}

int lq_add_rms_norm(const void* x, const void* r, const void* w, void* h, void* n, int rows, int D, float eps,
                    int dtype, void* stream) {
    if (!x || !r || !w || !h || !n) return LQ_E_ARG;
    if (!is16(dtype)) return LQ_E_UNSUPPORTED;
    if (rows < 1 || !norm_shape_ok(D) || !(eps >= 0.0f)) return LQ_E_SHAPE;
    if (!aligned(x, 16) || !aligned(r, 16) || !aligned(w, 16) || !aligned(h, 16) || !aligned(n, 16)) return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    return finish(add_rms_run(x, r, w, h, n, rows, D, eps, dtype, reinterpret_cast<cudaStream_t>(stream)));
}

size_t lq_qmm_dense_workspace(int N, int K) {
    if (N < 1 || K < 1) return 0;
    return qmm_dense_workspace_bytes(N, K);
}

int lq_qmm_dense(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N, int K,
                 int bits, int group_size, int dtype, void* workspace, size_t workspace_bytes, const lq_cfg* cfg,
                 void* stream) {
    int rc = check_common(x, w, scales, biases, M, N, K, bits, group_size, dtype);
    if (rc) return rc;
    if (!y || !workspace) return LQ_E_ARG;
    if (!qmm_dense_shape_ok(M, N, K, bits)) return LQ_E_SHAPE;
    if (workspace_bytes < qmm_dense_workspace_bytes(N, K)) return LQ_E_ARG;
    if (!aligned(workspace, 16) || !aligned(y, 16) || (bits == 4 && (!aligned(scales, 2) || !aligned(biases, 2))))
        return LQ_E_ALIGN;
    rc = check_device();
    if (rc) return rc;
    return finish(qmm_dense_run(x, w, scales, biases, y, M, N, K, bits, dtype, workspace,
                                (cfg && cfg->family == LQ_FAM_TC) ? cfg->p : nullptr,
                                reinterpret_cast<cudaStream_t>(stream)));
}

int lq_qmm_dense_gather(const void* x, const uint32_t* w, const void* scales, const void* biases, void* const* dst,
                        int ndst, int col_off, int ldo, int M, int N, int K, int bits, int group_size, int dtype,
                        void* workspace, size_t workspace_bytes, const lq_cfg* cfg, void* stream) {
    int rc = check_common(x, w, scales, biases, M, N, K, bits, group_size, dtype);
    if (rc) return rc;
    if (!dst || !workspace || ndst < 1 || ndst > 8 || col_off < 0 || ldo < col_off + N) return LQ_E_ARG;
    if (ndst > 1 && (N % 8 || col_off % 8 || ldo % 8)) return LQ_E_ALIGN;  // 16-byte pieces for the peer copy
    for (int d = 0; d < ndst; ++d)
        if (!dst[d]) return LQ_E_ARG;
        else if (!aligned(dst[d], 16)) return LQ_E_ALIGN;
    if (!qmm_dense_shape_ok(M, N, K, bits)) return LQ_E_SHAPE;
    if (workspace_bytes < qmm_dense_workspace_bytes(N, K)) return LQ_E_ARG;
    if (!aligned(workspace, 16) || (bits == 4 && (!aligned(scales, 2) || !aligned(biases, 2)))) return LQ_E_ALIGN;
    rc = check_device();
    if (rc) return rc;
    return finish(qmm_dense_gather_run(x, w, scales, biases, dst, ndst, col_off, ldo, M, N, K, bits, dtype, workspace,
                                       (cfg && cfg->family == LQ_FAM_TC) ? cfg->p : nullptr,
                                       reinterpret_cast<cudaStream_t>(stream)));
}

int lq_ipc_export(const void* ptr, void* handle, size_t* offset) {
    if (!ptr || !handle || !offset) return LQ_E_ARG;
    const void* base = nullptr;
    int rc = alloc_base(ptr, &base);
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(base));
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return LQ_E_CUDA;
    }
    memcpy(handle, &h, sizeof(h));
    *offset = size_t(reinterpret_cast<const uint8_t*>(ptr) - reinterpret_cast<const uint8_t*>(base));
    return LQ_OK;
}

int lq_ipc_import(const void* handle, size_t offset, void** ptr) {
    if (!handle || !ptr) return LQ_E_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return LQ_E_CUDA;
    }
    *ptr = static_cast<uint8_t*>(base) + offset;
    return LQ_OK;
}

int lq_ipc_close(void* ptr, size_t offset) {
    if (!ptr) return LQ_E_ARG;
    const cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return LQ_E_CUDA;
    }
    return LQ_OK;
}

size_t lq_kv_attend_workspace(int B, int H, int KVH, int n) {
    if (B < 1 || H < 1 || KVH < 1 || n < 0) return 0;
    if (check_device() != LQ_OK) return 0;
    return kv_attend_workspace_bytes(B, H, KVH, n, device_info().sm_count);
}

int lq_kv_attend(const void* q, const uint32_t* kq, const void* ks, const void* kb, const uint32_t* vq, const void* vs,
                 const void* vb, const int32_t* start, int n, const float* sinks, float scale, int B, int H, int KVH,
                 int cap, int head_dim, int dtype, void* workspace, size_t workspace_bytes, void* out, void* stream) {
    if (!q || !kq || !ks || !kb || !vq || !vs || !vb || !out) return LQ_E_ARG;
    if (!is16(dtype)) return LQ_E_UNSUPPORTED;
    if (!kv_attend_shape_ok(B, H, KVH, n, cap, head_dim) || !(scale == scale)) return LQ_E_SHAPE;
    if (!aligned(q, 16) || !aligned(kq, 16) || !aligned(vq, 16) || !aligned(ks, 4) || !aligned(kb, 4) ||
        !aligned(vs, 4) || !aligned(vb, 4) || !aligned(out, 2) || !aligned(start, 4) || !aligned(sinks, 4) ||
        !aligned(workspace, 16))
        return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    return finish(kv_attend_run(q, kq, ks, kb, vq, vs, vb, start, n, sinks, scale, B, H, KVH, cap, dtype, workspace,
                                workspace_bytes, out, reinterpret_cast<cudaStream_t>(stream)));
}

int lq_moe_combine_norm(const void* ys, const float* weights, const int32_t* pos, const void* shared, const void* res,
                        const void* nw, void* y, void* n, int T, int k, int D, float eps, int dtype, void* stream) {
    if (!ys || !weights || !res || !nw || !y || !n) return LQ_E_ARG;
    if (!is16(dtype)) return LQ_E_UNSUPPORTED;
    if (T < 1 || k < 1 || !norm_shape_ok(D) || !(eps >= 0.0f)) return LQ_E_SHAPE;
    if (!aligned(ys, 16) || !aligned(res, 16) || !aligned(nw, 16) || !aligned(y, 16) || !aligned(n, 16) ||
        (shared && !aligned(shared, 16)))
        return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    return finish(combine_norm_run(ys, weights, pos, shared, res, nw, y, n, T, k, D, eps, dtype,
                                   reinterpret_cast<cudaStream_t>(stream)));
}

int lq_scatter_rows(const void* src, const int32_t* idx, int R, int N, void* dst, int dst_rows, int dtype,
                    void* stream) {
    if (!src || !idx || !dst) return LQ_E_ARG;
    if (!is16(dtype)) return LQ_E_UNSUPPORTED;
    if (R < 0 || N < 1 || dst_rows < 1 || (N * 2) % 16) return LQ_E_SHAPE;
    if (!aligned(src, 16) || !aligned(dst, 16)) return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    return finish(scatter_rows_run(src, idx, R, N * 2, dst, dst_rows, reinterpret_cast<cudaStream_t>(stream)));
}

int lq_supported(int family, int M, int N, int K, int bits, int group_size, int dtype) {
    if (!is16(dtype) || (bits != 4 && bits != 8) || group_size != 64) return 0;
    if (M < 1 || N < 1 || K < 64 || K % 64) return 0;
    const bool qmv = qmv_shape_ok(K, bits), tcv = tcv_shape_ok(M, K, bits), tc = tc_shape_ok(M, N, K, bits);
    const bool qmvg = qmvg_shape_ok(M, K, bits), qmvq = qmvq_shape_ok(M, K, bits);
    switch (family) {
        case LQ_FAM_AUTO: return (qmv || qmvg || qmvq || tcv || (M > 64 && tc)) ? 1 : 0;
        case LQ_FAM_QMVQ: return qmvq ? 1 : 0;
        case LQ_FAM_QMV: return qmv ? 1 : 0;
        case LQ_FAM_QMVG: return qmvg ? 1 : 0;
        case LQ_FAM_TCV: return tcv ? 1 : 0;
        case LQ_FAM_TC: return tc ? 1 : 0;
        default: return 0;
    }
}

int lq_list_configs(int M, int N, int K, int bits, int group_size, int dtype, lq_cfg* cfgs, int max_cfgs) {
    int n = 0;
    auto add = [&](int fam, int p0, int p1, int p2, int p3) {
        if (cfgs && n < max_cfgs) {
            lq_cfg c = {};
            c.family = fam;
            c.p[0] = p0;
            c.p[1] = p1;
            c.p[2] = p2;
            c.p[3] = p3;
            cfgs[n] = c;
        }
        ++n;
    };
    if (!lq_supported(LQ_FAM_AUTO, M, N, K, bits, group_size, dtype)) return 0;
    if (lq_supported(LQ_FAM_QMV, M, N, K, bits, group_size, dtype)) {
        add(LQ_FAM_QMV, 0, 0, 0, 0);
        if (M <= 64) {
            const int bk = 2048 / bits;
            const int nchunk = (K + bk - 1) / bk;
            const int mt = M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8;
            const int wks[3] = {1, 2, 4}, kss[6] = {1, 2, 3, 4, 5, 8};
            for (int wk : wks) {
                if (mt >= 4 && wk > 2) continue;
                for (int ks : kss)
                    if (ks <= nchunk) add(LQ_FAM_QMV, mt, wk, ks, 0);
            }
        }
    }
    if (lq_supported(LQ_FAM_QMVG, M, N, K, bits, group_size, dtype)) {
        add(LQ_FAM_QMVG, 0, 0, 0, 0);
        for (int fr = 1; fr <= 4; ++fr) add(LQ_FAM_QMVG, fr, 0, 0, 0);
    }
    if (lq_supported(LQ_FAM_QMVQ, M, N, K, bits, group_size, dtype)) {
        add(LQ_FAM_QMVQ, 0, 0, 0, 0);
        const int sxs = bits == 4 ? 2 : 1;  // (x sums by adds: 4-bit single matrices only)
        for (int sx = 1; sx <= sxs; ++sx)
            for (int fr = 0; fr <= 4; ++fr) add(LQ_FAM_QMVQ, fr, 0, 0, sx);
        const int kss[3] = {1, 2, 4};  // K slices over a cluster
        for (int ks : kss)
            if (ks <= (K + 511) / 512) add(LQ_FAM_QMVQ, 0, 0, ks, 0);
    }
    if (lq_supported(LQ_FAM_TCV, M, N, K, bits, group_size, dtype)) {
        add(LQ_FAM_TCV, 0, 0, 0, 0);
        const int kss[6] = {1, 2, 3, 4, 6, 8};
        for (int ks : kss)
            if (ks <= K / 128) add(LQ_FAM_TCV, 0, ks, 0, 0);
        if (M > 64) add(LQ_FAM_TCV, M > 128 ? 256 : 128, 1, 0, 0);
        if (tcvp_shape_ok(M, K, bits)) add(LQ_FAM_TCV, 0, 0, 0, 1);  // the persistent form
    }
    if (M > 64 && lq_supported(LQ_FAM_TC, M, N, K, bits, group_size, dtype)) {
        add(LQ_FAM_TC, 0, 0, 0, 0);
        const int bns[3] = {256, 224, 128};
        for (int bn : bns)
            if (N % bn == 0) add(LQ_FAM_TC, bn, 0, 0, 0);
    }
    return n;
}

int lq_moe_combine(const void* ys, const float* weights, const int32_t* pos, void* y, int T, int k, int D, int dtype,
                   void* stream) {
    if (!ys || !weights || !y) return LQ_E_ARG;
    if (!is16(dtype)) return LQ_E_UNSUPPORTED;
    if (T < 1 || k < 1 || D < 1) return LQ_E_SHAPE;
    int rc = check_device();
    if (rc) return rc;
    return finish(combine_run(ys, weights, pos, y, T, k, D, dtype, reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
