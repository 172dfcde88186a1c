/*
 * lq — C ABI of the B200-native (sm_100a) MLX affine group-quantized matmul path.
 *
 * Plain pointers and sizes only. Every pointer is device memory on the current CUDA device
 * unless stated; `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream).
 * Nothing here allocates device memory: outputs are caller-allocated, as MLX allocates them for
 * the reference's kernels. Every entry point returns LQ_OK or an LQ_E_* code and never aborts.
 *
 * Weight format (MLX affine, the format every reference kernel consumes; locals/kernels.py:12-13,
 * locals/qmv_multi.py:23-29, locals/moe.py:181-204): w (N, K*bits/32) uint32, code i of word j is
 * K index (32/bits)*j + i at bits bits*i (low bits first); scales and biases (N, K/group) in the
 * activation dtype; dequantized weight = scale * q + bias.
 */
#ifndef LQ_H_
#define LQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LQ_OK 0
#define LQ_E_ARG 1          /* null pointer, bad enum value */
#define LQ_E_SHAPE 2        /* shape outside what the kernels accept */
#define LQ_E_ALIGN 3        /* pointer or row stride not aligned as the kernels need */
#define LQ_E_UNSUPPORTED 4  /* bits / group size / dtype combination not built */
#define LQ_E_CUDA 5         /* a CUDA runtime call failed (see lq_last_cuda_error) */
#define LQ_E_DEVICE 6       /* the current device is not an sm_100 GPU */
#define LQ_E_SCRATCH 7      /* the shape needs more scratch than lq_kv_attend_noalloc's fixed buffer holds */

#define LQ_F16 0
#define LQ_BF16 1
#define LQ_F32 2

/* Kernel families, the analogue of the reference's tuning choices (locals/kernels.py:136-144). */
#define LQ_FAM_AUTO 0   /* pick by shape: TC from 65 rows; TCV for 33-64 rows or >= 24 MB of weights from 9 rows;
                           QMVQ for 1-8 rows of a 4-bit matrix with K <= 4096 (K % 256 == 0) and 9-16 rows with
                           K <= 2560, N <= 8192; else QMV */
#define LQ_FAM_QMV 1    /* decode: TMA-staged packed weights, register dequant, mma.sync; p = {MT, WK, KS, NS} */
#define LQ_FAM_TC 2     /* prefill: dequant tiles into shared memory, tcgen05.mma into TMEM */
#define LQ_FAM_TCV 3    /* tcgen05 with weights dequantized into TMEM (A operand), tokens as N;
                           p = {NTOK, KS, WS, PERSISTENT (1: one CTA per SM walks the tiles)} */
#define LQ_FAM_QMVQ 5   /* as QMVG, with the codes fed raw to the MMA (128 + q / 1024 + q) and each group's scale and
                           bias folded in fp32 (y += s acc + (b - magic s) sum x), the weights never rounded to the
                           activation dtype: the reference's fragq formulation; p = {FR, NS} */
#define LQ_FAM_QMVG 4   /* dense 4-bit decode, M <= 16, K % 256 == 0: each warp takes one 64-wide group of every
                           stage for all of its CTA's 16-row fragments, fragments spread over every SM;
                           p = {FR (max fragments a CTA, <= 4), NS} */

typedef struct lq_cfg {
    int family;  /* LQ_FAM_* */
    int p[7];    /* family parameters, 0 = choose */
} lq_cfg;

/* y (M, N) = x (M, K) . dequant(w)^T, fp32 accumulation, y in the activation dtype.
 * Replaces the reference's quantized-linear launcher contract `_launcher(choice, M, K, N, dtype)
 * -> f(x, w, scales, biases) -> y` (locals/kernels.py:516-576) and `mx.quantized_matmul(x, w,
 * scales, biases, transpose=True, group_size=64, bits)` (locals/kernels.py:574,1004,1192).
 * dtype: LQ_F16 / LQ_BF16 for x, scales, biases and y. bits 4 or 8, group_size 64. */
int lq_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N, int K,
           int bits, int group_size, int dtype, const lq_cfg* cfg, void* stream);

/* Large-M quantized matmul the way the reference's dense prefill path computes it (locals/kernels.py:999-1025,
 * `_dense_matmul`: mx.dequantize into a temporary, then x @ w.T; chosen there for N x K <= 2^27 weights,
 * kernels.py:858-866): the weights are dequantized once into `workspace` (N x K in dtype, rounded once to dtype as
 * mx.dequantize rounds them) and y (M, N) = x . w^T runs as a dense tcgen05 GEMM (fp32 accumulation).
 * workspace_bytes >= lq_qmm_dense_workspace(N, K); workspace and y 16-byte aligned; K % 64 == 0; bits 4 or 8.
 * cfg: NULL, or family LQ_FAM_TC with p[0] = the N tile (128, 224 or 256; 0 = choose). */
int lq_qmm_dense(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N, int K,
                 int bits, int group_size, int dtype, void* workspace, size_t workspace_bytes, const lq_cfg* cfg,
                 void* stream);

/* Bytes of workspace lq_qmm_dense needs: N * K * 2. Host-only. */
size_t lq_qmm_dense_workspace(int N, int K);

/* Fused projection with its output split along N (the fused q/k/v projection): columns
 * [0, widths[0]) of x . dequant(w)^T go to outs[0] (M, widths[0]), the next widths[1] to outs[1],
 * ... (nout <= 3, sum of widths = N). Replaces fuse._concat_quantized + FusedAttention's reshape
 * and split (locals/fuse.py:28-63). */
int lq_qmm_split(const void* x, const uint32_t* w, const void* scales, const void* biases, int nout, void* const* outs,
                 const int* widths, int M, int N, int K, int bits, int group_size, int dtype, const lq_cfg* cfg,
                 void* stream);

/* h (M, I) = swiglu(x . gate^T, x . up^T) with the rounding points of locals/moe.py:284-289 (each
 * projection rounded to the activation dtype, then sigmoid, g*sig, act*u each rounded). gate and
 * up are (I, K) quantized matrices; for a concatenated gate||up (locals/fuse.py:160-199) pass the
 * same arrays offset by I rows. Replaces FusedMLP's gate_up_proj + swiglu (locals/fuse.py:161-164). */
int lq_qmm_glu(const void* x, const uint32_t* w_gate, const void* s_gate, const void* b_gate, const uint32_t* w_up,
               const void* s_up, const void* b_up, void* h, int M, int I, int K, int bits, int group_size, int dtype,
               const lq_cfg* cfg, void* stream);

/* MLX affine quantization (mx.quantize(w, group_size, bits), as called in the reference's tests,
 * e.g. tests/test_kernel_patching.py:163): w (N, K) in w_dtype (LQ_F32/LQ_F16/LQ_BF16) ->
 * wq (N, K*bits/32) uint32, scales and biases (N, K/group_size) in sb_dtype. */
int lq_quantize(const void* w, int w_dtype, int N, int K, int bits, int group_size, uint32_t* wq, void* scales,
                void* biases, int sb_dtype, void* stream);

/* mx.dequantize (locals/kernels.py:1007,1024): w_out (N, K) in dtype = scale * q + bias rounded
 * to dtype (scales/biases in dtype). */
int lq_dequantize(const uint32_t* wq, const void* scales, const void* biases, int N, int K, int bits, int group_size,
                  int dtype, void* w_out, void* stream);

/* Router logits in float32: logits (T, E) = float(x) (T, D) . float(w)^T (E, D); x and w may be
 * f16/bf16 of different dtypes. Replaces moe.router / router_logits (locals/moe.py:118-139). */
int lq_router_logits(const void* x, int x_dtype, const void* w, int w_dtype, float* logits, int T, int E, int D,
                     void* stream);

/* Top-k routing of float32 logits (T, E): mode 0 = softmax over E then the k largest, mode 1 =
 * sigmoid (NaN -> 0) then the k largest (locals/moe.py:36-82,145-165); ties go to the lower expert
 * index; weights renormalised to sum 1. inds (T, k) uint32 in descending score order, weights
 * (T, k) float32. E <= 1024, k <= 32. */
int lq_route_topk(const float* logits, int T, int E, int k, int mode, uint32_t* inds, float* weights, void* stream);

/* Router logits and top-k in one kernel, one CTA per token (lq_router_logits then lq_route_topk without
 * the logits round trip): inds (T, k) uint32, weights (T, k) float32; logits (T, E) float32 is written
 * too when not NULL. E <= 1024, k <= 32. */
int lq_moe_route(const void* x, int x_dtype, const void* w, int w_dtype, int T, int E, int D, int k, int mode,
                 uint32_t* inds, float* weights, float* logits, void* stream);

/* Counting sort of P expert ids (locals/moe_kernel.py:28-66,191-197): order (P) = pair ids grouped
 * by ascending expert (ascending pair id within an expert), starts (min(E,P)+1), experts (min(E,P)),
 * nseg (1) and, if pos != NULL, pos (P) = the inverse of order. All int32 device arrays. E <= 8192. */
int lq_moe_group(const uint32_t* inds, int P, int E, int32_t* order, int32_t* starts, int32_t* experts, int32_t* nseg,
                 int32_t* pos, void* stream);

/* The same counting sort over only the pairs routed to experts [lo, lo + range) (one rank's experts in an
 * expert-parallel layer; no counterpart in the reference, which runs on one GPU): they are grouped under local ids
 * 0 .. range - 1 in the stable order of lq_moe_group, every other pair under the padding bucket `range`, which sorts
 * last and which lq_moe_experts skips (pass E = range there). starts (min(range + 1, P) + 1), experts and order as
 * lq_moe_group; range <= 8191. */
int lq_moe_group_range(const uint32_t* inds, int P, int lo, int range, int32_t* order, int32_t* starts,
                       int32_t* experts, int32_t* nseg, int32_t* pos, void* stream);

/* xs (P, D) = x[order[j] / k] for j < P: the tokens of the pairs in expert order (16-bit x, D % 8 == 0). */
int lq_moe_gather(const void* x, const int32_t* order, int P, int k, int D, void* xs, void* stream);

/* Grouped expert projections (locals/moe_kernel.py:68-155,206-239; mx.gather_qmm of mlx-lm's SwitchGLU,
 * locals/moe_kernel.py:279): segment s of lq_moe_group covers rows [starts[s], starts[s+1]) of the
 * pair-ordered xs (P, K) and uses expert experts[s]; each used expert's weights are read once for all
 * its rows (a segment longer than 64 rows streams them once per 64).
 * glu != 0: out (P, N) = swiglu(xs . gate_e^T, xs . up_e^T) (rounding of locals/moe.py:284-289);
 *           gate = (w0, s0, b0), up = (w1, s1, b1), each stacked (E, N, K*bits/32) / (E, N, K/group).
 * glu == 0: out (P, N) = xs . w0_e^T.
 * max_rows bounds the rows of one segment (the token count of the step: a token names an expert at
 * most once). out in dtype, rows in pair order. Rows grouped under expert id E (group with E + 1
 * buckets) are padding: they are skipped and their output rows left unwritten.
 * gather_order != NULL: xs is the token matrix (T, K) and segment row j reads token gather_order[j] /
 * gather_k (the order of lq_moe_group), fetched inside the kernel -- no lq_moe_gather pass. */
int lq_moe_experts(const void* xs, const int32_t* starts, const int32_t* experts, const int32_t* nseg, int P,
                   int max_rows, int glu, const uint32_t* w0, const void* s0, const void* b0, const uint32_t* w1,
                   const void* s1, const void* b1, void* out, int E, int N, int K, int bits, int group_size, int dtype,
                   const int32_t* gather_order, int gather_k, void* stream);

/* The down projection and the weighted combine of ONE token's k slots in one launch (decode; 4-bit, k <= 4):
 * y (1, N) = sum over slots r of weights[r] * round(h[pos[r]] . down_e^T), e = experts[pos[r]], the products rounded
 * to dtype and summed in float32 in slot order, then rounded -- lq_moe_experts (glu = 0) followed by lq_moe_combine
 * without the (k, N) round trip. Replaces the reference's experts_down and its combine kernel for one token
 * (locals/moe.py:465-512, 339-348). h (k, K) holds the token's k pairs in the grouping's order, one pair a segment (the order of
 * lq_moe_group, or the pairs' own order with experts = the token's k expert ids and pos = NULL); w, s, b are the
 * stacked (E, N, ...) down experts. K % 256 == 0, N % 16 == 0. LQ_E_SHAPE for shapes outside this (use the two
 * calls then). */
int lq_moe_down_combine(const void* h, const int32_t* experts, const int32_t* pos, const float* weights,
                        const uint32_t* w, const void* s, const void* b, void* y, int k, int E, int N, int K, int bits,
                        int group_size, int dtype, void* stream);

/* ONE token's whole routed MoE layer in one launch (decode at batch 1): the router logits and top-k of lq_moe_route
 * (bit-identical experts and weights), each slot's gate/up SwiGLU, its down projection and the weighted combine of
 * lq_moe_down_combine, y (1, D) in dtype. Replaces, for one token, the chain router -> route_topk -> experts_up ->
 * experts_down of the reference's FusedFlintMoe.__call__ (locals/moe.py:577-591) without its shared expert.
 * x (1, D) dtype; router_w (E, D) f16/bf16; gate/up (E, I, D/8) packed 4-bit, down (E, D, I/8), scales and biases
 * (E, rows, K/64) in dtype, group size 64, every pointer 16-byte aligned. inds (k) and weights (k) receive the routing when not NULL. workspace:
 * lq_moe_decode_workspace(E, k, D, I) bytes, 16-byte aligned, zero-filled before its first use (the kernel leaves
 * its counters at zero); one workspace serves launches in stream order, not concurrent launches. D % 128 == 0,
 * I % 64 == 0, k <= 32, E <= 1024; LQ_E_SHAPE outside this (use the unfused calls then). */
size_t lq_moe_decode_workspace(int E, int k, int D, int I);
int lq_moe_decode(const void* x, const void* router_w, int router_dtype, int E, int k, int mode, const uint32_t* wg,
                  const void* sg, const void* bg, const uint32_t* wu, const void* su, const void* bu,
                  const uint32_t* wd, const void* sd, const void* bd, int D, int I, int bits, int group_size,
                  int dtype, void* y, uint32_t* inds, float* weights, void* workspace, size_t workspace_bytes,
                  void* stream);

/* y (T, D) = sum over slots r of weights[t, r] * ys[pos[t*k + r], :] in float32, slots in order, rounded
 * to dtype (locals/moe.py:339-348). pos == NULL reads row t*k + r. */
int lq_moe_combine(const void* ys, const float* weights, const int32_t* pos, void* y, int T, int k, int D, int dtype,
                   void* stream);

/* h = x + r (rounded to dtype) and n = w * rms_norm(h) in one pass over rows of D values, the sum of squares
 * in fp32: n = T(w * T(h * 1/sqrt(mean(h^2) + eps))). Replaces norm_kernel.add_rms (locals/norm_kernel.py:73-85),
 * the residual add and input norm between a decoder layer's projections. D % 8 == 0, D <= 8192; x, r, w, h,
 * n 16-byte aligned. */
int lq_add_rms_norm(const void* x, const void* r, const void* w, void* h, void* n, int rows, int D, float eps,
                    int dtype, void* stream);

/* The MoE combine with the shared expert, the layer's residual add and the next layer's input norm in one
 * pass (locals/moe.py:353-389): y[t] = T(res[t] + T(T(sum_r weights[t,r] * ys[pos[t*k + r]]) + shared[t])),
 * n[t] = T(nw * T(y[t] / sqrt(mean(y[t]^2) + eps))). shared == NULL: no shared expert; pos == NULL: row
 * t*k + r. Same shape rules as lq_add_rms_norm. */
int lq_moe_combine_norm(const void* ys, const float* weights, const int32_t* pos, const void* shared, const void* res,
                        const void* nw, void* y, void* n, int T, int k, int D, float eps, int dtype, void* stream);

/* Row packing's scatter (locals/kernels.py:840-851): dst (dst_rows, N) is zeroed, then dst row idx[j] = src row j
 * for j < R. The gather half is lq_moe_gather(x, idx, R, 1, N, xs). N * 2 % 16 == 0. */
int lq_scatter_rows(const void* src, const int32_t* idx, int R, int N, void* dst, int dst_rows, int dtype,
                    void* stream);

/* Decode attention over an 8-bit key/value cache, replacing qkv.attend (locals/qkv.py:213-249): for every row b
 * and query head h, softmax over the keys at positions max(start[b], 0) .. n-1 and the head's sink logit
 * (sinks[h], natural-log units; NULL = none) of scale * q.k, times the values; out = T(sum p v / sum p).
 * q (B, H, head_dim) and out (B, H, head_dim) in dtype; the cache is read in place in the reference's layout:
 * kq, vq uint32 (B, KVH, cap, head_dim/4) (MLX affine 8-bit, four codes a word, low byte first), ks, kb, vs, vb
 * (B, KVH, cap, head_dim/64) in dtype. start may be NULL (every row from 0). head_dim == 128, H % KVH == 0,
 * H / KVH <= 16, 0 <= n <= cap. workspace: lq_kv_attend_workspace(B, H, KVH, n) bytes (16-byte aligned; NULL
 * when that is 0). */
int lq_kv_attend(const void* q, const uint32_t* kq, const void* ks, const void* kb, const uint32_t* vq, const void* vs,
                 const void* vb, const int32_t* start, int n, const float* sinks, float scale, int B, int H, int KVH,
                 int cap, int head_dim, int dtype, void* workspace, size_t workspace_bytes, void* out, void* stream);

/* Bytes of workspace lq_kv_attend needs for this shape on the current device (0: none). */
size_t lq_kv_attend_workspace(int B, int H, int KVH, int n);

/* lq_kv_attend without a workspace argument, for callers that cannot allocate device memory when they attend (a
 * plugin given only raw device pointers, code inside a CUDA graph someone else built, a runtime whose memory pool is
 * fixed at start-up). It has no counterpart in the reference, whose MLX kernels have outputs allocated for them.
 * The per-block softmax parts go to a 4 MiB buffer inside the library (a __device__ array that every GPU loading
 * the library holds until the process exits); nothing is allocated or freed. Shapes whose parts need more than
 * 4 MiB (lq_kv_attend_workspace(B, H, KVH, n) > 4194304) return LQ_E_SCRATCH before any launch. The first call on a
 * device looks up the buffer's device address (cudaGetSymbolAddress) and should come before any stream capture; the
 * address is kept for the life of the process, so do not call this again on a device after cudaDeviceReset on it.
 * All calls share the buffer: calls that overlap on the GPU (unordered streams) race and may return wrong
 * results. Other arguments, results and errors as lq_kv_attend. */
int lq_kv_attend_noalloc(const void* q, const uint32_t* kq, const void* ks, const void* kb, const uint32_t* vq,
                         const void* vs, const void* vb, const int32_t* start, int n, const float* sinks, float scale,
                         int B, int H, int KVH, int cap, int head_dim, int dtype, void* out, void* stream);

/* The column-sharded prefill with its own all-gather: this rank's N output columns of y = x . dequant(w)^T (the
 * dense path of lq_qmm_dense) are written by the GEMM in place at columns [col_off, col_off + N) of dst[0], this GPU's
 * row-major (M, ldo) buffer, then copied by one kernel of plain 16-byte peer stores into the same columns of
 * dst[1 .. ndst) (ndst <= 8; peers' buffers, pointers from lq_ipc_import) -- no staging buffer, no strided copy, no
 * NCCL all-gather. N, col_off and ldo are multiples of 8 when ndst > 1. The caller orders completion across ranks (a
 * collective after the call) before any rank reads its buffer. No counterpart in the reference, which runs on one
 * GPU; it replaces the all-gather that follows a column-sharded kernels._dense_matmul (locals/kernels.py:1020-1025). */
int lq_qmm_dense_gather(const void* x, const uint32_t* w, const void* scales, const void* biases, void* const* dst,
                        int ndst, int col_off, int ldo, int M, int N, int K, int bits, int group_size, int dtype,
                        void* workspace, size_t workspace_bytes, const lq_cfg* cfg, void* stream);

/* CUDA IPC for peer buffers between the processes of one node (no counterpart in the reference): export writes the
 * 64-byte handle of the allocation that holds ptr and ptr's offset in it; import maps a peer's allocation into this
 * process for the current device (peer access enabled on first use) and returns the address of the peer's ptr;
 * close unmaps it. */
int lq_ipc_export(const void* ptr, void* handle, size_t* offset);
int lq_ipc_import(const void* handle, size_t offset, void** ptr);
int lq_ipc_close(void* ptr, size_t offset);

/* The exchange between column shards at decode sizes without NCCL (no counterpart in the reference, which runs on one
 * GPU; it replaces the all-gather after a column-sharded projection): copies this rank's row-major (M, n) block src
 * into columns [col_off, col_off + n) of every rank's (M, ldo) buffer dst[0 .. G) (dst[rank] this GPU's own, the
 * others peers' buffers from lq_ipc_import), then meets the other ranks on flags: when the launch ends, dst[rank]
 * holds every rank's columns. sync[p] is rank p's sync block (lq_peer_sync_bytes() bytes, zero-filled before first
 * use, exported and imported like the buffers; sync[rank] this rank's own). Ranks on distinct GPUs (G <= 8), the
 * same calls in the same order on every rank, and buffers reused no sooner than every second call (a peer may be one
 * call ahead). elem_bytes 2 or 4; n, col_off and ldo in 16-byte multiples. A peer that does not arrive within one
 * second leaves LQ_DEV_TIMEOUT in the device status. */
size_t lq_peer_sync_bytes(void);
int lq_peer_gather_cols(const void* src, int M, int n, int col_off, int ldo, int elem_bytes, void* const* dst, int G,
                        int rank, void* const* sync, void* stream);

/* The combine-side exchange of an expert-parallel MoE layer over peer memory (no counterpart in the reference): row
 * j of src (R, row_bytes) -- the rows this rank's grouped expert kernels wrote, those before the padding bucket of
 * a lq_moe_group_range grouping (starts, experts, nseg, bucket = range; read on the device) -- goes to row idx[j]
 * (the grouping's order: its pair index) of every rank's (dst_rows, row_bytes) buffer dst[0 .. G); then the ranks meet
 * on the sync blocks as in lq_peer_gather_cols. rows_max bounds the rows sent (sizes the launch); row_bytes a
 * multiple of 16. */
int lq_peer_scatter_rows(const void* src, const int32_t* idx, const int32_t* starts, const int32_t* experts,
                         const int32_t* nseg, int bucket, int rows_max, int row_bytes, int dst_rows, void* const* dst,
                         int G, int rank, void* const* sync, void* stream);

/* 1 if kernel family `family` (LQ_FAM_*; LQ_FAM_AUTO = any) accepts this shape and format, else 0. Host-only,
 * needs no GPU. Replaces the per-family supported(M, K, N, cfg) predicates the reference's tuner filters
 * its candidates with (locals/qmv_frag.py:162,519; locals/nax_kernel.py:399-408; locals/kernels.py:654-674). */
int lq_supported(int family, int M, int N, int K, int bits, int group_size, int dtype);

/* The tuning candidates for one shape (the reference's candidate list, locals/kernels.py:654-674): writes
 * up to max_cfgs entries (family + parameters, 0 = the library's choice) into cfgs and returns how many
 * exist (cfgs may be NULL to count). Host-only, needs no GPU. */
int lq_list_configs(int M, int N, int K, int bits, int group_size, int dtype, lq_cfg* cfgs, int max_cfgs);

/* Read (and with clear != 0 reset) the device status word kernels OR their LQ_DEV_* codes into
 * (1 = a bounded wait gave up, 2 = an index check failed, 4 = a TMEM allocation failed). Synchronizes
 * the current device. Returns the word, or 0xffffffff if the read itself failed. */
unsigned int lq_device_status(int clear);

/* The last CUDA error string seen by the library (static storage). */
const char* lq_last_cuda_error(void);

/* Human-readable name of an LQ_* code. */
const char* lq_strerror(int code);

/* ABI version (major * 100 + minor). */
int lq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LQ_H_ */
