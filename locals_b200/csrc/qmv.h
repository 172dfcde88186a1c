// Launch interface of the qmv (decode / grouped-expert) kernel family.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace lq {

struct QmvArgs {
    int M, N, K;      // M: rows of a dense call (tokens); N: output columns per matrix (per expert)
    int nchunk;       // ceil(K / 512), set by the launcher
    int ks;           // split-K factor (cluster size along y), set by the launcher
    int ns;           // pipeline stages, set by the launcher
    int sb_vec;       // cp.async width for scale/bias rows, set by the launcher
    int row_off[2];   // row offset of each matrix inside its arrays (gate||up concatenation)
    int rows_total[2];
    const void* sptr[2];
    const void* bptr[2];
    void* out[3];     // output column segments (q/k/v split), or out[0] only
    int seg_end[3];
    int ldo[3];
    int nseg_out;
    int grouped;      // 1: blockIdx.z indexes expert segments (starts / experts / nseg)
    const int32_t* starts;
    const int32_t* experts;
    const int32_t* nseg;
    int n_experts;
    const void* x;          // x base (gather mode reads rows through it)
    const int32_t* gather;  // grouped mode: segment row j reads x row gather[j] / gather_k (null: row j)
    int gather_k;
};

struct QmvMats {
    const uint32_t* w[2];
    const void* s[2];
    const void* b[2];
    int row_off[2];
    int rows_total[2];  // rows of the arrays behind each matrix (tensor-map and cp.async bounds)
};

// K accepted by the kernel: 4-bit K % 256 == 0, 8-bit K % 128 == 0 (group size 64).
bool qmv_shape_ok(int K, int bits);

// p = {MT, R, KS, NS} (0 = choose). x has x_rows rows of K values. max_seg_rows bounds the rows of
// one segment (M for a dense call; the tokens of the call for a grouped one). n_seg_grid: grid z
// (1 dense; min(E, P) grouped).
int qmv_run(const void* x, int x_rows, const QmvMats& mats, int nmat, QmvArgs a, int bits, int dtype, const int* p,
            int max_seg_rows, int n_seg_grid, cudaStream_t st);

}  // namespace lq
