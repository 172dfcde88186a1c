// Column all-gather among the GPUs of one node for decode-size payloads, over peer memory and without NCCL: the
// exchange between the column shards of a sharded projection (each rank computes N/G output columns of an (M, N)
// result, and every rank needs all N). At decode sizes the payload is a few KB and a collective library call costs
// far more than the bytes (a 4-byte NCCL all-reduce measured 22 us on this pool's B200 pairs); here one kernel moves
// the bytes with plain peer stores and the ranks meet on flags in each other's memory.
//
// peer_gather_kernel: every thread copies 16-byte pieces of this rank's (M, n) block into columns
// [col_off, col_off + n) of every rank's (M, ldo) buffer (its own and the peers', mapped through CUDA IPC), consecutive
// threads along a row so each warp store is one contiguous run. The last CTA to finish (a counter in this rank's sync
// block, counted with device-scope acquire/release) takes the next round number, stores it into its slot of every
// peer's flag array (a release at system scope: with the counter's chain it orders every CTA's stores before the
// flag), and waits until every peer's slot of its own array holds that round (an
// acquire at system scope, bounded by one second of %globaltimer: on expiry it records LQ_DEV_TIMEOUT and returns).
// When the kernel ends, this rank's buffer holds every rank's columns. No TMA and no multicast: plain loads and stores.
//
// The ranks must sit on distinct GPUs (the waits of two ranks sharing one GPU would not be guaranteed to run at the same
// time), call the gathers in the same order, and keep at least two buffers in turn (a peer can be one round ahead).
#include <cuda_runtime.h>
#include <stdint.h>

#include "lq_host.h"
#include "lq_ptx.cuh"
#include "lq_status.cuh"

namespace lq {

constexpr int PEER_MAX = 8;           // ranks
constexpr int PEER_ROUND_OFF = 16;    // uint32 offsets in a sync block: flags [0, PEER_MAX), the round, the counter
constexpr int PEER_DONE_OFF = 32;
constexpr size_t PEER_SYNC_BYTES = 256;
constexpr unsigned long long PEER_WAIT_NS = 1000000000ull;  // one second

struct PeerPtrs {
    void* p[PEER_MAX];
};

__device__ __forceinline__ unsigned long long peer_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void peer_st_release(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t peer_ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// After a CTA's stores: its thread 0 counts the CTA in (device-scope acquire/release on this rank's counter); the last
// CTA takes the next round, releases it into its slot of every peer's flag array (system scope: with the counter's
// chain it orders every CTA's stores before the flag for the peer that acquires it) and waits -- bounded by one second
// of %globaltimer, then LQ_DEV_TIMEOUT -- until every peer's slot of its own array holds that round.
__device__ __forceinline__ void peer_meet(const PeerPtrs& sync, int G, int rank) {
    __syncthreads();  // every store of this CTA before thread 0's release (cumulative) and count
    if (threadIdx.x != 0) return;
    uint32_t* own = reinterpret_cast<uint32_t*>(sync.p[rank]);
    uint32_t prev;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(own + PEER_DONE_OFF) : "memory");
    if (prev != gridDim.x - 1) return;
    const uint32_t r = own[PEER_ROUND_OFF] + 1u;
    own[PEER_ROUND_OFF] = r;
    own[PEER_DONE_OFF] = 0u;
    for (int p = 0; p < G; ++p)
        if (p != rank) peer_st_release(reinterpret_cast<uint32_t*>(sync.p[p]) + rank, r);
    const unsigned long long t0 = peer_now();
    for (int p = 0; p < G; ++p) {
        if (p == rank) continue;
        while (int32_t(peer_ld_acquire(own + p) - r) < 0) {
            if (peer_now() - t0 > PEER_WAIT_NS) {
                record_status(LQ_DEV_TIMEOUT);
                return;
            }
            __nanosleep(64);
        }
    }
}

__global__ void __launch_bounds__(256) peer_gather_kernel(const uint4* __restrict__ src, const PeerPtrs dst,
                                                          const PeerPtrs sync, int G, int rank, int M, int pieces_row,
                                                          int ld_pieces, int off_pieces) {
    grid_dep_wait();  // src is the previous kernel's output
    // the next kernel may launch now and stream its own weights during the exchange: it waits for this grid's end
    // (griddepcontrol.wait) before it reads the gathered buffer
    grid_dep_launch();
    const int64_t total = int64_t(M) * pieces_row;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t m = i / pieces_row, c = i - m * pieces_row;
        const uint4 v = src[i];
        const int64_t off = m * ld_pieces + off_pieces + c;
#pragma unroll
        for (int d = 0; d < PEER_MAX; ++d)
            if (d < G) reinterpret_cast<uint4*>(dst.p[d])[off] = v;
    }
    peer_meet(sync, G, rank);
}

// Rows of an expert-parallel layer's local results to every rank: src row j (j < the number of pairs this rank
// computed: the rows before the grouping's padding bucket) goes to row idx[j] (its pair index) of every rank's buffer.
// One thread a 16-byte piece of a row.
__global__ void __launch_bounds__(256) peer_scatter_rows_kernel(const uint4* __restrict__ src,
                                                                const int32_t* __restrict__ idx,
                                                                const int32_t* __restrict__ starts,
                                                                const int32_t* __restrict__ experts,
                                                                const int32_t* __restrict__ nseg, int bucket,
                                                                int dst_rows, const PeerPtrs dst, const PeerPtrs sync,
                                                                int G, int rank, int pieces_row) {
    grid_dep_wait();  // src, idx and the grouping come from the previous kernels
    grid_dep_launch();
    const int ns = *nseg;
    const int rows = (ns > 0 && experts[ns - 1] == bucket) ? starts[ns - 1] : starts[ns];
    const int64_t total = int64_t(rows) * pieces_row;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t j = i / pieces_row, c = i - j * pieces_row;
        const int r = idx[j];
        if (r < 0 || r >= dst_rows) {
            record_status(LQ_DEV_BOUNDS);
            continue;
        }
        const uint4 v = src[i];
        const int64_t off = int64_t(r) * pieces_row + c;
#pragma unroll
        for (int d = 0; d < PEER_MAX; ++d)
            if (d < G) reinterpret_cast<uint4*>(dst.p[d])[off] = v;
    }
    peer_meet(sync, G, rank);
}

size_t peer_sync_bytes() { return PEER_SYNC_BYTES; }

int peer_gather_run(const void* src, int M, int n, int col_off, int ldo, int elem_bytes, void* const* dst, int G,
                    int rank, void* const* sync, cudaStream_t st) {
    if (G < 1 || G > PEER_MAX || rank < 0 || rank >= G || M < 1 || n < 1 || col_off < 0 || ldo < col_off + n)
        return LQ_E_ARG;
    if (elem_bytes != 2 && elem_bytes != 4) return LQ_E_ARG;
    if ((int64_t(n) * elem_bytes) % 16 || (int64_t(col_off) * elem_bytes) % 16 || (int64_t(ldo) * elem_bytes) % 16 ||
        reinterpret_cast<uintptr_t>(src) % 16)
        return LQ_E_ALIGN;
    PeerPtrs d = {}, s = {};
    for (int p = 0; p < G; ++p) {
        if (!dst[p] || !sync[p] || reinterpret_cast<uintptr_t>(dst[p]) % 16 || reinterpret_cast<uintptr_t>(sync[p]) % 16)
            return LQ_E_ARG;
        d.p[p] = dst[p];
        s.p[p] = sync[p];
    }
    const int pieces_row = int(int64_t(n) * elem_bytes / 16);
    const int64_t total = int64_t(M) * pieces_row;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = int64_t(device_info().sm_count) * 4;
    if (blocks > cap) blocks = cap;
    const uint4* sp = reinterpret_cast<const uint4*>(src);
    const int ldp = int(int64_t(ldo) * elem_bytes / 16), offp = int(int64_t(col_off) * elem_bytes / 16);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(blocks), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, peer_gather_kernel, sp, d, s, G, rank, M, pieces_row, ldp, offp));
}

int peer_scatter_rows_run(const void* src, const int32_t* idx, const int32_t* starts, const int32_t* experts,
                          const int32_t* nseg, int bucket, int rows_max, int row_bytes, int dst_rows,
                          void* const* dst, int G, int rank, void* const* sync, cudaStream_t st) {
    if (G < 1 || G > PEER_MAX || rank < 0 || rank >= G || rows_max < 1 || row_bytes < 16 || dst_rows < 1)
        return LQ_E_ARG;
    if (row_bytes % 16 || reinterpret_cast<uintptr_t>(src) % 16) return LQ_E_ALIGN;
    PeerPtrs d = {}, s = {};
    for (int p = 0; p < G; ++p) {
        if (!dst[p] || !sync[p] || reinterpret_cast<uintptr_t>(dst[p]) % 16 || reinterpret_cast<uintptr_t>(sync[p]) % 16)
            return LQ_E_ARG;
        d.p[p] = dst[p];
        s.p[p] = sync[p];
    }
    const int pieces_row = row_bytes / 16;
    int64_t blocks = (int64_t(rows_max) * pieces_row + 255) / 256;  // (the rows sent are known on the device only)
    const int64_t cap = int64_t(device_info().sm_count) * 4;
    if (blocks > cap) blocks = cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(blocks), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, peer_scatter_rows_kernel, reinterpret_cast<const uint4*>(src), idx,
                                          starts, experts, nseg, bucket, dst_rows, d, s, G, rank, pieces_row));
}

}  // namespace lq
