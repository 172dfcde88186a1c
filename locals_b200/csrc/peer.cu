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
    __syncthreads();  // every store of this CTA before thread 0's release (cumulative) and count
    if (threadIdx.x != 0) return;
    uint32_t* own = reinterpret_cast<uint32_t*>(sync.p[rank]);
    // device-scope release / acquire on the counter, then the last CTA's system-scope release of each flag: the
    // chain orders every CTA's peer stores before the flag for the peer that acquires it
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

}  // namespace lq
