// Device-side status word of the library's kernels. Kernels never trap: a bounded wait that gives up, or a check
// that fails, ORs a code into the status word and the kernel returns; the host reads and clears it with
// lq_device_status().
//
// The library is built as separate translation units without relocatable device code, so each translation unit that
// includes this header gets its own word (internal linkage) and registers a host-side reader for it when the library
// is loaded; lq_device_status() ORs the words of every translation unit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define LQ_DEV_TIMEOUT 0x1u   // an mbarrier / flag wait ran out of polls
#define LQ_DEV_BOUNDS 0x2u    // an index check failed (expert id, token id out of range)
#define LQ_DEV_TMEM 0x4u      // tensor-memory allocation did not return the expected columns

namespace lq {

// Host side: readers of the translation units' status words (defined in lq_host.cu).
typedef unsigned int (*StatusReader)(bool clear);
void register_status_reader(StatusReader r);

namespace {
__device__ unsigned int g_status = 0;

// This translation unit's word on the current device: 0xffffffff if the copy failed.
unsigned int read_tu_status(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (clear) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(g_status, &z, sizeof(z)) != cudaSuccess) return 0xffffffffu;
    }
    return v;
}

struct StatusRegistration {
    StatusRegistration() { register_status_reader(&read_tu_status); }
};
StatusRegistration g_status_registration;
}  // namespace

__device__ __forceinline__ void record_status(unsigned int code) { atomicOr(&g_status, code); }

}  // namespace lq
