// Device-side status word shared by every kernel of the library. Kernels never trap: a bounded
// wait that gives up, or a check that fails, ORs a code in here and the kernel returns; the host
// reads and clears it with lq_device_status().
#pragma once

#include <stdint.h>

#define LQ_DEV_TIMEOUT 0x1u   // an mbarrier / flag wait ran out of polls
#define LQ_DEV_BOUNDS 0x2u    // an index check failed (expert id, token id out of range)
#define LQ_DEV_TMEM 0x4u      // tensor-memory allocation did not return the expected columns

namespace lq {
// Defined here: liblq.so is one translation unit (liblq.cu), so this header is included once.
__device__ unsigned int g_status = 0;

__device__ __forceinline__ void record_status(unsigned int code) { atomicOr(&g_status, code); }
}  // namespace lq
