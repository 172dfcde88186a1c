// Host-side helpers shared by the launchers: status codes, tensor-map encoding through the driver
// entry point (no link-time libcuda dependency, so the library loads on machines without a GPU),
// and cached device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lq.h"

namespace lq {

// Encode a tiled tensor map. dims/strides are innermost-first; strides has rank-1 entries (bytes).
// Returns LQ_OK or LQ_E_ALIGN / LQ_E_CUDA.
int make_tmap(CUtensorMap* out, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// The start of the device allocation that holds ptr (LQ_E_ARG if ptr is not device memory of this process).
int alloc_base(const void* ptr, const void** base);

struct DeviceInfo {
    int device = -1;
    int sm_count = 0;
    int major = 0, minor = 0;
    size_t smem_optin = 0;
    size_t smem_per_sm = 0;
};

// Properties of the current device (cached per device).
const DeviceInfo& device_info();

// LQ_OK if the current device is sm_100 (B200 class), else LQ_E_DEVICE.
int check_device();

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? LQ_OK : LQ_E_CUDA; }

// The last CUDA error the library saw (for lq_last_cuda_error) and the device status words.
void note_cuda_error(cudaError_t e);
const char* last_cuda_error();
unsigned int read_status(bool clear);

// Argument-check helpers of the C ABI's entry points.
inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline bool is16(int dt) { return dt == LQ_F16 || dt == LQ_BF16; }
inline int finish(int rc) {
    if (rc == LQ_E_CUDA) note_cuda_error(cudaGetLastError());
    return rc;
}

}  // namespace lq
