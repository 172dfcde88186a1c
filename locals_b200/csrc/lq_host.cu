// Host helpers: tensor-map encoding through the driver entry point, device properties, status word.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "lq_host.h"
#include "lq_status.cuh"

namespace lq {

static char g_last_cuda_error[256] = "";

void note_cuda_error(cudaError_t e) {
    if (e != cudaSuccess) snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s", cudaGetErrorString(e));
}

const char* last_cuda_error() { return g_last_cuda_error; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddrRangeFn addr_range_fn() {
    static AddrRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddrRangeFn>(p);
    });
    return fn;
}

int alloc_base(const void* ptr, const void** base) {
    AddrRangeFn fn = addr_range_fn();
    if (!fn) return LQ_E_CUDA;
    CUdeviceptr b = 0;
    size_t size = 0;
    if (fn(&b, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return LQ_E_ARG;
    *base = reinterpret_cast<const void*>(b);
    return LQ_OK;
}

int make_tmap(CUtensorMap* out, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
    if (reinterpret_cast<uintptr_t>(base) % 16) return LQ_E_ALIGN;
    for (int i = 0; i < rank - 1; ++i)
        if (strides_bytes[i] % 16) return LQ_E_ALIGN;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return LQ_E_CUDA;
    cuuint64_t d[5];
    cuuint64_t s[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
    }
    for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
    CUresult r = fn(out, dt, cuuint32_t(rank), const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuTensorMapEncodeTiled failed (%d)", int(r));
        return LQ_E_CUDA;
    }
    return LQ_OK;
}

const DeviceInfo& device_info() {
    static DeviceInfo cache[16];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) {
        static DeviceInfo none;
        return none;
    }
    DeviceInfo& di = cache[dev];
    if (di.device != dev) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, dev) == cudaSuccess) {
            di.sm_count = p.multiProcessorCount;
            di.major = p.major;
            di.minor = p.minor;
            di.smem_optin = p.sharedMemPerBlockOptin;
            di.smem_per_sm = p.sharedMemPerMultiprocessor;
            di.device = dev;
        }
    }
    return di;
}

int check_device() {
    const DeviceInfo& di = device_info();
    if (di.device < 0) return LQ_E_CUDA;
    return di.major == 10 ? LQ_OK : LQ_E_DEVICE;
}

static std::mutex& status_mutex() {
    static std::mutex m;
    return m;
}

static StatusReader* status_readers(int** count) {
    static StatusReader readers[64];
    static int n = 0;
    *count = &n;
    return readers;
}

void register_status_reader(StatusReader r) {
    std::lock_guard<std::mutex> lock(status_mutex());
    int* n = nullptr;
    StatusReader* readers = status_readers(&n);
    if (*n < 64) readers[(*n)++] = r;
}

unsigned int read_status(bool clear) {
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
    std::lock_guard<std::mutex> lock(status_mutex());
    int* n = nullptr;
    StatusReader* readers = status_readers(&n);
    unsigned int v = 0;
    for (int i = 0; i < *n; ++i) {
        const unsigned int w = readers[i](clear);
        if (w == 0xffffffffu) return w;
        v |= w;
    }
    return v;
}

}  // namespace lq
