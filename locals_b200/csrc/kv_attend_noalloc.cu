// lq_kv_attend_noalloc: the 8-bit KV decode attention of kv_attend.cu for callers that cannot allocate device
// memory. lq_kv_attend needs a caller-allocated workspace for its per-block softmax parts whenever the keys of a
// (row, kv head) are split over several CTAs. Some callers have no allocator at hand at that point: code that runs
// inside a captured or replayed CUDA graph built by someone else, a plugin handed only raw device pointers by its
// host, a runtime whose memory pool is fixed at start-up. For them this entry point keeps the parts in a buffer the
// library owns: a file-scope __device__ array, created when the module is loaded, held by every GPU that loads the
// library until the process exits, and never freed or grown.
//
// The array is KVA_STATIC_SCRATCH_BYTES (4 MiB). A shape whose parts need more (more than 4 MiB of
// B * H * nsplit * 130 floats; on a 148-SM B200 only shapes with several hundred (row, kv head) pairs and 16 query
// heads a kv head reach it) is rejected with LQ_E_SCRATCH before anything is launched.
//
// In host code `kva_static_scratch` names a host-side shadow, not device memory: handing it to a kernel would fault
// or, where the GPU can reach host memory, silently use the wrong memory. The device address is therefore looked up
// with cudaGetSymbolAddress once per device, with that device current, on the first call made on it, and cached.
// That first call on a device should come before any stream capture. The cache lives as long as the process: a
// caller that destroys its context on a device (cudaDeviceReset) and then calls this entry point again on that
// device would be handed the old, stale address, so such callers must not use this entry point after a reset.
//
// Every call shares the one array, and nothing in it survives a call in a useful way: each launch writes every part
// it later reads, so nothing needs clearing first. Calls whose kernels overlap on the GPU (different streams, or
// different host threads' streams without ordering between them) race on the array and may return wrong results;
// order them on one stream or use lq_kv_attend with separate workspaces.

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/lq.h"
#include "lq_host.h"

namespace lq {
bool kv_attend_shape_ok(int B, int H, int KVH, int n, int cap, int head_dim);
size_t kv_attend_workspace_bytes(int B, int H, int KVH, int n, int sms);
int kv_attend_run(const void* q, const uint32_t* kq, const void* ks, const void* kb, const uint32_t* vq,
                  const void* vs, const void* vb, const int32_t* start, int n, const float* sinks, float scale, int B,
                  int H, int KVH, int cap, int dtype, void* workspace, size_t workspace_bytes, void* out,
                  cudaStream_t st);

constexpr size_t KVA_STATIC_SCRATCH_BYTES = size_t(4) << 20;
static __device__ __align__(256) uint8_t kva_static_scratch[KVA_STATIC_SCRATCH_BYTES];

// Device address of kva_static_scratch on the current device (looked up on the first use per device).
static int kva_static_scratch_address(void** out) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    int dev = -1;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return LQ_E_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) return LQ_E_DEVICE;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t g = cudaGetSymbolAddress(&p, kva_static_scratch);
        if (g != cudaSuccess || !p) {
            note_cuda_error(g);
            return LQ_E_CUDA;
        }
        addr[dev] = p;
    }
    *out = addr[dev];
    return LQ_OK;
}

}  // namespace lq

using namespace lq;

extern "C" int lq_kv_attend_noalloc(const void* q, const uint32_t* kq, const void* ks, const void* kb, const uint32_t* vq,
                         const void* vs, const void* vb, const int32_t* start, int n, const float* sinks, float scale,
                         int B, int H, int KVH, int cap, int head_dim, int dtype, void* out, void* stream) {
    if (!q || !kq || !ks || !kb || !vq || !vs || !vb || !out) return LQ_E_ARG;
    if (!is16(dtype)) return LQ_E_UNSUPPORTED;
    if (!kv_attend_shape_ok(B, H, KVH, n, cap, head_dim) || !(scale == scale)) return LQ_E_SHAPE;
    if (!aligned(q, 16) || !aligned(kq, 16) || !aligned(vq, 16) || !aligned(ks, 4) || !aligned(kb, 4) ||
        !aligned(vs, 4) || !aligned(vb, 4) || !aligned(out, 2) || !aligned(start, 4) || !aligned(sinks, 4))
        return LQ_E_ALIGN;
    int rc = check_device();
    if (rc) return rc;
    const size_t need = kv_attend_workspace_bytes(B, H, KVH, n, device_info().sm_count);
    if (need > KVA_STATIC_SCRATCH_BYTES) return LQ_E_SCRATCH;
    void* scratch = nullptr;
    if (need) {
        rc = kva_static_scratch_address(&scratch);
        if (rc) return rc;
    }
    return finish(kv_attend_run(q, kq, ks, kb, vq, vs, vb, start, n, sinks, scale, B, H, KVH, cap, dtype, scratch,
                                need ? KVA_STATIC_SCRATCH_BYTES : 0, out, reinterpret_cast<cudaStream_t>(stream)));
}
