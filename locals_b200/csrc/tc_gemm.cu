// Prefill-size quantized GEMM on the 5th-generation tensor cores (tcgen05). Placeholder until the
// kernel lands: shapes are rejected so callers fall back to the qmv family.
#include <cuda_runtime.h>
#include <stdint.h>

#include "lq_host.h"

namespace lq {
bool tc_shape_ok(int, int, int, int) { return false; }
int tc_run(const void*, const uint32_t*, const void*, const void*, void*, int, int, int, int, int, const int*,
           cudaStream_t) {
    return LQ_E_UNSUPPORTED;
}
}  // namespace lq
