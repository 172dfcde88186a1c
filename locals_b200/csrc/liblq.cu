// Unity translation unit of liblq.so: every kernel family and the C ABI compile together so the
// device status word (lq::g_status) is one symbol without relocatable device code.
#include "lq_host.cu"
#include "quant.cu"
#include "qmv.cu"
#include "qmvg.cu"
#include "tcv.cu"
#include "tcvp.cu"
#include "moe.cu"
#include "tc_gemm.cu"
#include "norm.cu"
#include "kv_attend.cu"
#include "capi.cu"
#include "kv_attend_noalloc.cu"
