// libmq.so is one translation unit: the kernels share the device status word (g_status) without
// relocatable device code, and each file keeps its helpers in its own namespace.
#include <algorithm>

#include "capi.cu"
#include "unpack.cu"
#include "gemv_q4.cu"
#include "tgemv.cu"
#include "gemm_q4.cu"
#include "moe.cu"
#include "pack.cu"
#include "io.cu"
#include "ep.cu"
