// Shared host and device helpers of libmq: argument checks with the thread-local error string,
// the device status word that bounded waits set, and the inline-PTX wrappers the kernels use.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/mq.h"

namespace mq {

// ---- host: errors ---------------------------------------------------------------------------

// Records the message of a failure for mq_last_error() and returns `code`.
int fail(int code, const char *fmt, ...);
// MQ_OK after a launch, or MQ_ECUDA with the CUDA error string.
int check_launch(const char *what);
// True when `p` is a multiple of `a` bytes.
inline bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
// The SM count and compute capability of the current device (cached per device).
struct DeviceInfo {
  int sms = 0, major = 0, minor = 0;
  size_t smem_optin = 0;
};
int device_info(DeviceInfo *out);

#define MQ_REQUIRE(cond, code, ...)           \
  do {                                        \
    if (!(cond)) return ::mq::fail(code, __VA_ARGS__); \
  } while (0)

// ---- device: status word ----------------------------------------------------------------------

// Set (first writer wins) by a kernel whose bounded wait ran out; read by mq_device_status().
// Defined here: libmq is one translation unit (csrc/libmq.cu), so this is its only definition.
__device__ int g_status = 0;

// Wait-site codes written into g_status.
enum : int { kStatusGemmTmaWait = 1, kStatusGemmMmaWait = 2, kStatusGemmDeqWait = 3, kStatusGemmEpiWait = 4 };

__device__ __forceinline__ void raise_status(int code) { atomicCAS(&g_status, 0, code); }

// ---- device: PTX wrappers ---------------------------------------------------------------------

// D += A * B on the legacy warp-level tensor path: m16n8k16, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 128-bit streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ldg_stream_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

}  // namespace mq
