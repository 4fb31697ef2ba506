// Shared host and device helpers of libmq: argument checks with the thread-local error string,
// the device status word that bounded waits set, and the inline-PTX wrappers the kernels use.
#pragma once

#include <cuda.h>
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
// Encodes a 2-D tiled map over a row-major [rows][cols] array of `elem_bytes` elements.
int encode_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                   uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                   CUtensorMapSwizzle swizzle, const char *what);

#define MQ_REQUIRE(cond, code, ...)           \
  do {                                        \
    if (!(cond)) return ::mq::fail(code, __VA_ARGS__); \
  } while (0)

// ---- device: status word ----------------------------------------------------------------------

// Set (first writer wins) by a kernel whose bounded wait ran out; read by mq_device_status().
// Defined here: libmq is one translation unit (csrc/libmq.cu), so this is its only definition.
__device__ int g_status = 0;

// Wait-site codes written into g_status.
enum : int {
  kStatusGemmTmaWait = 1,
  kStatusGemmMmaWait = 2,
  kStatusGemmDeqWait = 3,
  kStatusGemmEpiWait = 4,
  kStatusGemvProducerWait = 5,
  kStatusGemvConsumerWait = 6,
  kStatusGemvDrainWait = 7,
};

__device__ __forceinline__ void raise_status(int code) { atomicCAS(&g_status, 0, code); }

// ---- device: PTX wrappers ---------------------------------------------------------------------

// Bounded waits give up after this many nanoseconds (kernels here wait microseconds at most).
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `bar` with the given parity to complete; false if kWaitTimeoutNs passed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitTimeoutNs) return false;
  }
}

// 2-D tiled TMA load of box (x, y) of `map` into shared memory, completing on `bar`.
// x (the innermost coordinate) times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Named barrier over `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

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
