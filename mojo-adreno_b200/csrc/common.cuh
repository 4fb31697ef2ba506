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

// Launches `kern` so that it may start while the previous kernel on `stream` is still finishing
// (programmatic dependent launch). Such a kernel runs only set-up that touches no global memory
// (barriers, TMEM, descriptor prefetch) before griddep_wait(); after it, every write of earlier
// work on the stream is visible, exactly as with an ordinary launch.
template <typename... KArgs, typename... Args>
int launch_overlapped(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char *what,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return fail(MQ_ECUDA, "%s: launch: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

namespace gemv {
// The expert-indirect GEMV of the MoE decode (gemv_q4.cu); gate_up fuses the SwiGLU of gate|up rows;
// x is fp32, or fp16 with x_f16.
// gate (may be null): a device count; when *gate > gate_max the launch does nothing.
int gemv_q4_grouped(const uint32_t *wq, const uint16_t *ws, int64_t wrows, const void *x, float *y,
                    const int32_t *ids, int ngroups, int group_rows, int rows_per_group, int64_t k, int group, int xpg,
                    cudaStream_t stream, int gate_up, int x_f16, const int32_t *gate = nullptr, int gate_max = 0);
}  // namespace gemv

// The grouped expert GEMM (gemm_q4.cu): mode 1 gate|up + SiLU (fp16 out), mode 2 plain (fp32 out).
// perm: xs rows (and mode 1's output rows) in the k order 0, 4, 1, 5, 2, 6, 3, 7 within each 8.
int moe_gemm_run(int mode, const uint32_t *wq, const uint16_t *ws, const uint16_t *xs, int64_t pairs, int64_t k,
                 int experts, int64_t rows_per_expert, int group, const int32_t *tiles, const int32_t *ntiles,
                 int max_tiles, int tile_m, void *out, cudaStream_t stream, int perm);

// The tcgen05 GEMM (gemm_q4.cu), shared by mq_gemm_q4 and the batched path of mq_gemv_q4.
int gemm_q4_run(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y, int64_t n, int64_t k,
                int64_t m, int group, int add, void *workspace, size_t workspace_bytes, cudaStream_t stream);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
// Encodes a 2-D tiled map over a row-major [rows][cols] array of `elem_bytes` elements.
int encode_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                   uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                   CUtensorMapSwizzle swizzle, const char *what);
// A 3-D map: `planes` copies of a [rows][cols] matrix, plane_stride_bytes apart (two row blocks of
// one matrix, fetched by one box).
int encode_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                   uint64_t rows, uint64_t planes, uint64_t row_stride_bytes, uint64_t plane_stride_bytes,
                   uint32_t box_cols, uint32_t box_rows, uint32_t box_planes, CUtensorMapSwizzle swizzle,
                   const char *what);

// Raises kern's dynamic shared-memory limit to at least `smem` on the current device, once per
// device: the attribute belongs to the device's context, so a process that drives several GPUs sets
// it on each. `seen` is the kernel's own table of the limits already set, by device.
template <typename Kern>
int ensure_smem(Kern kern, size_t smem, size_t (&seen)[64], const char *what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return fail(MQ_ECUDA, "%s: cudaGetDevice failed", what);
  if (smem > seen[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(MQ_ECUDA, "%s: cudaFuncSetAttribute: %s", what, cudaGetErrorString(e));
    seen[dev] = smem;
  }
  return MQ_OK;
}

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
  kStatusMoeBadExpertId = 8,  // an expert id >= experts: the pair was left out (negative ids mean "none")
  kStatusEpOverflow = 9,      // more pairs for one rank than the plan's capacity: the excess was left out
  kStatusEpDispatchWait = 10,  // an expert-parallel rank's rows did not arrive in time (the layer went on without them)
  kStatusEpReturnWait = 11,    // an owner's expert outputs did not come back in time
};

// Waits until the kernels this grid depends on (earlier work on its stream) have completed and
// their writes are visible; a no-op for an ordinary launch.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel on the stream begin launching (its own griddep_wait still orders its accesses).
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void raise_status(int code) { atomicCAS(&g_status, 0, code); }


// ---- device: waiting for expert-parallel peers ------------------------------------------------

// A wait for the flags of an expert-parallel exchange (ep.cu): flags[which * world + s] >= *epoch for
// every rank s. Kernels that start a step of the exchange take one (flags null: no wait) and wait in
// every CTA before touching the data the flags announce.
struct FlagWait {
  const int *flags = nullptr;
  int which = 0, world = 0;
  const int *epoch = nullptr;
};

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

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

// Threads 0 .. world - 1 of the CTA wait (bounded: 2 s, then status 10 or 11 and go on) for their
// rank's flag, then the CTA synchronises; the acquire loads make the peers' writes visible.
__device__ __forceinline__ void wait_flags(const FlagWait &w) {
  if (!w.flags) return;
  const int e = *w.epoch;
  for (int s = threadIdx.x; s < w.world; s += blockDim.x) {
    const int *f = w.flags + w.which * w.world + s;
    if (ld_acquire_sys(f) >= e) continue;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) < e) {
      if (globaltimer() - t0 > 2000000000ull) {
        raise_status(w.which == 0 ? kStatusEpDispatchWait : kStatusEpReturnWait);
        break;
      }
      __nanosleep(200);
    }
  }
  __syncthreads();
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

// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `bar` with the given parity to complete; false if kWaitTimeoutNs passed.
// try_wait suspends the thread in hardware between polls, so waiting warps leave issue slots to
// the warps that compute.
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

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 2-D tiled TMA store (or, with add, an fp32 reduce-add) of the box at (x, y) from shared memory,
// in the calling thread's bulk group; x times the element size must be a multiple of 16 bytes and
// both coordinates non-negative. Elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y, bool add) {
  if (add)
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
  else
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
// Closes the calling thread's bulk group and waits until its copies are complete (written).
__device__ __forceinline__ void bulk_commit_and_wait() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Warms L2 with `bytes` (a multiple of 16) of global memory from a 16-byte aligned address.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes) : "memory");
}

// Warms L2 with a box of a tensor map (no shared memory, no barrier). Safe before griddep_wait:
// it binds no data, and later loads read whatever the memory then holds.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap *map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 (5th-generation tensor core) and TMEM ---------------------------------------------

// Shared-memory matrix descriptor for a K-major tile in the canonical 128-byte-swizzle layout:
// rows of 128 bytes (64 fp16 along K), 8-row atoms 1024 bytes apart (SBO), LBO unused (1),
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B. `addr` must be 1024-aligned;
// advancing along K by 16 elements adds 32 bytes to the start address.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16: fp32 accumulator, fp16 A and B, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T with A (128 x 16 fp16, K-major) in tensor memory: row m in
// lane m, its 16 K values as fp16 pairs in the 8 columns from a_tmem (lower K in the low half).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 consecutive 32-bit columns of TMEM lane (warp quarter * 32 + lane) from registers; warp-collective.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 consecutive 32-bit columns of TMEM lane (warp quarter * 32 + lane) from registers; warp-collective.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Waits until this thread's earlier tcgen05.st have completed.
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of TMEM lane (warp quarter * 32 + lane) into registers.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads
// (TMA stores, tcgen05.mma operand fetches).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Named barrier over `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// D += A * B on the legacy warp-level tensor path: m16n8k16, fp16 inputs, fp32 accumulators.
// D (16x8 s32) += A (16x32 s8, row) * B (32x8 s8, col): each A/B register holds 4 consecutive k.
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

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
