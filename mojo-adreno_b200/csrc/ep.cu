// Expert-parallel exchange over NVLink peer memory (one process per GPU).
//
// The reference runs every expert on one device (qwen3moe/model.mojo:256-267); here rank r owns the
// experts [r E / world, (r + 1) E / world) and the tokens' rows travel to their experts' owners and
// back. Instead of NCCL all-to-alls with host-known split sizes, the exchange is four kernels on the
// stream, so a layer needs no host read and can be captured in a CUDA graph:
//  * mq_ep_dispatch advances the layer's epoch (a device counter; every rank runs the same layers,
//    so the epochs agree) and rank r writes its pairs' fp16 rows and owner-local expert ids straight into
//    each owner's receive buffer (plain stores through CUDA IPC mappings of the peers' memory), at
//    the fixed slots [r * cap, r * cap + cap), ids -1 past its pairs. The CTA that finishes last
//    raises rank r's dispatch flag on every owner to the epoch (one system-scope fence, then strong
//    stores, after every CTA's stores were fenced).
//  * mq_ep_expert_step waits until every rank's rows arrived (acquire loads in the first kernel, a
//    bounded wait: on time-out it records a status and lets the layer go on), runs the owner's experts
//    on the received rows (ids -1 skipped) and writes each output row straight back into its sender's
//    return buffer at the slot the row came from, then raises its return flag there.
//  * mq_ep_combine waits for every owner's return flag and sums each token's returned rows.
// Only rows of real pairs move over NVLink. One receive buffer per rank suffices: a sender's next
// dispatch follows its wait for this layer's returns, and an owner raises its return flag only after
// its last read of the receive buffer (the return kernel itself), so layer L + 1's rows never
// overwrite rows of layer L still in use; likewise for the returned rows.
#include <cstring>

#include "common.cuh"

namespace mq {
namespace ep {


// A strong (relaxed, system-scope) store; after a system-scope fence it is a release.
__device__ __forceinline__ void st_relaxed_sys(int *p, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The CTA that arrives last at `done` (after every CTA fenced its stores at system scope) raises
// flag slot `which * world + rank` on every peer to the epoch, re-arms `done` for the next layer and,
// when `epoch` is given, stores the new epoch (every CTA read the old one before its arrival).
// The CTA barrier orders the CTA's writes before its thread 0, whose GPU-scope fence and arrival
// pass them on to the last CTA to arrive (the grid-barrier pattern: fences are cumulative); that
// CTA's one system-scope fence, followed by plain strong stores of the flags (a fence then a strong
// store is a release), then publishes every CTA's writes to the peers: one fence however many peers
// (a store-release per peer would fence once per peer). A system-scope fence in every thread
// serialised thousands of them (15 us for a handful of rows).
__device__ void signal_peers(int *const *peer_flags, int which, int world, int rank, int e, int *done,
                             int *epoch = nullptr) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1) {
      *done = 0;
      if (epoch) *epoch = e;
      __threadfence_system();
      for (int d = 0; d < world; ++d) st_relaxed_sys(peer_flags[d] + which * world + rank, e);
    }
  }
}

// Work item it: (slot, 16-byte chunk); slot = d * cap + i is send position i for owner d.
__global__ void dispatch_kernel(const void *__restrict__ x, int x_f16, const int32_t *__restrict__ order,
                                const int32_t *__restrict__ local_ids, int topk, int dm, int world, int rank, int cap,
                                uint16_t *const *peer_rows, int32_t *const *peer_ids, int *const *peer_flags,
                                int *epoch, int *done) {
  griddep_launch_dependents();
  griddep_wait();            // programmatic dependent launch: earlier work on the stream is complete
  const int e = *epoch + 1;  // this layer's epoch: the last CTA stores it for the later steps
  const int vec = dm / 8, slots = world * cap;
  const size_t base_row = static_cast<size_t>(rank) * cap;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < static_cast<int64_t>(slots) * vec;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int slot = static_cast<int>(it / vec), c = static_cast<int>(it % vec) * 8;
    const int o = order[slot];
    if (o < 0) continue;  // an empty slot: its id (-1) tells the owner
    const int d = slot / cap, i = slot % cap, t = o / topk;
    uint4 v;
    if (x_f16) {
      v = *reinterpret_cast<const uint4 *>(static_cast<const __half *>(x) + static_cast<size_t>(t) * dm + c);
    } else {
      const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(x) + static_cast<size_t>(t) * dm + c);
      const float4 a = src[0], b = src[1];
      v = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y), pack_half2(b.z, b.w));
    }
    *reinterpret_cast<uint4 *>(peer_rows[d] + (base_row + i) * dm + c) = v;
  }
  for (int slot = blockIdx.x * blockDim.x + threadIdx.x; slot < slots; slot += gridDim.x * blockDim.x) {
    const int d = slot / cap, i = slot % cap;
    peer_ids[d][base_row + i] = order[slot] < 0 ? -1 : local_ids[slot];
  }
  signal_peers(peer_flags, 0, world, rank, e, done, epoch);
}

// Waits for flag slot `which * world + s` of every rank s to reach the epoch.
__global__ void wait_kernel(const int *flags, int which, int world, const int *epoch) {
  griddep_launch_dependents();
  griddep_wait();
  FlagWait w;
  w.flags = flags;
  w.which = which;
  w.world = world;
  w.epoch = epoch;
  wait_flags(w);
}

// Output rows back to their senders: row slot = s * cap + i of the receive buffer (ids[slot] >= 0)
// goes to sender s's return buffer at row rank * cap + i. z_row(slot) is its row of the expert
// outputs: slot_of[slot] (the grouped products' sorted order), or slot itself when slot_of is null.
__global__ void return_kernel(const float *__restrict__ z, const int32_t *__restrict__ slot_of,
                              const int32_t *__restrict__ ids, int dm, int world, int rank, int cap,
                              float *const *peer_ret, int *const *peer_flags, const int *epoch, int *done) {
  griddep_launch_dependents();
  griddep_wait();
  const int e = *epoch;
  const int vec = dm / 4, slots = world * cap;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < static_cast<int64_t>(slots) * vec;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int slot = static_cast<int>(it / vec), c = static_cast<int>(it % vec) * 4;
    if (ids[slot] < 0) continue;
    const int zr = slot_of ? slot_of[slot] : slot;
    if (zr < 0) continue;
    const int s = slot / cap, i = slot % cap;
    const float4 v = *reinterpret_cast<const float4 *>(z + static_cast<size_t>(zr) * dm + c);
    *reinterpret_cast<float4 *>(peer_ret[s] + (static_cast<size_t>(rank) * cap + i) * dm + c) = v;
  }
  signal_peers(peer_flags, 1, world, rank, e, done);
}

// CTAs for `work` 16-byte items, a few per thread: every CTA of an exchange kernel fences and counts
// itself in before the flags go up, so fewer CTAs shorten that chain (the loops stride over the rest).
inline int grid_for(int64_t work, const DeviceInfo &dev) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(dev.sms) * 4)));
}

}  // namespace ep
}  // namespace mq

namespace {
typedef CUresult (*AddrRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);
AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  }
  return fn;
}
}  // namespace

extern "C" int mq_ipc_handle(const void *ptr, void *handle, int64_t *offset) {
  MQ_REQUIRE(ptr && handle && offset, MQ_EINVAL, "mq_ipc_handle: null pointer");
  AddrRangeFn fn = addr_range_fn();
  MQ_REQUIRE(fn, MQ_ECUDA, "mq_ipc_handle: cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  MQ_REQUIRE(fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) == CUDA_SUCCESS, MQ_ECUDA,
             "mq_ipc_handle: the pointer is not device memory of this process");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  MQ_REQUIRE(e == cudaSuccess, MQ_ECUDA, "mq_ipc_handle: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  std::memcpy(handle, &h, sizeof h);
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MQ_OK;
}

extern "C" int mq_ipc_open(const void *handle, int64_t offset, void **ptr) {
  MQ_REQUIRE(handle && ptr && offset >= 0, MQ_EINVAL, "mq_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void *base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  MQ_REQUIRE(e == cudaSuccess, MQ_ECUDA, "mq_ipc_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr = static_cast<uint8_t *>(base) + offset;
  return MQ_OK;
}

extern "C" int mq_ipc_close(void *ptr, int64_t offset) {
  MQ_REQUIRE(ptr && offset >= 0, MQ_EINVAL, "mq_ipc_close: bad arguments");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t *>(ptr) - offset);
  MQ_REQUIRE(e == cudaSuccess, MQ_ECUDA, "mq_ipc_close: cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return MQ_OK;
}

extern "C" int mq_ep_dispatch(const void *x, int x_dtype, const int32_t *order, const int32_t *local_ids, int64_t tokens,
                              int topk, int64_t d, int world, int rank, int cap, uint16_t *const *peer_rows,
                              int32_t *const *peer_ids, int *const *peer_flags, int *epoch, int *done,
                              void *stream) {
  MQ_REQUIRE(order && local_ids && peer_rows && peer_ids && peer_flags && epoch && done, MQ_EINVAL,
             "mq_ep_dispatch: null pointer");
  MQ_REQUIRE(tokens == 0 || x, MQ_EINVAL, "mq_ep_dispatch: null x");
  MQ_REQUIRE(world >= 1 && world <= 256 && rank >= 0 && rank < world && cap >= 1 && topk >= 1, MQ_EINVAL,
             "mq_ep_dispatch: bad world / rank / capacity");
  MQ_REQUIRE(d > 0 && d % 8 == 0 && static_cast<int64_t>(world) * cap * d < (1LL << 40), MQ_EINVAL,
             "mq_ep_dispatch: d must be a multiple of 8");
  MQ_REQUIRE(x_dtype == MQ_F32 || x_dtype == MQ_F16, MQ_EINVAL, "mq_ep_dispatch: x_dtype must be MQ_F32 or MQ_F16");
  MQ_REQUIRE(!x || mq::aligned(x, 16), MQ_EALIGN, "mq_ep_dispatch: x must be 16-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  const int xh = x_dtype == MQ_F16;
  // At most tokens * topk slots hold a row: size the grid for those (the loop strides over all slots).
  const int64_t busy = std::min<int64_t>(static_cast<int64_t>(world) * cap, std::max<int64_t>(1, tokens * topk));
  return mq::launch_overlapped(mq::ep::dispatch_kernel, dim3(mq::ep::grid_for(busy * (d / 8) / 4, dev)),
                               dim3(256), 0, static_cast<cudaStream_t>(stream), "mq_ep_dispatch", x, xh, order, local_ids,
                               topk, static_cast<int>(d), world, rank, cap, peer_rows, peer_ids, peer_flags, epoch, done);
}

extern "C" int mq_ep_wait(const int *flags, int which, int world, const int *epoch, void *stream) {
  MQ_REQUIRE(flags && epoch && (which == 0 || which == 1) && world >= 1 && world <= 256, MQ_EINVAL,
             "mq_ep_wait: bad arguments");
  return mq::launch_overlapped(mq::ep::wait_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), "mq_ep_wait",
                               flags, which, world, epoch);
}

extern "C" int mq_ep_return(const float *z, const int32_t *slot_of, const int32_t *ids, int64_t d, int world, int rank,
                            int cap, float *const *peer_ret, int *const *peer_flags, const int *epoch, int *done,
                            void *stream) {
  MQ_REQUIRE(z && ids && peer_ret && peer_flags && epoch && done, MQ_EINVAL, "mq_ep_return: null pointer");
  MQ_REQUIRE(world >= 1 && world <= 256 && rank >= 0 && rank < world && cap >= 1 && d > 0 && d % 4 == 0, MQ_EINVAL,
             "mq_ep_return: bad shape");
  MQ_REQUIRE(mq::aligned(z, 16), MQ_EALIGN, "mq_ep_return: z must be 16-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  return mq::launch_overlapped(mq::ep::return_kernel, dim3(mq::ep::grid_for(static_cast<int64_t>(world) * cap * (d / 4) / 4, dev)),
                               dim3(256), 0, static_cast<cudaStream_t>(stream), "mq_ep_return", z, slot_of, ids,
                               static_cast<int>(d), world, rank, cap, peer_ret, peer_flags, epoch, done);
}
