// Library-wide entry points (error string, version, device status word) and the host helpers
// declared in common.cuh.
#include "common.cuh"

namespace mq {

namespace {
thread_local char t_error[512] = "";
}

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof t_error, fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MQ_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return MQ_OK;
}

int device_info(DeviceInfo *out) {
  static DeviceInfo cache[64];
  static bool valid[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MQ_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(MQ_EUNSUPPORTED, "device index %d out of range", dev);
  if (!valid[dev]) {
    DeviceInfo d;
    int v = 0;
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return fail(MQ_ECUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    d.smem_optin = static_cast<size_t>(v);
    if (d.major != 10) return fail(MQ_EUNSUPPORTED, "libmq is built for sm_100a; device is sm_%d%d", d.major, d.minor);
    cache[dev] = d;
    valid[dev] = true;
  }
  *out = cache[dev];
  return MQ_OK;
}

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
}  // namespace

namespace {
// The last maps this thread encoded, by their full description: a decode step encodes the same
// few maps every call, and the driver call costs about as much as the kernel launch. A map holds
// only the address, sizes and strides it was built from, so an equal description gives an equal map.
struct TmapKey {
  const void *base;
  uint64_t cols, rows, row_stride;
  uint32_t box_cols, box_rows;
  int dtype, swizzle;
  bool operator==(const TmapKey &o) const {
    return base == o.base && cols == o.cols && rows == o.rows && row_stride == o.row_stride &&
           box_cols == o.box_cols && box_rows == o.box_rows && dtype == o.dtype && swizzle == o.swizzle;
  }
};
constexpr int kTmapCache = 32;
thread_local TmapKey t_keys[kTmapCache];
thread_local CUtensorMap t_maps[kTmapCache];
thread_local int t_nkeys = 0, t_next = 0;
}  // namespace

int encode_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                   uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                   CUtensorMapSwizzle swizzle, const char *what) {
  const TmapKey key{base, cols, rows, row_stride_bytes, box_cols, box_rows, static_cast<int>(dtype),
                    static_cast<int>(swizzle)};
  for (int i = 0; i < t_nkeys; ++i)
    if (t_keys[i] == key) {
      *map = t_maps[i];
      return MQ_OK;
    }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MQ_ECUDA, "%s: cuTensorMapEncodeTiled is not available from the driver", what);
  if (reinterpret_cast<uintptr_t>(base) % 16 || row_stride_bytes % 16 || (box_cols * elem_bytes) % 16)
    return fail(MQ_EALIGN, "%s: tensor map needs a 16-byte aligned base, row stride and box row", what);
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MQ_ECUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  t_keys[t_next] = key;
  t_maps[t_next] = *map;
  t_next = (t_next + 1) % kTmapCache;
  if (t_nkeys < kTmapCache) ++t_nkeys;
  return MQ_OK;
}

int encode_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                   uint64_t rows, uint64_t planes, uint64_t row_stride_bytes, uint64_t plane_stride_bytes,
                   uint32_t box_cols, uint32_t box_rows, uint32_t box_planes, CUtensorMapSwizzle swizzle,
                   const char *what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MQ_ECUDA, "%s: cuTensorMapEncodeTiled is not available from the driver", what);
  if (reinterpret_cast<uintptr_t>(base) % 16 || row_stride_bytes % 16 || plane_stride_bytes % 16 ||
      (box_cols * elem_bytes) % 16)
    return fail(MQ_EALIGN, "%s: tensor map needs a 16-byte aligned base, strides and box row", what);
  const cuuint64_t dims[3] = {cols, rows, planes};
  const cuuint64_t strides[2] = {row_stride_bytes, plane_stride_bytes};
  const cuuint32_t box[3] = {box_cols, box_rows, box_planes};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MQ_ECUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return MQ_OK;
}

}  // namespace mq

extern "C" {

const char *mq_last_error(void) { return mq::t_error; }

int mq_version(void) { return 100; }

int mq_device_status(int reset, void *stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int value = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&value, mq::g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_device_status: %s", cudaGetErrorString(e));
  if (reset && value) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(mq::g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_device_status reset: %s", cudaGetErrorString(e));
  }
  return value;
}

}  // extern "C"
