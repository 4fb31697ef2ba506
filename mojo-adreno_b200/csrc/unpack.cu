// Bit-exact unpack hook (mq_unpack_q4): the integer half of the reference's dequantiser.
//
// q[r][8w + j] = ((word >> 4j) & 15 ^ 8) - 8 as int8, the decode of gemv_q4
// (llama/kernels/gemv_q4.mojo:23-25) and of Weights.int4 (qwen3moe/reference.py:53-65); the scales
// are copied unchanged. One thread per word, two 32-bit stores of four int8 each.
#include "common.cuh"

namespace mq {
namespace unpack {

__global__ void unpack_q4_kernel(const uint32_t *__restrict__ wq, uint32_t *__restrict__ q, int64_t words) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t u = wq[i] ^ 0x88888888u;  // offset binary: value + 8
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo |= ((((u >> (4 * j)) & 15u) - 8u) & 0xFFu) << (8 * j);
      hi |= ((((u >> (4 * j + 16)) & 15u) - 8u) & 0xFFu) << (8 * j);
    }
    q[2 * i] = lo;
    q[2 * i + 1] = hi;
  }
}

}  // namespace unpack
}  // namespace mq

extern "C" int mq_unpack_q4(const uint32_t *wq, const uint16_t *ws, int8_t *q, uint16_t *s_out, int64_t n, int64_t k,
                            int group, void *stream) {
  MQ_REQUIRE(wq && ws && q, MQ_EINVAL, "mq_unpack_q4: null pointer");
  MQ_REQUIRE(n > 0 && k > 0, MQ_EINVAL, "mq_unpack_q4: bad shape");
  MQ_REQUIRE(group > 0 && k % 8 == 0 && k % group == 0, MQ_EINVAL, "mq_unpack_q4: k must be a multiple of 8 and of group");
  MQ_REQUIRE(mq::aligned(q, 4) && mq::aligned(wq, 4), MQ_EALIGN, "mq_unpack_q4: q and wq must be 4-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t words = n * (k / 8);
  const int grid = static_cast<int>(std::min<int64_t>((words + 255) / 256, static_cast<int64_t>(dev.sms) * 16));
  mq::unpack::unpack_q4_kernel<<<grid, 256, 0, s>>>(wq, reinterpret_cast<uint32_t *>(q), words);
  if (int rc = mq::check_launch("mq_unpack_q4")) return rc;
  if (s_out) {
    cudaError_t e = cudaMemcpyAsync(s_out, ws, static_cast<size_t>(n) * (k / group) * 2, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_unpack_q4: scale copy: %s", cudaGetErrorString(e));
  }
  return MQ_OK;
}
