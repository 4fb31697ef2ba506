// Weight packers on the device: the byte layouts the matmul kernels read, produced from raw weights
// at load time (the reference produces them offline with its converters).
//
//  * mq_quantize_q4, method MQ_Q4_MAX7: symmetric int4 with scale fp16(max|w| / 7) per group and
//    q = clip(rint(w / scale), -8, 7) on fp16-rounded values: llama/run.py:56-70 (quantize4) and
//    llama/st2bin.c:54-70 (bf16 input, rounded to fp16 first).
//  * method MQ_Q4_SEARCH: the searched scale of qwen3moe/convert.c:124-157 and :394-433: candidates
//    t = fp16(max|w| / d) for d = 6.5, 6.75, ..., 9, squared error summed in fp32 in element order,
//    the first least error kept; the values are used as they are (bf16 / fp16 / fp32).
//  * mq_q4_0_to_words: GGUF Q4_0 blocks (fp16 d + 16 bytes, element j the low nibble of byte j and
//    element j + 16 its high nibble, value nibble - 8) to the word layout (nibble ^ 8 at element
//    8w + i) and the scales unchanged: lfm2/convert.c:58-71.
//  * mq_pack_ternary: MLX 2-bit rows to the transposed ternary layout, checking that every group is
//    ternary (bias == -scale): qwen3/convert.cpp:39-74.
//  * mq_pack_half: fp32 pairs to fp16 pairs in one 32-bit word (pack_half, qwen3/kernels/qwen3k.mojo:
//    17-20,45-48), the activation format of the ternary GEMV.
// The arithmetic that decides a scale is written with explicitly rounded operations (no fused
// multiply-add), so the bytes equal the reference converters', which build with contraction off.
#include <mutex>

#include "common.cuh"

namespace mq {
namespace pack {

__device__ __forceinline__ float load_value(const void *w, int dtype, int64_t i) {
  if (dtype == MQ_F32) return static_cast<const float *>(w)[i];
  const uint16_t bits = static_cast<const uint16_t *>(w)[i];
  if (dtype == MQ_F16) return __half2float(__ushort_as_half(bits));
  return __uint_as_float(static_cast<uint32_t>(bits) << 16);  // bf16
}

__device__ __forceinline__ int quantize(float w, float s) {
  const float q = s > 0.f ? rintf(__fdiv_rn(w, s)) : 0.f;
  return q < -8.f ? -8 : q > 7.f ? 7 : static_cast<int>(q);
}

// One thread per group of G consecutive weights of a row.
template <int G, int METHOD>
__global__ void quantize_kernel(const void *__restrict__ w, int dtype, int64_t groups, uint32_t *__restrict__ wq,
                                __half *__restrict__ ws) {
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t base = g * G;
    auto value = [&](int j) {
      const float v = load_value(w, dtype, base + j);
      return METHOD == MQ_Q4_MAX7 ? __half2float(__float2half_rn(v)) : v;
    };
    float m = 0.f;
    for (int j = 0; j < G; ++j) m = fmaxf(m, fabsf(value(j)));
    float s;
    if (METHOD == MQ_Q4_MAX7) {
      s = __half2float(__float2half_rn(__fdiv_rn(m, 7.f)));
    } else {
      float best = INFINITY;
      s = 0.f;
      for (float d = 6.5f; d <= 9.0f; d = __fadd_rn(d, 0.25f)) {
        const float t = __half2float(__float2half_rn(__fdiv_rn(m, d)));
        if (!(t > 0.f)) break;
        float e = 0.f;
        for (int j = 0; j < G; ++j) {
          const float v = value(j);
          const float diff = __fsub_rn(v, __fmul_rn(static_cast<float>(quantize(v, t)), t));
          e = __fadd_rn(e, __fmul_rn(diff, diff));
        }
        if (e < best) {
          best = e;
          s = t;
        }
      }
    }
    ws[g] = __float2half_rn(s);
#pragma unroll 1
    for (int wi = 0; wi < G / 8; ++wi) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) word |= static_cast<uint32_t>(quantize(value(8 * wi + i), s) & 15) << (4 * i);
      wq[g * (G / 8) + wi] = word;
    }
  }
}

// One thread per 18-byte block.
__global__ void q4_0_kernel(const uint8_t *__restrict__ blocks, int64_t nblocks, uint32_t *__restrict__ wq,
                            uint16_t *__restrict__ ws) {
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(blocks + b * 18);  // 18 is even: 2-byte aligned
    ws[b] = h[0];
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = static_cast<uint32_t>(h[1 + 2 * i]) | (static_cast<uint32_t>(h[2 + 2 * i]) << 16);
    // byte j of the 16 holds element j (low nibble) and element j + 16 (high nibble)
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = 8 * wi + i, byte = e & 15;
        const uint32_t nib = (q[byte >> 2] >> (8 * (byte & 3) + (e >= 16 ? 4 : 0))) & 15u;
        word |= (nib ^ 8u) << (4 * i);
      }
      wq[b * 4 + wi] = word;
    }
  }
}

// out[c][r] = in[r][c] for an [rows][cols] matrix of 4- or 2-byte elements, 32 x 32 tiles through
// shared memory (both sides coalesced).
template <typename T>
__global__ void transpose_kernel(const T *__restrict__ in, T *__restrict__ out, int64_t rows, int64_t cols) {
  __shared__ T tile[32][33];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][i];
  }
}

__device__ int g_not_ternary;

__global__ void ternary_check_kernel(const uint16_t *__restrict__ s, const uint16_t *__restrict__ b, int64_t count) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (__half2float(__ushort_as_half(b[i])) != -__half2float(__ushort_as_half(s[i]))) atomicExch(&g_not_ternary, 1);
  }
}

__global__ void pack_half_kernel(const float2 *__restrict__ x, __half2 *__restrict__ q, int64_t pairs) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float2 v = x[i];
    q[i] = __halves2half2(__float2half_rn(v.x), __float2half_rn(v.y));
  }
}

inline int grid_for(int64_t items, int threads, const DeviceInfo &dev) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + threads - 1) / threads, dev.sms * 16LL)));
}

template <int METHOD>
void launch_quantize(const void *w, int dtype, int64_t groups, int group, uint32_t *wq, __half *ws, int grid,
                     cudaStream_t s) {
  switch (group) {
    case 32: quantize_kernel<32, METHOD><<<grid, 128, 0, s>>>(w, dtype, groups, wq, ws); break;
    case 64: quantize_kernel<64, METHOD><<<grid, 128, 0, s>>>(w, dtype, groups, wq, ws); break;
    default: quantize_kernel<128, METHOD><<<grid, 128, 0, s>>>(w, dtype, groups, wq, ws); break;
  }
}

}  // namespace pack
}  // namespace mq

extern "C" int mq_quantize_q4(const void *w, int w_dtype, int64_t n, int64_t k, int group, int method, uint32_t *wq,
                              uint16_t *ws, void *stream) {
  MQ_REQUIRE(w && wq && ws, MQ_EINVAL, "mq_quantize_q4: null pointer");
  MQ_REQUIRE(w_dtype == MQ_F32 || w_dtype == MQ_F16 || w_dtype == MQ_BF16, MQ_EINVAL,
             "mq_quantize_q4: w_dtype must be MQ_F32, MQ_F16 or MQ_BF16");
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL, "mq_quantize_q4: group must be 32, 64 or 128");
  MQ_REQUIRE(method == MQ_Q4_MAX7 || method == MQ_Q4_SEARCH, MQ_EINVAL,
             "mq_quantize_q4: method must be MQ_Q4_MAX7 or MQ_Q4_SEARCH");
  MQ_REQUIRE(n > 0 && k > 0 && k % group == 0, MQ_EINVAL, "mq_quantize_q4: k must be a positive multiple of group");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  const int64_t groups = n * (k / group);
  const int grid = mq::pack::grid_for(groups, 128, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  __half *hs = reinterpret_cast<__half *>(ws);
  if (method == MQ_Q4_MAX7)
    mq::pack::launch_quantize<MQ_Q4_MAX7>(w, w_dtype, groups, group, wq, hs, grid, s);
  else
    mq::pack::launch_quantize<MQ_Q4_SEARCH>(w, w_dtype, groups, group, wq, hs, grid, s);
  return mq::check_launch("mq_quantize_q4");
}

extern "C" int mq_q4_0_to_words(const uint8_t *blocks, int64_t nblocks, uint32_t *wq, uint16_t *ws, void *stream) {
  MQ_REQUIRE(blocks && wq && ws, MQ_EINVAL, "mq_q4_0_to_words: null pointer");
  MQ_REQUIRE(nblocks > 0, MQ_EINVAL, "mq_q4_0_to_words: nblocks must be positive");
  MQ_REQUIRE(mq::aligned(blocks, 2) && mq::aligned(ws, 2) && mq::aligned(wq, 4), MQ_EALIGN,
             "mq_q4_0_to_words: blocks and ws must be 2-byte aligned, wq 4-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  mq::pack::q4_0_kernel<<<mq::pack::grid_for(nblocks, 256, dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      blocks, nblocks, wq, ws);
  return mq::check_launch("mq_q4_0_to_words");
}

extern "C" int mq_pack_ternary(const uint32_t *codes, const uint16_t *scales, const uint16_t *biases, int64_t n,
                               int64_t k, uint32_t *w, uint16_t *s, void *stream) {
  MQ_REQUIRE(codes && scales && w && s, MQ_EINVAL, "mq_pack_ternary: null pointer");
  MQ_REQUIRE(n > 0 && k > 0 && k % 128 == 0 && n < (1LL << 31), MQ_EINVAL,
             "mq_pack_ternary: k must be a positive multiple of 128");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static std::mutex mu;  // one check flag per process: checks run one at a time
  std::lock_guard<std::mutex> lock(mu);
  if (biases) {
    const int zero = 0;
    cudaError_t e = cudaMemcpyToSymbolAsync(mq::pack::g_not_ternary, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_pack_ternary: %s", cudaGetErrorString(e));
    const int64_t count = n * (k / 128);
    mq::pack::ternary_check_kernel<<<mq::pack::grid_for(count, 256, dev), 256, 0, st>>>(scales, biases, count);
    if (int rc = mq::check_launch("mq_pack_ternary (check)")) return rc;
    int bad = 0;
    e = cudaMemcpyFromSymbolAsync(&bad, mq::pack::g_not_ternary, sizeof bad, 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_pack_ternary: %s", cudaGetErrorString(e));
    MQ_REQUIRE(!bad, MQ_EINVAL, "mq_pack_ternary: not ternary (bias != -scale)");
  }
  const dim3 block(32, 8);
  mq::pack::transpose_kernel<uint32_t><<<dim3((k / 16 + 31) / 32, (n + 31) / 32), block, 0, st>>>(codes, w, n, k / 16);
  if (int rc = mq::check_launch("mq_pack_ternary (codes)")) return rc;
  mq::pack::transpose_kernel<uint16_t><<<dim3((k / 128 + 31) / 32, (n + 31) / 32), block, 0, st>>>(scales, s, n, k / 128);
  return mq::check_launch("mq_pack_ternary (scales)");
}

extern "C" int mq_pack_half(const float *x, uint32_t *q, int64_t n, void *stream) {
  MQ_REQUIRE(x && q, MQ_EINVAL, "mq_pack_half: null pointer");
  MQ_REQUIRE(n > 0 && n % 2 == 0, MQ_EINVAL, "mq_pack_half: n must be a positive even count");
  MQ_REQUIRE(mq::aligned(x, 8) && mq::aligned(q, 4), MQ_EALIGN, "mq_pack_half: x must be 8-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  mq::pack::pack_half_kernel<<<mq::pack::grid_for(n / 2, 256, dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float2 *>(x), reinterpret_cast<__half2 *>(q), n / 2);
  return mq::check_launch("mq_pack_half");
}
