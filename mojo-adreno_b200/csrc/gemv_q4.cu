// Decode GEMV over int4 word-layout weights (mq_gemv_q4), batch 1..4.
//
// Replaces gemv_q4 / gemv_add_q4 (llama/kernels/gemv_q4.mojo:13-30, gemv_add_q4.mojo:13-30), the
// Q4_0 G=32 variant (lfm2/kernels/lk.mojo:56-72,134-143) and the small-batch t_gemv_q4 / p_gemv_q4
// (qwen3moe/kernels/moek.mojo:273-281,528-545). Same arithmetic: y[r] = sum over words of
// scale * sum_j ((nib_j ^ 8) - 8) * x[8w + j], fp32 x and y.
//
// B200 design (HBM-bound: 0.5625 B per weight at G=32):
//  * Issue budget. At ~6.5 TB/s an SM must retire ~46 weights per clock; it issues 128 lane
//    instructions per clock, so decode + multiply must cost well under 2.8 instructions per
//    weight. An fp32 FMA path (extract, convert, subtract, FMA) costs ~4. Here the warp-level
//    tensor op mma.m16n8k16 (fp16 in, fp32 accumulate) does the multiply-add, and the decode is
//    two logic ops per pair of weights.
//  * Decode. A nibble pair masked straight into the mantissa bits of an fp16x2 register is an
//    exact fp16 subnormal: (u & 0x000F000F) holds u_lo * 2^-24 | u_hi * 2^-24 and
//    (u & 0x00F000F0) holds 16u * 2^-24 (still below the 2^-14 normal threshold), where
//    u = nib ^ 8 = value + 8 in 0..15 (offset binary). So per 32-bit word: one XOR, one shift and
//    four ANDs give all eight weights, exactly. The factors 2^-24 (and 16) are undone on the
//    activation side (x/16 in the matching B slots) and in the fp32 epilogue (scale * 2^24), and
//    the offset is removed with the precomputed sum of x: sum (u - 8) x = sum u x - 8 sum x.
//  * Exact per-group scales. Lanes of a quad (lane % 4 == q) load 16 consecutive bytes of a row
//    (32 weights = 32 k of the same scale group for G=32). The B fragment puts quad q's slots of
//    x in column q only, so D column q holds quad q's dot product alone: the fp32 epilogue applies
//    each group's scale to its own partial sum, in fp32, as the reference does.
//  * fp32 x fidelity. Columns 4..7 carry the fp16 residual x - fp16(x) (batch <= 2), so the
//    product sees ~22 bits of x; the weights are exact integers; accumulation is fp32.
//  * Memory. Each lane streams 128-bit, L1-no-allocate loads (rows g and g+8 of a 16-row tile,
//    64 contiguous bytes per row per quad), 4 chunks of 128 k in flight. Small matrices split K
//    across the 8 warps of a CTA (partials reduced in shared memory); CTAs are persistent over
//    row blocks so x is staged once per CTA.
#include <algorithm>

#include "common.cuh"

namespace mq {
namespace gemv {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kPrefetch = 4;  // 128-k chunks whose loads a warp issues together

struct GemvQ4Params {
  const uint32_t *wq;
  const __half *ws;
  const void *x;
  float *y;
  int n, k, batch, x_f16, add;
  int ks;       // warps of a CTA that split K
  int rt;       // 16-row tiles of a CTA (rt * ks == kWarps)
  int nblocks;  // row blocks (rt tiles each)
};

// The eight weights of one word as four fp16x2 subnormal pairs (see the file comment).
__device__ __forceinline__ void decode_q4(uint32_t w, uint32_t &p0, uint32_t &p1, uint32_t &p2, uint32_t &p3) {
  const uint32_t u = w ^ 0x88888888u;
  p0 = u & 0x000F000Fu;  // nibbles 0 | 4, factor 1
  p1 = u & 0x00F000F0u;  // nibbles 1 | 5, factor 16
  const uint32_t v = u >> 8;
  p2 = v & 0x000F000Fu;  // nibbles 2 | 6, factor 1
  p3 = v & 0x00F000F0u;  // nibbles 3 | 7, factor 16
}

__device__ __forceinline__ float load_x(const void *x, int x_f16, size_t i) {
  return x_f16 ? __half2float(static_cast<const __half *>(x)[i]) : static_cast<const float *>(x)[i];
}

// NT: mma n-tiles per k step; LO: column 4+q carries the residual of column q (batch <= 2),
// otherwise columns 4..7 carry a second token.
template <int G, int NT, bool LO>
__global__ void __launch_bounds__(kThreads) gemv_q4_kernel(const GemvQ4Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = p.k, N = p.n, B = p.batch;
  const int kc = (K + 127) / 128;  // chunks of 128 k
  const int nsteps = kc * 8;       // mma k16 steps
  const int wpr = K / 8;           // words per row
  const int spr = K / G;           // scales per row
  uint2 *bfrag = reinterpret_cast<uint2 *>(smem);                 // [NT][nsteps][8]
  float *xsum = reinterpret_cast<float *>(bfrag + NT * nsteps * 8);  // [B][kc*4]
  float *red = xsum + B * kc * 4;                                 // [kWarps][16][B]

  // ---- stage x: B fragments (fp16 hi/lo, permuted to the decode's slot order) and quad sums --
  for (int i = threadIdx.x; i < NT * nsteps * 8; i += kThreads) bfrag[i] = make_uint2(0u, 0u);
  __syncthreads();
  for (int it = threadIdx.x; it < B * kc * 16; it += kThreads) {
    const int t = it / (kc * 16), wi = it % (kc * 16);
    const int c = wi / 16, q = (wi / 4) % 4, j = wi % 4;
    float xv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int kk = 8 * wi + e;
      xv[e] = kk < K ? load_x(p.x, p.x_f16, static_cast<size_t>(t) * K + kk) : 0.f;
      if (e == 1 || e == 3 || e == 5 || e == 7) xv[e] *= 0.0625f;  // slots whose weights carry 16
    }
    float hv[8], lv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      hv[e] = __half2float(__float2half_rn(xv[e]));
      lv[e] = xv[e] - hv[e];
    }
    const int s0 = c * 8 + 2 * j;
    int tile, col;
    if (LO) {
      tile = t;
      col = q;
    } else {
      tile = t / 2;
      col = 4 * (t % 2) + q;
    }
    uint2 *dst = bfrag + (static_cast<size_t>(tile) * nsteps + s0) * 8;
    dst[col] = make_uint2(pack_half2(hv[0], hv[4]), pack_half2(hv[1], hv[5]));
    dst[8 + col] = make_uint2(pack_half2(hv[2], hv[6]), pack_half2(hv[3], hv[7]));
    if (LO) {
      dst[4 + col] = make_uint2(pack_half2(lv[0], lv[4]), pack_half2(lv[1], lv[5]));
      dst[8 + 4 + col] = make_uint2(pack_half2(lv[2], lv[6]), pack_half2(lv[3], lv[7]));
    }
  }
  for (int it = threadIdx.x; it < B * kc * 4; it += kThreads) {
    const int t = it / (kc * 4), qi = it % (kc * 4);
    float s = 0.f;
    for (int e = 0; e < 32; ++e) {
      const int kk = 32 * qi + e;
      if (kk < K) s += load_x(p.x, p.x_f16, static_cast<size_t>(t) * K + kk);
    }
    xsum[t * kc * 4 + qi] = s;
  }
  __syncthreads();

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane >> 2, q = lane & 3;
  const int kw = warp % p.ks, rtl = warp / p.ks;
  const int cpw = (kc + p.ks - 1) / p.ks;
  const int cb = kw * cpw, ce = min(kc, cb + cpw);
  const bool act = q == (g & 3);  // lanes whose B fragment is non-zero
  const int qa = 2 * (q & 1);     // first of the two quads whose columns this lane's D holds

  for (int rb = blockIdx.x; rb < p.nblocks; rb += gridDim.x) {
    const int row0 = (rb * p.rt + rtl) * 16;
    const int ra = row0 + g, rbw = row0 + g + 8;
    const bool va = ra < N, vb = rbw < N;
    const uint32_t *pa = p.wq + static_cast<size_t>(va ? ra : 0) * wpr + 4 * q;
    const uint32_t *pb = p.wq + static_cast<size_t>(vb ? rbw : 0) * wpr + 4 * q;
    const __half *sa = p.ws + static_cast<size_t>(va ? ra : 0) * spr;
    const __half *sb = p.ws + static_cast<size_t>(vb ? rbw : 0) * spr;
    float acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = 0.f;

    for (int c = cb; c < ce; c += kPrefetch) {
      uint4 wa[kPrefetch], wb[kPrefetch];
      float s_a[kPrefetch][2], s_b[kPrefetch][2];
#pragma unroll
      for (int i = 0; i < kPrefetch; ++i) {
        const int cc = c + i;
        const bool okw = cc < ce && (cc * 16 + 4 * q) < wpr;
        wa[i] = (okw && va) ? ldg_stream_v4(pa + cc * 16) : make_uint4(0u, 0u, 0u, 0u);
        wb[i] = (okw && vb) ? ldg_stream_v4(pb + cc * 16) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int si = (128 * cc + 32 * (qa + h)) / G;
          const bool oks = cc < ce && si < spr;
          s_a[i][h] = (oks && va) ? __half2float(sa[si]) : 0.f;
          s_b[i][h] = (oks && vb) ? __half2float(sb[si]) : 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < kPrefetch; ++i) {
        const int cc = c + i;
        if (cc >= ce) break;
        float d[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t) d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0.f;
        const uint32_t wav[4] = {wa[i].x, wa[i].y, wa[i].z, wa[i].w};
        const uint32_t wbv[4] = {wb[i].x, wb[i].y, wb[i].z, wb[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
          decode_q4(wav[j], a0, a1, a2, a3);
          decode_q4(wbv[j], b0, b1, b2, b3);
          const int s = cc * 8 + 2 * j;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint2 *bf = bfrag + (static_cast<size_t>(t) * nsteps + s) * 8 + g;
            const uint2 f0 = act ? bf[0] : make_uint2(0u, 0u);
            const uint2 f1 = act ? bf[8] : make_uint2(0u, 0u);
            mma_16816(d[t], a0, b0, a1, b1, f0.x, f0.y);
            mma_16816(d[t], a2, b2, a3, b3, f1.x, f1.y);
          }
        }
        // fp32 epilogue: per-column group scale, 2^24 factor, offset through the quad sums of x.
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int tok = LO ? t : 2 * t + (q >> 1);
          const bool hi = LO ? (q < 2) : true;
          if (tok < B) {
            const float *xs = xsum + tok * kc * 4 + cc * 4 + qa;
            const float x0 = hi ? 8.f * xs[0] : 0.f, x1 = hi ? 8.f * xs[1] : 0.f;
            acc[t][0] += s_a[i][0] * fmaf(d[t][0], 16777216.f, -x0) + s_a[i][1] * fmaf(d[t][1], 16777216.f, -x1);
            acc[t][1] += s_b[i][0] * fmaf(d[t][2], 16777216.f, -x0) + s_b[i][1] * fmaf(d[t][3], 16777216.f, -x1);
          }
        }
      }
    }
    // Reduce the quad's lanes, then the K-splitting warps through shared memory.
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float v = acc[t][r];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if (LO) v += __shfl_xor_sync(0xffffffffu, v, 2);
        acc[t][r] = v;
      }
      const int tok = LO ? t : 2 * t + (q >> 1);
      const bool writer = LO ? (q == 0) : ((q & 1) == 0);
      if (writer && tok < B) {
        red[(kw * 16 * p.rt + rtl * 16 + g) * B + tok] = acc[t][0];
        red[(kw * 16 * p.rt + rtl * 16 + g + 8) * B + tok] = acc[t][1];
      }
    }
    __syncthreads();
    const int rows = 16 * p.rt;
    for (int it = threadIdx.x; it < rows * B; it += kThreads) {
      const int rl = it / B, tok = it % B;
      const int r = rb * rows + rl;
      if (r < N) {
        float v = 0.f;
        for (int w = 0; w < p.ks; ++w) v += red[(w * rows + rl) * B + tok];
        float *out = p.y + static_cast<size_t>(tok) * N + r;
        *out = p.add ? *out + v : v;
      }
    }
    __syncthreads();
  }
}

template <int G, int NT, bool LO>
int launch(const GemvQ4Params &p0, cudaStream_t stream, const DeviceInfo &dev) {
  GemvQ4Params p = p0;
  const int kc = (p.k + 127) / 128;
  const size_t smem = static_cast<size_t>(NT) * (kc * 8) * 8 * sizeof(uint2) +
                      static_cast<size_t>(p.batch) * kc * 4 * sizeof(float) +
                      static_cast<size_t>(kWarps) * 16 * p.batch * sizeof(float);
  MQ_REQUIRE(smem <= dev.smem_optin, MQ_EUNSUPPORTED, "mq_gemv_q4: k=%d batch=%d needs %zu B of shared memory (max %zu)",
             p.k, p.batch, smem, dev.smem_optin);
  auto kern = gemv_q4_kernel<G, NT, LO>;
  static size_t configured = 0;  // largest dynamic smem size set on this instantiation
  if (smem > 48 * 1024 && smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(MQ_ECUDA, "mq_gemv_q4: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = smem;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1) return fail(MQ_ECUDA, "mq_gemv_q4: occupancy query failed (%s)", cudaGetErrorString(e));
  const int grid = std::min(p.nblocks, dev.sms * per_sm);
  kern<<<grid, kThreads, smem, stream>>>(p);
  return check_launch("mq_gemv_q4");
}

template <int G>
int dispatch_nt(const GemvQ4Params &p, cudaStream_t s, const DeviceInfo &dev) {
  const bool lo = !p.x_f16 && p.batch <= 2;
  if (lo) return p.batch == 1 ? launch<G, 1, true>(p, s, dev) : launch<G, 2, true>(p, s, dev);
  return p.batch <= 2 ? launch<G, 1, false>(p, s, dev) : launch<G, 2, false>(p, s, dev);
}

// Used by the batched path and by the MoE decode: one GEMV launch over [n, k] with batch <= 4.
int gemv_q4_small(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y, int64_t n,
                  int64_t k, int group, int batch, int add, cudaStream_t stream) {
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  GemvQ4Params p{};
  p.wq = wq;
  p.ws = reinterpret_cast<const __half *>(ws);
  p.x = x;
  p.y = y;
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = batch;
  p.x_f16 = x_dtype == MQ_F16;
  p.add = add != 0;
  const int kc = static_cast<int>((k + 127) / 128);
  const int tiles = static_cast<int>((n + 15) / 16);
  const int target = dev.sms * 16;  // warps wanted in flight
  int ks = 1;
  while (ks < kWarps && static_cast<long>(tiles) * ks < target && ks * 2 <= kc) ks *= 2;
  p.ks = ks;
  p.rt = kWarps / ks;
  p.nblocks = (tiles + p.rt - 1) / p.rt;
  switch (group) {
    case 32: return dispatch_nt<32>(p, stream, dev);
    case 64: return dispatch_nt<64>(p, stream, dev);
    default: return dispatch_nt<128>(p, stream, dev);
  }
}

}  // namespace gemv
}  // namespace mq

extern "C" int mq_gemv_q4(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y, int64_t n,
                          int64_t k, int group, int batch, int add, void *stream) {
  MQ_REQUIRE(wq && ws && x && y, MQ_EINVAL, "mq_gemv_q4: null pointer");
  MQ_REQUIRE(n > 0 && k > 0 && n < (1LL << 31) && k <= (1 << 20), MQ_EINVAL, "mq_gemv_q4: bad shape n=%lld k=%lld",
             static_cast<long long>(n), static_cast<long long>(k));
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL, "mq_gemv_q4: group must be 32, 64 or 128 (got %d)", group);
  MQ_REQUIRE(k % 32 == 0 && k % group == 0, MQ_EINVAL, "mq_gemv_q4: k=%lld must be a multiple of 32 and of group=%d",
             static_cast<long long>(k), group);
  MQ_REQUIRE(x_dtype == MQ_F32 || x_dtype == MQ_F16, MQ_EINVAL, "mq_gemv_q4: x_dtype must be MQ_F32 or MQ_F16");
  MQ_REQUIRE(batch >= 1 && batch <= 64, MQ_EINVAL, "mq_gemv_q4: batch must be in 1..64 (got %d)", batch);
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(ws, 2) && mq::aligned(x, 4) && mq::aligned(y, 4), MQ_EALIGN,
             "mq_gemv_q4: wq must be 16-byte aligned, x and y 4-byte aligned");
  if (batch > 4) return mq::fail(MQ_EUNSUPPORTED, "mq_gemv_q4: batch > 4 needs the tensor-core GEMM path");
  return mq::gemv::gemv_q4_small(wq, ws, x, x_dtype, y, n, k, group, batch, add, static_cast<cudaStream_t>(stream));
}
