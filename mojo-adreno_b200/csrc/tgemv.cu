// Ternary decode GEMV (mq_tgemv) over the transposed 2-bit layout, batch 1..4.
//
// Replaces packed_linear + packed_reduce (bonsai/kernels/kernels.mojo:283-325,437-448) and the
// product part of packed_head (:451-489): y[i] = sum over 128-k groups g of
// s[g][i] * sum_k (code(k, i) - 1) * x[k], code(k, i) = (w[(k/16) n + i] >> 2 (k % 16)) & 3.
// The reference accumulates each group in fp16 FMA chains (_group_dot8, :227-280); this kernel
// multiplies exactly (codes are small integers, x is fp16) and accumulates in fp32, so its error
// against exact arithmetic is far below the reference's own.
//
// B200 design (HBM-bound: 0.2656 B per weight, ~92 weights per SM clock at 6.5 TB/s, leaving
// under 1.4 issued instructions per weight):
//  * Decode: a 2-bit code pair masked into the mantissa of an fp16x2 register is an exact
//    subnormal: (w & (0x00030003 << 2j)) holds c * 4^j * 2^-24 for j = 0..3; one shift by 8 gives
//    the other four pairs. Eight ANDs and one shift per 16 weights; the 4^-j factors go into the
//    activation (B) slots and 2^24 into the fp32 epilogue; the -1 offset is removed with the
//    group's sum of x: sum (c - 1) x = sum c x - sum x.
//  * Multiply: mma.m16n8k16 (fp16 in, fp32 accumulate); one group (128 k) = 8 k16 steps, after
//    which the group's fp16 scale is applied in fp32.
//  * Memory: the layout is [k/16][n] words, so a lane loads one 128-bit vector = 4 adjacent
//    outputs x 16 k; 8 lanes of a quad row read 128 contiguous bytes. A warp owns 32 outputs
//    (two m16 tiles) over a K range; small matrices split K over the CTA's 8 warps.
#include <algorithm>

#include "common.cuh"

namespace mq {
namespace tg {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kPrefetch = 4;  // groups (2 x 128-bit loads per lane each) in flight

struct TgemvParams {
  const uint16_t *x;
  const uint32_t *w;
  const __half *s;
  float *y;
  int n, k, batch;
  int ks, rt, nblocks;
};

// Pairs j = 0..7 of a word: codes (j, j + 8) for j < 4 from w, (j, j + 8) for j >= 4 from w >> 8.
__device__ __forceinline__ void decode_t2(uint32_t w, uint32_t (&q)[8]) {
  q[0] = w & 0x00030003u;
  q[1] = w & 0x000C000Cu;
  q[2] = w & 0x00300030u;
  q[3] = w & 0x00C000C0u;
  const uint32_t v = w >> 8;
  q[4] = v & 0x00030003u;
  q[5] = v & 0x000C000Cu;
  q[6] = v & 0x00300030u;
  q[7] = v & 0x00C000C0u;
}

template <int NB>  // NB = batch (columns used)
__global__ void __launch_bounds__(kThreads) tgemv_kernel(const TgemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = p.k, N = p.n;
  const int kb = K / 64;    // blocks of 4 k16 steps
  const int kg = K / 128;   // scale groups
  const int nsteps = kb * 4;
  uint2 *bfrag = reinterpret_cast<uint2 *>(smem);             // [nsteps][NB][4]
  float *xsum = reinterpret_cast<float *>(bfrag + nsteps * NB * 4);  // [NB][kg]
  float *red = xsum + NB * kg;                                // [kWarps][32][NB]

  // ---- stage x: per step s = 4b + t and lane (column tok, quad q):
  //      b0 = (x[16(4b+q) + 2t], x[.. + 2t + 8]) / 4^e(2t), b1 = (x[.. + 2t + 1], x[.. + 2t + 9]) / 4^e(2t+1)
  for (int it = threadIdx.x; it < NB * kb * 4; it += kThreads) {
    const int tok = it / (kb * 4), wr = it % (kb * 4);  // wr = word row k/16
    const int b = wr / 4, q = wr % 4;
    const __half *xr = reinterpret_cast<const __half *>(p.x) + static_cast<size_t>(tok) * K + 16 * wr;
    float xv[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) xv[e] = __half2float(xr[e]);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int j0 = 2 * t, j1 = 2 * t + 1;  // pair indices
      const float f0 = 1.f / static_cast<float>(1 << (2 * (j0 & 3))), f1 = 1.f / static_cast<float>(1 << (2 * (j1 & 3)));
      bfrag[((4 * b + t) * NB + tok) * 4 + q] =
          make_uint2(pack_half2(xv[j0] * f0, xv[j0 + 8] * f0), pack_half2(xv[j1] * f1, xv[j1 + 8] * f1));
    }
  }
  for (int it = threadIdx.x; it < NB * kg; it += kThreads) {
    const int tok = it / kg, gi = it % kg;
    const __half *xr = reinterpret_cast<const __half *>(p.x) + static_cast<size_t>(tok) * K + 128 * gi;
    float s = 0.f;
    for (int e = 0; e < 128; ++e) s += __half2float(xr[e]);
    xsum[tok * kg + gi] = s;
  }
  __syncthreads();

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane >> 2, q = lane & 3;
  const int kw = warp % p.ks, rtl = warp / p.ks;
  const int gpw = (kg + p.ks - 1) / p.ks;
  const int gb = kw * gpw, ge = min(kg, gb + gpw);
  const bool act = g < NB;
  const int t0 = 2 * q, t1 = 2 * q + 1;  // D columns (tokens) of this lane

  for (int rb = blockIdx.x; rb < p.nblocks; rb += gridDim.x) {
    const int n0 = (rb * p.rt + rtl) * 32;
    const int col = n0 + 4 * g;
    const bool valid = col < N;
    const uint32_t *wp = p.w + (valid ? col : 0) + static_cast<size_t>(q) * N;
    const __half *sp = p.s + (valid ? col : 0);
    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[0][i] = acc[1][i] = 0.f;

    for (int gr = gb; gr < ge; gr += kPrefetch) {
      uint4 wv[kPrefetch][2];
      float sc[kPrefetch][4];
#pragma unroll
      for (int i = 0; i < kPrefetch; ++i) {
        const int gg = gr + i;
        const bool ok = valid && gg < ge;
#pragma unroll
        for (int h = 0; h < 2; ++h)  // blocks 2gg and 2gg+1: word rows 4(2gg+h) + q
          wv[i][h] = ok ? ldg_stream_v4(wp + static_cast<size_t>(4 * (2 * gg + h)) * N) : make_uint4(0u, 0u, 0u, 0u);
        if (ok) {
          const uint2 sv = *reinterpret_cast<const uint2 *>(sp + static_cast<size_t>(gg) * N);
          const __half2 lo = *reinterpret_cast<const __half2 *>(&sv.x), hi = *reinterpret_cast<const __half2 *>(&sv.y);
          sc[i][0] = __low2float(lo);
          sc[i][1] = __high2float(lo);
          sc[i][2] = __low2float(hi);
          sc[i][3] = __high2float(hi);
        } else {
          sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < kPrefetch; ++i) {
        const int gg = gr + i;
        if (gg >= ge) break;
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t qx[8], qy[8], qz[8], qw[8];
          decode_t2(wv[i][h].x, qx);  // output col + 0: tile 0 row g
          decode_t2(wv[i][h].y, qy);  // col + 1: tile 0 row g + 8
          decode_t2(wv[i][h].z, qz);  // col + 2: tile 1 row g
          decode_t2(wv[i][h].w, qw);  // col + 3: tile 1 row g + 8
          const int b = 2 * gg + h;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint2 f = act ? bfrag[((4 * b + t) * NB + g) * 4 + q] : make_uint2(0u, 0u);
            mma_16816(d0, qx[2 * t], qy[2 * t], qx[2 * t + 1], qy[2 * t + 1], f.x, f.y);
            mma_16816(d1, qz[2 * t], qw[2 * t], qz[2 * t + 1], qw[2 * t + 1], f.x, f.y);
          }
        }
        // D: d[0] = (row g, col t0), d[1] = (row g, col t1), d[2] = (row g+8, col t0), d[3] = (row g+8, col t1)
        if (t0 < NB) {
          const float xs = xsum[t0 * kg + gg];
          acc[0][0] += sc[i][0] * fmaf(d0[0], 16777216.f, -xs);
          acc[0][1] += sc[i][1] * fmaf(d0[2], 16777216.f, -xs);
          acc[0][2] += sc[i][2] * fmaf(d1[0], 16777216.f, -xs);
          acc[0][3] += sc[i][3] * fmaf(d1[2], 16777216.f, -xs);
        }
        if (t1 < NB) {
          const float xs = xsum[t1 * kg + gg];
          acc[1][0] += sc[i][0] * fmaf(d0[1], 16777216.f, -xs);
          acc[1][1] += sc[i][1] * fmaf(d0[3], 16777216.f, -xs);
          acc[1][2] += sc[i][2] * fmaf(d1[1], 16777216.f, -xs);
          acc[1][3] += sc[i][3] * fmaf(d1[3], 16777216.f, -xs);
        }
      }
    }
    // Partials of this warp's K range into shared memory: red[kw][32 outputs][NB].
    const int rows = 32 * p.rt;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int tok = 2 * q + u;
      if (tok < NB) {
#pragma unroll
        for (int o = 0; o < 4; ++o) red[(kw * rows + rtl * 32 + 4 * g + o) * NB + tok] = acc[u][o];
      }
    }
    __syncthreads();
    for (int it = threadIdx.x; it < rows * NB; it += kThreads) {
      const int rl = it / NB, tok = it % NB;
      const int i = rb * rows + rl;
      if (i < N) {
        float v = 0.f;
        for (int w = 0; w < p.ks; ++w) v += red[(w * rows + rl) * NB + tok];
        p.y[static_cast<size_t>(tok) * N + i] = v;
      }
    }
    __syncthreads();
  }
}

template <int NB>
int launch(const TgemvParams &p, cudaStream_t stream, const DeviceInfo &dev) {
  const int kb = p.k / 64, kg = p.k / 128;
  const size_t smem = static_cast<size_t>(kb) * 4 * NB * 4 * sizeof(uint2) + static_cast<size_t>(NB) * kg * sizeof(float) +
                      static_cast<size_t>(kWarps) * 32 * NB * sizeof(float);
  MQ_REQUIRE(smem <= dev.smem_optin, MQ_EUNSUPPORTED, "mq_tgemv: k=%d batch=%d needs %zu B of shared memory (max %zu)", p.k,
             NB, smem, dev.smem_optin);
  auto kern = tgemv_kernel<NB>;
  static size_t configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(MQ_ECUDA, "mq_tgemv: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = smem;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1) return fail(MQ_ECUDA, "mq_tgemv: occupancy query failed (%s)", cudaGetErrorString(e));
  const int grid = std::min(p.nblocks, dev.sms * per_sm);
  kern<<<grid, kThreads, smem, stream>>>(p);
  return check_launch("mq_tgemv");
}

}  // namespace tg
}  // namespace mq

extern "C" int mq_tgemv(const uint16_t *x, const uint32_t *w, const uint16_t *s, float *y, int64_t n, int64_t k, int batch,
                        void *stream) {
  MQ_REQUIRE(x && w && s && y, MQ_EINVAL, "mq_tgemv: null pointer");
  MQ_REQUIRE(n > 0 && k > 0 && n < (1LL << 31) && k <= (1 << 20), MQ_EINVAL, "mq_tgemv: bad shape n=%lld k=%lld",
             static_cast<long long>(n), static_cast<long long>(k));
  MQ_REQUIRE(k % 128 == 0, MQ_EINVAL, "mq_tgemv: k=%lld must be a multiple of 128", static_cast<long long>(k));
  MQ_REQUIRE(n % 4 == 0, MQ_EINVAL, "mq_tgemv: n=%lld must be a multiple of 4", static_cast<long long>(n));
  MQ_REQUIRE(batch >= 1 && batch <= 4, MQ_EINVAL, "mq_tgemv: batch must be in 1..4 (got %d)", batch);
  MQ_REQUIRE(mq::aligned(w, 16) && mq::aligned(s, 8) && mq::aligned(x, 2) && mq::aligned(y, 4), MQ_EALIGN,
             "mq_tgemv: w must be 16-byte aligned, s 8-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  mq::tg::TgemvParams p{};
  p.x = x;
  p.w = w;
  p.s = reinterpret_cast<const __half *>(s);
  p.y = y;
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = batch;
  const int kg = static_cast<int>(k / 128);
  const int tiles = static_cast<int>((n + 31) / 32);
  const int target = dev.sms * 16;
  int ks = 1;
  while (ks < mq::tg::kWarps && static_cast<long>(tiles) * ks < target && ks * 2 <= kg) ks *= 2;
  p.ks = ks;
  p.rt = mq::tg::kWarps / ks;
  p.nblocks = (tiles + p.rt - 1) / p.rt;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (batch) {
    case 1: return mq::tg::launch<1>(p, st, dev);
    case 2: return mq::tg::launch<2>(p, st, dev);
    case 3: return mq::tg::launch<3>(p, st, dev);
    default: return mq::tg::launch<4>(p, st, dev);
  }
}
