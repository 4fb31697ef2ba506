// Ternary decode GEMV (mq_tgemv) over the transposed 2-bit layout, batch 1..4.
//
// Replaces packed_linear + packed_reduce (bonsai/kernels/kernels.mojo:283-325,437-448) and the
// product part of packed_head (:451-489): y[i] = sum over 128-k groups g of
// s[g][i] * sum_k (code(k, i) - 1) * x[k], code(k, i) = (w[(k/16) n + i] >> 2 (k % 16)) & 3.
// The reference accumulates each group in fp16 FMA chains (_group_dot8, :227-280); this kernel
// multiplies exactly (codes are small integers, x is fp16) and accumulates in fp32, so its error
// against exact arithmetic is far below the reference's own.
//
// B200 design (HBM-bound: 0.2656 B per weight, ~92 weights per SM clock at 6.5 TB/s, so the
// instructions per weight decide the speed):
//  * Streaming: each of 16 warps TMA-loads its own 32-output x 1024-k tiles of the [k/16][n]
//    word array (64 word rows of 128 bytes, 128-byte swizzle) and their [k/128][n] scales into a
//    private shared-memory ring and refills a slot as soon as it is consumed. Persistent CTAs,
//    one per SM.
//  * Decode: (w >> 2j) & 0x03030303 puts codes j, j + 4, j + 8, j + 12 of a word into the four
//    bytes of a register as int8 0..2: seven integer operations per 16 weights.
//  * Multiply: the warp-level int8 tensor op mma.m16n8k32 (s8 x s8 -> s32, exact). x is staged
//    per CTA as 15-bit fixed point per 128-k group, two int8 limbs hi * 256 + lo; the 8 mma
//    columns are (token, limb) pairs, so a lane ends a group holding one token's hi and lo sums for
//    its four outputs. The -1 offset of the codes is removed exactly with the group's integer limb
//    sums: sum (c - 1) x = sum c x - sum x. The fp32 epilogue applies scale_w * scale_x per group.
//  * Bank conflicts: lane (g, q) reads word row 4b + q and the 16-byte column chunk
//    (g >> 1) | (g & 1) << 2; with the swizzle's XOR by row % 8 the 8 lanes of a phase hit 8
//    distinct chunks.
//  * Head argmax (mq_tgemv_head): with the K split off, round r of a CTA is exactly the 512 outputs
//    of candidate block r. Each warp reduces its 32 outputs to (best, index, non-finite) with
//    shuffles and leaves them in shared memory; the warp that arrives last at the round's counter
//    combines the 16 and writes the candidate. No warp waits for another.
//  * Any width n. A TMA tensor map needs a row stride that is a multiple of 16 bytes, so n % 4 == 0
//    streams the slots with TMA; any other n (the reference's second head half has 151669 - 75776 =
//    75893 outputs, qwen3/model.mojo:176-181) fills the same swizzled slots with 4-byte cp.async
//    copies issued by all 32 lanes of the warp (zero-filled past n), completing on the same slot
//    barrier, so the consumer is unchanged. Outputs past n are never stored and never compete for
//    the argmax, as the reference's per-output tail (kernels.mojo:477-487) leaves them out.
//  * Non-finite x. The fixed-point staging cannot carry Inf or NaN, so a 128-k group of x holding one
//    gets a NaN scale: every output it touches becomes NaN. In the reference's fp32 arithmetic such an
//    output is Inf or NaN (x * w with x infinite is infinite or, for w = 0, NaN), so the outputs that
//    are not finite are the same, and the head's non-finite flag fires where the reference's does.
#include <algorithm>
#include <climits>
#include <cstring>

#include "common.cuh"

namespace mq {
namespace tg {

constexpr int kWarps = 16;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxSlots = 2;
constexpr int kCols = 32;                 // outputs of a tile (two m16 tiles)
// A slot holds 32 outputs x SK k: SK/16 word rows of 128 bytes and SK/128 scale rows of 64 bytes.
// SK = 1024 normally; 512 when x (2 bytes per k per token) leaves too little shared memory.
template <int SK>
struct Slot {
  static constexpr int kSlotK = SK;
  static constexpr int kWordRows = SK / 16;
  static constexpr int kWordBytes = kWordRows * 128;
  static constexpr int kGroups = SK / 128;
  static constexpr int kScaleBytes = kGroups * kCols * 2;
  static constexpr int kSlotBytes = ((kWordBytes + kScaleBytes + 1023) / 1024) * 1024;
};

struct Params {
  const uint16_t *x;
  const __half *s;
  float *y;
  int n, k, batch;
  int ks, rt, tiles, nrounds, slots, scales_tma;
  float *cand;      // head argmax candidates [batch][ncand][3], or null
  int ncand;        // ceil(n / 512)
  int cand_rounds;  // rounds of one CTA (shared-memory partials per round)
  int plain;        // 1: the lanes fill the slots with cp.async (n % 4 != 0: no tensor map of w)
  int y_vec;        // 1: a lane stores its 4 outputs as one float4 (n % 4 == 0, y 16-byte aligned)
  const uint32_t *w;  // the words, read directly when plain
};

constexpr int kCandOutputs = 512;   // outputs of a candidate block = one round of 16 warps x 32
constexpr int kMaxCandRounds = 8;   // rounds per CTA with candidates (n <= 8 * 512 * SMs)

constexpr float kLimbMax = 32512.f;  // 127 * 256: |x| maps to at most this, so both limbs fit in int8

// 4 bytes from global to shared memory, asynchronously; src_bytes = 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async4(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes) : "memory");
}
// Arrives on `bar` once this thread's earlier cp.async copies have landed (the barrier's expected
// count includes this arrival).
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint32_t pack_bytes(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 255u) | (static_cast<uint32_t>(b) & 255u) << 8 |
         (static_cast<uint32_t>(c) & 255u) << 16 | (static_cast<uint32_t>(d) & 255u) << 24;
}

// Shared memory: the rings; x as mma B fragments [k/32 steps][2 NB columns][4 lanes] (uint2); per
// (token, group) the x scale and the integer sums of the hi and lo limbs; K-split partials; barriers.
// With candidates: per (round, warp, token) the warp's (best value, index, non-finite, -) as int4,
// and one arrival counter per round.
struct Layout {
  uint32_t slots, bfrag, xs, lsum, red, cpart, ccnt, bars, total;
};

template <int SK>
__host__ __device__ inline Layout layout(int k, int nb, int slots, int cand_rounds) {
  Layout L;
  const int kg = k / 128;
  L.slots = 0;
  L.bfrag = kWarps * slots * Slot<SK>::kSlotBytes;
  L.xs = L.bfrag + (k / 32) * 2 * nb * 4 * 8;
  L.lsum = L.xs + nb * kg * 4;
  L.red = L.lsum + nb * kg * 2 * 4;
  L.cpart = (L.red + kWarps * kCols * nb * 4 + 15) / 16 * 16;
  L.ccnt = L.cpart + cand_rounds * kWarps * nb * 16;
  L.bars = (L.ccnt + cand_rounds * 4 + 7) / 8 * 8;
  L.total = L.bars + kWarps * kMaxSlots * 8;
  return L;
}

// (v, i) beats (bv, bi): larger value, or the same value at a lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// spread (whole outputs per warp, no candidate blocks, several rounds): round j of warp rtl covers
// tile (j * rt + rtl) * gridDim.x + blockIdx.x, so every CTA gets the same number of tiles within
// one (the 151936-output head: 4748 tiles are 32 or 33 per CTA, where whole rounds of 16 gave one
// CTA a third round while the others had finished two).
struct Items {
  int rtl, kw, spw, per_round, rt, tiles, grid, cta;
  bool spread;
  __device__ int tile_of(int j) const { return spread ? (j * rt + rtl) * grid + cta : (cta + j * grid) * rt + rtl; }
  __device__ bool get(uint32_t u, int &tile, int &sk) const {
    if (per_round <= 0) return false;
    const int j = static_cast<int>(u) / per_round, i = static_cast<int>(u) % per_round;
    tile = tile_of(j);
    sk = kw * spw + i;
    return tile < tiles;
  }
};

template <int NB, int SK>  // NB = batch (D columns used), SK = k of a slot
__global__ void __launch_bounds__(kThreads, 1)
    tgemv_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap, const Params p) {
  constexpr int kSlotK = Slot<SK>::kSlotK, kWordRows = Slot<SK>::kWordRows, kWordBytes = Slot<SK>::kWordBytes;
  constexpr int kGroups = Slot<SK>::kGroups, kScaleBytes = Slot<SK>::kScaleBytes, kSlotBytes = Slot<SK>::kSlotBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const Layout L = layout<SK>(p.k, NB, p.slots, p.cand_rounds);
  const int K = p.k, N = p.n, S = p.slots;
  const int kg = K / 128;
  const int nslotk = (K + kSlotK - 1) / kSlotK;
  const int spw = (nslotk + p.ks - 1) / p.ks;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars) + warp * kMaxSlots;
  uint8_t *ring = smem + L.slots + warp * S * kSlotBytes;
  const uint32_t bytes = kWordBytes + (p.scales_tma ? kScaleBytes : 0);

  Items items;
  items.rtl = warp / p.ks;
  items.kw = warp % p.ks;
  items.spw = spw;
  items.per_round = min(spw, nslotk - items.kw * spw);
  items.rt = p.rt;
  items.tiles = p.tiles;
  items.grid = gridDim.x;
  items.cta = blockIdx.x;
  items.spread = !p.cand && p.ks == 1 && p.nrounds > static_cast<int>(gridDim.x);

  auto issue = [&](uint32_t u) {
    int tile, sk;
    if ((lane != 0 && !p.plain) || !items.get(u, tile, sk)) return;
    const int slot = u % S;
    uint64_t *bar = full + slot;
    uint8_t *dst = ring + slot * kSlotBytes;
    if (p.plain) {  // lane l copies column tile * 32 + l of each word row into its swizzled place
      const int col = tile * kCols + lane, row0 = sk * kWordRows, nrows = K / 16;
      const bool in = col < N;
      const uint32_t *src = p.w + (in ? col : 0);
      uint8_t *d0 = dst + (lane & 3) * 4;
#pragma unroll 8
      for (int wr = 0; wr < kWordRows; ++wr) {
        const bool live = in && row0 + wr < nrows;
        cp_async4(d0 + wr * 128 + (((lane >> 2) ^ (wr & 7)) << 4), live ? src + static_cast<size_t>(row0 + wr) * N : p.w,
                  live ? 4u : 0u);
      }
      cp_async_arrive(bar);
      return;
    }
    mbar_expect_tx(bar, bytes);
    tma_load_2d(dst, &wmap, bar, tile * kCols, sk * kWordRows);
    if (p.scales_tma) tma_load_2d(dst + kWordBytes, &smap, bar, tile * kCols, sk * kGroups);
  };
  griddep_launch_dependents();
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(full + s, p.plain ? 32 : 1);
    fence_mbar_init();
    if (!p.plain) prefetch_tmap(&wmap);
    if (p.scales_tma) prefetch_tmap(&smap);
  }
  __syncwarp();
  // In a launch of one round per CTA (latency-bound) the first S weight tiles of each warp go out before the dependency
  // wait: the only kernels that let this one start before they finish (this library's GEMV, GEMM, MoE and exchange
  // kernels) write outputs and scratch, never weights, and any other kernel finishes before this one starts, so the
  // weights are final (12288 x 4096: 7.6 -> 7.0 us). Multi-round launches (the head) keep the loads after the staging,
  // which measured faster there.
  const bool pre = p.nrounds <= static_cast<int>(gridDim.x);
  if (pre)
    for (int s = 0; s < S; ++s) issue(s);
  griddep_wait();  // everything above only read weights

  uint2 *bfrag = reinterpret_cast<uint2 *>(smem + L.bfrag);  // [K/32 steps][2 NB][4]
  float *xs = reinterpret_cast<float *>(smem + L.xs);         // [NB][kg]
  int *lsum = reinterpret_cast<int *>(smem + L.lsum);         // [NB][kg][hi, lo]
  float *red = reinterpret_cast<float *>(smem + L.red);       // [kWarps][32][NB]
  int4 *cpart = reinterpret_cast<int4 *>(smem + L.cpart);     // [cand_rounds][kWarps][NB]
  int *ccnt = reinterpret_cast<int *>(smem + L.ccnt);         // [cand_rounds]
  for (int i = threadIdx.x; i < p.cand_rounds; i += kThreads) ccnt[i] = 0;  // visible after the staging barrier

  // Stage x: item (token t, word row wr) = x[16 wr .. 16 wr + 15]; the 8 items of a group are 8
  // consecutive lanes, which share its scale and limb sums. For step 2b + h (word rows 4b .. 4b + 3,
  // codes h * 2 + 4i and h * 2 + 1 + 4i) lane q' of column 2t + l holds limb l of x at those codes of
  // word row 4b + q'.
  const int nrow = K / 16;
  // Without the early loads: warps with no staging item issue their first loads now (they would only
  // wait at the staging barrier); the others after it, so that lane 0's TMA holds do not delay the
  // barrier. When every warp stages (long K), all issue now: the loads then cover the longer staging.
  const bool early = 32 * warp >= NB * nrow || NB * nrow >= kThreads;
  if (!pre && early)
    for (int s = 0; s < S; ++s) issue(s);
  for (int base = 0; base < NB * nrow; base += kThreads) {
    const int it = base + threadIdx.x;
    const bool live = it < NB * nrow;
    const int t = live ? it / nrow : 0, wr = it % nrow;
    float xv[16];
    if (live) {
      const uint4 *xr = reinterpret_cast<const uint4 *>(p.x + static_cast<size_t>(t) * K + 16 * wr);
      const uint4 v0 = xr[0], v1 = xr[1];
      const __half *h0 = reinterpret_cast<const __half *>(&v0), *h1 = reinterpret_cast<const __half *>(&v1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        xv[e] = __half2float(h0[e]);
        xv[8 + e] = __half2float(h1[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) xv[e] = 0.f;
    }
    float m = 0.f;
    int bad = 0;  // a non-finite x in the group: its scale becomes NaN
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      m = fmaxf(m, fabsf(xv[e]));
      bad |= !isfinite(xv[e]);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    const float inv = m > 0.f && !bad ? kLimbMax / m : 0.f;
    int hi[16], lo[16], shi = 0, slo = 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int v = static_cast<int>(rintf(xv[e] * inv));
      hi[e] = (v + 128) >> 8;
      lo[e] = v - (hi[e] << 8);
      shi += hi[e];
      slo += lo[e];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      shi += __shfl_xor_sync(0xffffffffu, shi, o);
      slo += __shfl_xor_sync(0xffffffffu, slo, o);
    }
    if (!live) continue;
    const int gg = wr / 8;
    if (wr % 8 == 0) {
      xs[t * kg + gg] = bad ? __int_as_float(0x7fc00000) : m / kLimbMax;
      lsum[(t * kg + gg) * 2] = shi;
      lsum[(t * kg + gg) * 2 + 1] = slo;
    }
    const int b = wr / 4, q = wr % 4;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint2 *dst = bfrag + ((2 * b + h) * 2 * NB + 2 * t) * 4 + q;
      dst[0] = make_uint2(pack_bytes(hi[2 * h], hi[2 * h + 4], hi[2 * h + 8], hi[2 * h + 12]),
                          pack_bytes(hi[2 * h + 1], hi[2 * h + 5], hi[2 * h + 9], hi[2 * h + 13]));
      dst[4] = make_uint2(pack_bytes(lo[2 * h], lo[2 * h + 4], lo[2 * h + 8], lo[2 * h + 12]),
                          pack_bytes(lo[2 * h + 1], lo[2 * h + 5], lo[2 * h + 9], lo[2 * h + 13]));
    }
  }
  __syncthreads();

  if (!pre && !early)
    for (int s = 0; s < S; ++s) issue(s);

  const int g = lane >> 2, q = lane & 3;
  const bool act = g < 2 * NB;                // columns (token g / 2, limb g % 2) in use
  const int cgc = (g >> 1) | ((g & 1) << 2);  // this lane's 16-byte column chunk: outputs 4 cgc .. + 3
  constexpr uint32_t kCode = 0x03030303u;
  uint32_t u = 0, u_abort = 0;
  bool aborted = false;

  int jr = 0;  // this CTA's round count
  for (int r = blockIdx.x; items.spread ? items.tile_of(jr) - items.rtl * static_cast<int>(gridDim.x) < p.tiles
                                         : r < p.nrounds;
       r += gridDim.x, ++jr) {
    const int tile = items.tile_of(jr);
    const int col = tile * kCols + 4 * cgc;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // token q, outputs col .. col + 3
    if (tile < p.tiles) {
      for (int i = 0; i < items.per_round; ++i, ++u) {
        const int sk = items.kw * spw + i;
        const uint32_t slot = u % S;
        if (!aborted && !mbar_wait(&full[slot], (u / S) & 1)) {
          raise_status(kStatusGemvConsumerWait);
          aborted = true;
          u_abort = u;
        }
        const uint8_t *sb = ring + slot * kSlotBytes;
        const int ngr = min(kGroups, kg - sk * kGroups);
        if (!aborted) {
#pragma unroll  // all groups of the slot: their decode, MMA and epilogue chains interleave (+5%)
          for (int gi = 0; gi < kGroups; ++gi) {
            if (gi >= ngr) break;
            const int gg = sk * kGroups + gi;  // global group
            float sc[4];
            if (p.scales_tma) {
              const uint2 sv = *reinterpret_cast<const uint2 *>(sb + kWordBytes + gi * kCols * 2 + cgc * 8);
              const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&sv.x));
              const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&sv.y));
              sc[0] = a.x, sc[1] = a.y, sc[2] = b.x, sc[3] = b.y;
            } else {
#pragma unroll
              for (int o = 0; o < 4; ++o)
                sc[o] = col + o < N ? __half2float(p.s[static_cast<size_t>(gg) * N + col + o]) : 0.f;
            }
            int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};  // tile 0 (outputs col, col + 1), tile 1 (col + 2, col + 3)
#pragma unroll
            for (int bh = 0; bh < 2; ++bh) {
              const int b = 2 * gi + bh, wr = 4 * b + q;
              const uint4 wv = *reinterpret_cast<const uint4 *>(sb + wr * 128 + ((cgc ^ (wr & 7)) << 4));
              const int bg = sk * (kSlotK / 64) + b;  // global block of 4 word rows
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                uint2 f = make_uint2(0u, 0u);
                if (act) f = bfrag[((2 * bg + h) * 2 * NB + g) * 4 + q];
                const int j0 = 4 * h, j1 = 4 * h + 2;  // shifts of codes 2h + 4i and 2h + 1 + 4i
                mma_s8_16832(d0, (wv.x >> j0) & kCode, (wv.y >> j0) & kCode, (wv.x >> j1) & kCode, (wv.y >> j1) & kCode,
                             f.x, f.y);
                mma_s8_16832(d1, (wv.z >> j0) & kCode, (wv.w >> j0) & kCode, (wv.z >> j1) & kCode, (wv.w >> j1) & kCode,
                             f.x, f.y);
              }
            }
            // D: [0] = (output row g, hi), [1] = (row g, lo), [2] = (row g + 8, hi), [3] = (row g + 8, lo) of token q
            if (q < NB) {
              const float xsc = xs[q * kg + gg];
              const int shi = lsum[(q * kg + gg) * 2], slo = lsum[(q * kg + gg) * 2 + 1];
              const int r0 = (d0[0] - shi) * 256 + (d0[1] - slo), r1 = (d0[2] - shi) * 256 + (d0[3] - slo);
              const int r2 = (d1[0] - shi) * 256 + (d1[1] - slo), r3 = (d1[2] - shi) * 256 + (d1[3] - slo);
              acc[0] = fmaf(sc[0] * xsc, static_cast<float>(r0), acc[0]);
              acc[1] = fmaf(sc[1] * xsc, static_cast<float>(r1), acc[1]);
              acc[2] = fmaf(sc[2] * xsc, static_cast<float>(r2), acc[2]);
              acc[3] = fmaf(sc[3] * xsc, static_cast<float>(r3), acc[3]);
            }
          }
        }
        __syncwarp();
        if (!aborted) issue(u + S);
      }
    }
    const int rows = kCols * p.rt;
    if (q < NB) {
      if (p.ks == 1) {  // the warp owns whole outputs: store directly, no barrier
        if (tile < p.tiles && col < N && !aborted) {
          float *out = p.y + static_cast<size_t>(q) * N + col;
          if (p.y_vec) {
            *reinterpret_cast<float4 *>(out) = make_float4(acc[0], acc[1], acc[2], acc[3]);
          } else {
#pragma unroll
            for (int o = 0; o < 4; ++o)
              if (col + o < N) out[o] = acc[o];
          }
        }
      } else {
#pragma unroll
        for (int o = 0; o < 4; ++o) red[(items.kw * rows + items.rtl * kCols + 4 * cgc + o) * NB + q] = acc[o];
      }
    }
    if (p.cand) {  // ks == 1: this round is candidate block r, this warp its outputs 32 * warp ..
      float bv = -INFINITY;
      int bi = INT_MAX, bad = 0;
      if (q < NB && tile < p.tiles) {
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          if (col + o >= N) break;  // only real outputs compete
          bad |= !isfinite(acc[o]);
          if (better(acc[o], col + o, bv, bi)) bv = acc[o], bi = col + o;
        }
      }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {  // the 8 lanes of token q
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
      }
      if (lane < NB) {
        cpart[(jr * kWarps + warp) * NB + lane] = make_int4(__float_as_int(bv), bi, bad, 0);
        __threadfence_block();
      }
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&ccnt[jr], 1) == kWarps - 1;
      if (__shfl_sync(0xffffffffu, last, 0)) {  // every warp's partial of this round is in place
        __threadfence_block();
        if (lane < NB) {
          float cv = -INFINITY;
          int ci = INT_MAX, cbad = 0;
          for (int w = 0; w < kWarps; ++w) {  // warps in output order
            const int4 e = cpart[(jr * kWarps + w) * NB + lane];
            cbad |= e.z;
            if (better(__int_as_float(e.x), e.y, cv, ci)) cv = __int_as_float(e.x), ci = e.y;
          }
          float *c = p.cand + (static_cast<size_t>(lane) * p.ncand + r) * 3;
          c[0] = cv;
          c[1] = static_cast<float>(ci);
          c[2] = cbad ? 1.f : 0.f;
        }
      }
    }
    if (p.ks == 1) continue;
    __syncthreads();
    for (int it = threadIdx.x; it < rows * NB; it += kThreads) {
      const int rl = it / NB, tok = it % NB;
      const int i = r * rows + rl;
      if (i < N) {
        float v = 0.f;
        for (int w = 0; w < p.ks; ++w) v += red[(w * rows + rl) * NB + tok];
        p.y[static_cast<size_t>(tok) * N + i] = v;
      }
    }
    __syncthreads();
  }
  if (lane == 0 && aborted) {
    for (uint32_t v = u_abort; v < u_abort + S; ++v) {
      int tile, sk;
      if (items.get(v, tile, sk)) mbar_wait(&full[v % S], (v / S) & 1);
    }
  }
}

template <int NB, int SK>
int launch_sk(const uint32_t *w, Params p, cudaStream_t stream, const DeviceInfo &dev) {
  using Sl = Slot<SK>;
  const int nslotk = (p.k + SK - 1) / SK;
  int ks = 1;  // with candidates a round must be a whole 512-output block: no K split
  while (!p.cand && ks < kWarps && ks < nslotk && (p.tiles * ks + kWarps - 1) / kWarps < dev.sms) ks *= 2;
  p.ks = ks;
  p.rt = kWarps / ks;
  p.nrounds = (p.tiles + p.rt - 1) / p.rt;
  const int grid = std::min(p.nrounds, dev.sms);
  p.cand_rounds = p.cand ? (p.nrounds + grid - 1) / grid : 0;
  MQ_REQUIRE(p.cand_rounds <= kMaxCandRounds, MQ_EINVAL, "mq_tgemv_head: n=%d exceeds %d outputs on this device", p.n,
             kMaxCandRounds * kCandOutputs * dev.sms);
  Layout L{};
  for (p.slots = kMaxSlots; p.slots >= 1; --p.slots) {
    L = layout<SK>(p.k, NB, p.slots, p.cand_rounds);
    if (L.total + 1024 <= dev.smem_optin) break;
  }
  const size_t smem = L.total + 1024;
  MQ_REQUIRE(smem <= dev.smem_optin, MQ_EUNSUPPORTED, "mq_tgemv: k=%d batch=%d needs %zu B of shared memory (max %zu)", p.k,
             NB, smem, dev.smem_optin);
  CUtensorMap wmap, smap;
  p.plain = p.n % 4 != 0;  // the row stride n * 4 bytes is not a multiple of 16: no tensor map
  p.w = w;
  if (p.plain) {
    memset(&wmap, 0, sizeof(wmap));  // not read
  } else if (int rc = encode_tmap_2d(&wmap, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.n, p.k / 16,
                                     static_cast<uint64_t>(p.n) * 4, kCols, Sl::kWordRows, CU_TENSOR_MAP_SWIZZLE_128B,
                                     "mq_tgemv words")) {
    return rc;
  }
  p.y_vec = p.n % 4 == 0 && aligned(p.y, 16);
  p.scales_tma = p.n % 8 == 0 && aligned(p.s, 16);
  if (p.scales_tma) {
    if (int rc = encode_tmap_2d(&smap, p.s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.n, p.k / 128,
                                static_cast<uint64_t>(p.n) * 2, kCols, Sl::kGroups, CU_TENSOR_MAP_SWIZZLE_NONE,
                                "mq_tgemv scales"))
      return rc;
  } else {
    smap = wmap;  // not read
  }
  auto kern = tgemv_kernel<NB, SK>;
  static size_t configured[64] = {};
  if (int rc = ensure_smem(kern, smem, configured, "mq_tgemv")) return rc;
  return launch_overlapped(kern, dim3(grid), dim3(kThreads), smem, stream, "mq_tgemv", wmap, smap, p);
}

template <int NB>
int launch(const uint32_t *w, Params p, cudaStream_t stream, const DeviceInfo &dev) {
  const Layout big = layout<1024>(p.k, NB, 1, p.cand ? kMaxCandRounds : 0);
  if (big.total + 1024 <= dev.smem_optin) return launch_sk<NB, 1024>(w, p, stream, dev);
  return launch_sk<NB, 512>(w, p, stream, dev);
}

}  // namespace tg
}  // namespace mq

namespace mq {
namespace tg {

int tgemv_run(const uint16_t *x, const uint32_t *w, const uint16_t *s, float *y, float *cand, int64_t n, int64_t k,
              int batch, cudaStream_t st) {
  MQ_REQUIRE(x && w && s && y, MQ_EINVAL, "mq_tgemv: null pointer");
  MQ_REQUIRE(n > 0 && k > 0 && n < (1LL << 31) && k <= (1 << 20), MQ_EINVAL, "mq_tgemv: bad shape n=%lld k=%lld",
             static_cast<long long>(n), static_cast<long long>(k));
  MQ_REQUIRE(k % 128 == 0, MQ_EINVAL, "mq_tgemv: k=%lld must be a multiple of 128", static_cast<long long>(k));
  MQ_REQUIRE(batch >= 1 && batch <= 4, MQ_EINVAL, "mq_tgemv: batch must be in 1..4 (got %d)", batch);
  MQ_REQUIRE(mq::aligned(w, 16) && mq::aligned(s, 2) && mq::aligned(x, 16) && mq::aligned(y, 4) && mq::aligned(cand, 4),
             MQ_EALIGN, "mq_tgemv: w and x must be 16-byte aligned, s 2-byte and y 4-byte aligned");
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  Params p{};
  p.x = x;
  p.s = reinterpret_cast<const __half *>(s);
  p.y = y;
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = batch;
  p.tiles = static_cast<int>((n + kCols - 1) / kCols);
  p.cand = cand;
  p.ncand = static_cast<int>((n + kCandOutputs - 1) / kCandOutputs);
  switch (batch) {
    case 1: return launch<1>(w, p, st, dev);
    case 2: return launch<2>(w, p, st, dev);
    case 3: return launch<3>(w, p, st, dev);
    default: return launch<4>(w, p, st, dev);
  }
}

// index[b] = the best candidate of token b (lowest index among equal values), -1 if any is flagged.
__global__ void head_argmax_kernel(const float *__restrict__ cand, int ncand, int32_t *__restrict__ index) {
  __shared__ float sv[32];
  __shared__ int si[32], sb[32];
  const float *c = cand + static_cast<size_t>(blockIdx.x) * ncand * 3;
  float bv = -INFINITY;
  int bi = INT_MAX, bad = 0;
  for (int j = threadIdx.x; j < ncand; j += blockDim.x) {
    const float v = c[3 * j];
    const int i = static_cast<int>(c[3 * j + 1]);
    bad |= c[3 * j + 2] != 0.f;
    if (better(v, i, bv, bi)) bv = v, bi = i;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  if (lane == 0) sv[warp] = bv, si[warp] = bi, sb[warp] = bad;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w) {
      bad |= sb[w];
      if (better(sv[w], si[w], bv, bi)) bv = sv[w], bi = si[w];
    }
    index[blockIdx.x] = bad ? -1 : bi;
  }
}

}  // namespace tg
}  // namespace mq

extern "C" int mq_tgemv(const uint16_t *x, const uint32_t *w, const uint16_t *s, float *y, int64_t n, int64_t k, int batch,
                        void *stream) {
  return mq::tg::tgemv_run(x, w, s, y, nullptr, n, k, batch, static_cast<cudaStream_t>(stream));
}

extern "C" int mq_tgemv_head(const uint16_t *x, const uint32_t *w, const uint16_t *s, float *y, float *candidates,
                             int64_t n, int64_t k, int batch, void *stream) {
  MQ_REQUIRE(candidates, MQ_EINVAL, "mq_tgemv_head: null candidates");
  return mq::tg::tgemv_run(x, w, s, y, candidates, n, k, batch, static_cast<cudaStream_t>(stream));
}

extern "C" int mq_head_argmax(const float *candidates, int64_t ncand, int batch, int32_t *index, void *stream) {
  MQ_REQUIRE(candidates && index, MQ_EINVAL, "mq_head_argmax: null pointer");
  MQ_REQUIRE(ncand >= 1 && ncand < (1LL << 24) && batch >= 1 && batch <= 65535, MQ_EINVAL,
             "mq_head_argmax: bad ncand=%lld or batch=%d", static_cast<long long>(ncand), batch);
  MQ_REQUIRE(mq::aligned(candidates, 4) && mq::aligned(index, 4), MQ_EALIGN, "mq_head_argmax: misaligned pointer");
  mq::tg::head_argmax_kernel<<<batch, 256, 0, static_cast<cudaStream_t>(stream)>>>(candidates, static_cast<int>(ncand),
                                                                                  index);
  return mq::check_launch("mq_head_argmax");
}
