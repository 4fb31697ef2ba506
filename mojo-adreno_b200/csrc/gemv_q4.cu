// Decode GEMV over int4 word-layout weights (mq_gemv_q4), batch 1..4.
//
// Replaces gemv_q4 / gemv_add_q4 (llama/kernels/gemv_q4.mojo:13-30, gemv_add_q4.mojo:13-30), the
// Q4_0 G=32 variant (lfm2/kernels/lk.mojo:56-72,134-143) and the small-batch t_gemv_q4 / p_gemv_q4
// (qwen3moe/kernels/moek.mojo:273-281,528-545). Same arithmetic: y[r] = sum over groups of
// scale * sum_j ((nib_j ^ 8) - 8) * x[k_j], fp32 x and y.
//
// B200 design (HBM-bound: 0.5625 B per weight at G=32):
//  * Streaming. Each of 16 warps streams its own 32-row x 256-k weight tiles (4 KB, one TMA box of
//    32 rows x 128 bytes with the 128-byte swizzle) and their fp16 scales from HBM into a private
//    2-slot shared-memory ring (cp.async.bulk.tensor), refilling a slot as soon as it is consumed:
//    no hand-off between warps. Persistent CTAs, one per SM.
//  * Issue budget. At ~6.5 TB/s an SM must retire ~46 weights per clock, so the instructions per
//    packed word decide the speed. The products run on the warp-level int8 tensor op
//    mma.m16n8k32 (s8 x s8 -> s32, exact): a stored nibble is the 4-bit two's complement of its
//    value, so a nibble masked into the high half of a byte is the int8 16 * value. Per 32-bit word
//    (w << 4) & 0xF0F0F0F0 and w & 0xF0F0F0F0 give the even and the odd elements: three integer
//    operations for eight weights, no offset term. One mma covers two words per lane.
//  * Activations. x is staged once per CTA as 15-bit fixed point per 32-k group (scale
//    max|x| / 32512), split into two int8 limbs hi * 256 + lo (balanced, both in range); the
//    products are exact integers, and the fp32 epilogue applies scale_x * scale_w / 16 per group.
//    The x quantisation step is 1/65024 of the group's largest |x|.
//  * Exact per-group scales. The four lanes of a quad (lane % 4 == q) read 16 consecutive bytes of
//    a row (32 weights = one G=32 group). The B fragment puts quad q's x limbs in columns 2q (hi)
//    and 2q + 1 (lo) only, so the lane that owns columns 2q, 2q + 1 holds exactly its own group's
//    two limb sums and combines them without a shuffle.
//  * Bank conflicts. The 128-byte TMA swizzle XORs a row's 16-byte chunk index with row % 8; mma row
//    g reads physical row (g >> 1) | (g & 1) << 2, which puts the 8 lanes of every shared-memory
//    phase on 8 different chunks.
//  * Small matrices split K across the warps of a CTA (partials reduced in shared memory), so even
//    a 2048-row matrix keeps every SM streaming.
//  * Non-finite x. The fixed-point staging cannot carry Inf or NaN, so a 32-k group of x holding one
//    gets a NaN scale and every output it touches becomes NaN. In the reference's fp32 arithmetic
//    such an output is Inf or NaN (an infinite x times a weight is infinite, or NaN for weight 0), so
//    the same outputs are not finite.
#include <algorithm>

#include "common.cuh"

namespace mq {
namespace gemv {

constexpr int kWarps = 16;  // 4 per scheduler
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxSlots = 2;
constexpr int kRows = 32;     // rows of a tile: two m16 tiles
constexpr int kSlotK = 256;   // k of a slot: 32 words = one 128-byte swizzle row
constexpr int kWordBytes = kRows * 128;
constexpr int kScaleHalvesTma = 8;  // a TMA-loaded scale row: 8 halves (16 bytes), G = 32 only
constexpr int kPrefetchItems = 4;  // items per warp warmed in L2 while earlier kernels finish
constexpr float kLimbMax = 32512.f;  // 127 * 256: |x| maps to at most this, so both limbs fit in int8

struct Params {
  const __half *ws;  // scales in global memory (read directly when they are not TMA-loaded)
  const void *x;
  float *y;
  int n, k, batch, x_f16, add;  // batch: staged x vectors (tokens, or expert slots with xpg)
  int ks;       // warps that split a tile's K range (1 = no reduction between warps)
  int rt;       // tiles per round (rt * ks == kWarps)
  int tiles;    // ceil(n / 32)
  int nrounds;  // ceil(tiles / rt)
  int slots;    // ring slots per warp (<= kMaxSlots)
  int scales_tma;
  int slot_bytes;
  // Expert indirection (MoE decode): output tile t reads weight rows ids[t / tpg] * group_rows +
  // (t % tpg) * 32 ..; with xpg each expert slot t / tpg has its own x vector (staged as token t / tpg).
  const int32_t *ids;
  int group_rows, tpg, xpg;
  int wrows;  // rows of the weight matrix (== n without expert indirection)
  // Gate|up with the SwiGLU fused (gu != 0): a tile is 16 outputs j; slot rows 0..15 hold the gate
  // rows of those outputs, rows 16..31 the up rows, gu_off rows further down the matrix, and the
  // output is silu(gate . x) * (up . x). The maps are then 3-D (words, rows, gate/up plane gu_off
  // rows apart), so one box still fetches a whole slot.
  int gu, gu_off;
  // Device gate (expert-parallel owners): when *gate > gate_max the launch does nothing (another path
  // of the layer has the work).
  const int32_t *gate;
  int gate_max;
};

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

// First weight row of output tile `tile` (the rows themselves, or an expert's rows through ids).
// An expert id past the weight matrix is reported and read as expert 0; a negative id ("no expert",
// the padding of a fixed-capacity exchange) loads nothing (issue skips the tile) and its outputs are
// left unspecified.
__device__ __forceinline__ int weight_row0(const Params &p, int tile) {
  const int tr = p.gu ? kRows / 2 : kRows;  // weight rows (of one kind) per output tile
  if (!p.ids) return tile * tr;
  int e = __ldg(p.ids + tile / p.tpg);
  if (e >= p.wrows / p.group_rows) {
    raise_status(kStatusMoeBadExpertId);
    e = 0;
  } else if (e < 0) {
    e = 0;
  }
  return e * p.group_rows + (tile % p.tpg) * tr;
}

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

// Physical row (within 8) that mma row g reads: keeps the 8 lanes of a phase on distinct chunks.
__device__ __forceinline__ int phys_row(int g) { return (g >> 1) | ((g & 1) << 2); }

// Shared-memory layout (byte offsets from a 1024-aligned base): the weight rings, the staged x as
// mma B fragments [nt][kc * 4 steps][8 columns] (uint2 each), the x scales [nt][kc * 4 groups], the
// K-split partials and the ring barriers.
struct Layout {
  uint32_t slots, bfrag, xs, red, bars, total;
};

__host__ __device__ inline Layout layout(int k, int batch, int nt, int slots, int slot_bytes) {
  Layout L;
  const int kc = (k + 127) / 128;
  L.slots = 0;
  L.bfrag = kWarps * slots * slot_bytes;
  L.xs = L.bfrag + nt * kc * 4 * 8 * 8;
  L.red = (L.xs + nt * kc * 4 * 4 + 15) / 16 * 16;
  L.bars = (L.red + kWarps * kRows * batch * 4 + 7) / 8 * 8;
  L.total = L.bars + kWarps * kMaxSlots * 8;
  return L;
}

__device__ __forceinline__ uint32_t pack_bytes(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 255u) | (static_cast<uint32_t>(b) & 255u) << 8 |
         (static_cast<uint32_t>(c) & 255u) << 16 | (static_cast<uint32_t>(d) & 255u) << 24;
}

// The work of one warp, as a sequence of (tile, slot of K) items: round j of this CTA covers
// tile (blockIdx.x + j * gridDim.x) * rt + rtl, K slots kw * spw .. + per_round - 1. With spread
// (whole rows per warp, several rounds) tiles are dealt to the warps across the CTAs instead:
// round j of warp rtl covers tile (j * rt + rtl) * gridDim.x + blockIdx.x, so every CTA gets the
// same number of tiles within one (4008 lm_head tiles: 27 or 28 per CTA, where whole rounds of 16
// gave 103 CTAs 32 and 45 CTAs 16, leaving a third of the SMs idle in the second round).
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

template <int G, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_q4_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int K = p.k, N = p.n, B = p.batch, S = p.slots;
  const int nt = p.xpg ? B : NT;  // x vectors staged
  const Layout L = layout(K, B, nt, S, p.slot_bytes);
  const int kc = (K + 127) / 128;
  const int nsteps = kc * 4;
  const int nslotk = (K + kSlotK - 1) / kSlotK;
  const int spw = (nslotk + p.ks - 1) / p.ks;  // K slots per warp per round
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars) + warp * kMaxSlots;
  uint8_t *ring = smem + L.slots + warp * S * p.slot_bytes;
  const uint32_t bytes = kWordBytes + (p.scales_tma ? kRows * kScaleHalvesTma * 2 : 0);

  Items items;
  items.rtl = warp / p.ks;
  items.kw = warp % p.ks;
  items.spw = spw;
  items.per_round = min(spw, nslotk - items.kw * spw);
  items.rt = p.rt;
  items.tiles = p.tiles;
  items.grid = gridDim.x;
  items.cta = blockIdx.x;
  items.spread = p.ks == 1 && p.nrounds > static_cast<int>(gridDim.x);

  // Each warp streams its own tiles: lane 0 issues the TMA loads for the next S items.
  auto issue = [&](uint32_t u) {
    int tile, sk;
    if (lane != 0 || !items.get(u, tile, sk)) return;
    const int slot = u % S;
    uint64_t *bar = full + slot;
    uint8_t *dst = ring + slot * p.slot_bytes;
    if (p.ids && __ldg(p.ids + tile / p.tpg) < 0) {  // an empty slot ("no expert"): nothing to read; its outputs are unused
      mbar_arrive(bar);
      return;
    }
    const int wrow = weight_row0(p, tile);
    mbar_expect_tx(bar, bytes);
    if (p.gu) {  // [2 planes][16 rows]: the gate rows into slot rows 0..15, the up rows into 16..31
      tma_load_3d(dst, &wmap, bar, sk * (kSlotK / 8), wrow, 0);
      if (p.scales_tma) tma_load_3d(dst + kWordBytes, &smap, bar, sk * kScaleHalvesTma, wrow, 0);
    } else {
      tma_load_2d(dst, &wmap, bar, sk * (kSlotK / 8), wrow);
      if (p.scales_tma) tma_load_2d(dst + kWordBytes, &smap, bar, sk * kScaleHalvesTma, wrow);
    }
  };
  griddep_launch_dependents();
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(full + s, 1);
    fence_mbar_init();
    prefetch_tmap(&wmap);
    if (p.scales_tma) prefetch_tmap(&smap);
  }
  __syncwarp();
  // In a launch of one round per CTA (a small matrix, latency-bound) the first S weight tiles of each warp go out
  // before the dependency wait: the only kernels that let this one start before they finish (this library's GEMV, GEMM,
  // MoE and exchange kernels) write outputs and scratch, never weights, and any other kernel finishes before this one
  // starts, so the weights are final. Not with expert ids (written by earlier kernels) or a device gate (the launch may
  // exit before consuming them), and not in multi-round launches, where it measured slower (lm_head: 27.4 -> 28.8 us;
  // qkv 3072 x 2048: 4.4 -> 4.2 us).
  const bool pre = !p.ids && !p.gate && p.nrounds <= static_cast<int>(gridDim.x);
  if (pre)
    for (int s = 0; s < S; ++s) issue(s);
  // Until the kernels before this one finish, warm L2 with this warp's next items (lane i: item i).
  if (pre && lane >= S && lane < kPrefetchItems) {
    int tile, sk;
    if (items.get(lane, tile, sk)) {
      const int wrow = weight_row0(p, tile);
      if (p.gu) {
        tma_prefetch_l2_3d(&wmap, sk * (kSlotK / 8), wrow, 0);
        if (p.scales_tma) tma_prefetch_l2_3d(&smap, sk * kScaleHalvesTma, wrow, 0);
      } else {
        tma_prefetch_l2_2d(&wmap, sk * (kSlotK / 8), wrow);
        if (p.scales_tma) tma_prefetch_l2_2d(&smap, sk * kScaleHalvesTma, wrow);
      }
    }
  }
  // x, too (every CTA reads all of it): if earlier kernels write it, their writes still land in L2,
  // the point of coherence, before griddep_wait returns.
  if (threadIdx.x == 32 * (kWarps - 1)) {
    const size_t xbytes = static_cast<size_t>(p.batch) * K * (p.x_f16 ? 2 : 4);
    for (size_t off = 0; off < xbytes; off += 65536)
      prefetch_l2_bulk(static_cast<const uint8_t *>(p.x) + off, static_cast<uint32_t>(min(xbytes - off, size_t(65536))));
  }
  griddep_wait();  // everything above wrote no global memory
  if (p.gate && __ldg(p.gate) > p.gate_max) return;  // the same answer in every thread: nothing was issued yet

  uint2 *bfrag = reinterpret_cast<uint2 *>(smem + L.bfrag);  // [nt][nsteps][8 columns]
  float *xs = reinterpret_cast<float *>(smem + L.xs);         // [nt][kc * 4]
  float *red = reinterpret_cast<float *>(smem + L.red);       // [kWarps][32][B]

  // Stage x once per CTA. Item (t, c, q, j) = the 8 values of word j of quad q in 128-k chunk c of
  // vector t; the 4 items of a quad (one 32-k group) are 4 consecutive lanes, which share its scale.
  // Vectors t < B are written whole below (items past K as zeros); only the unused t >= B (NT > B)
  // are zeroed, so the two passes touch disjoint entries and need no barrier between them.
  for (int i = B * nsteps * 8 + threadIdx.x; i < nt * nsteps * 8; i += kThreads) bfrag[i] = make_uint2(0u, 0u);
  for (int i = B * kc * 4 + threadIdx.x; i < nt * kc * 4; i += kThreads) xs[i] = 0.f;
  const int nitems = B * kc * 16;
  // Without the early loads (expert ids, a gate): warps with no staging item (32 * warp >= nitems)
  // issue their first loads now: they would only wait at the staging barrier, which their TMA holds
  // do not outlast. The others issue after it.
  const bool early = 32 * warp >= nitems;
  if (early && !pre)
    for (int s = 0; s < S; ++s) issue(s);
  for (int base = 0; base < nitems; base += kThreads) {
    const int it = base + threadIdx.x;
    const bool live = it < nitems;
    const int t = live ? it / (kc * 16) : 0, wi = it % (kc * 16);
    const int c = wi / 16, q = (wi / 4) % 4, j = wi % 4;
    float xv[8];
    // a per-slot x vector of an empty expert slot is never used: stage zeros without reading it
    const bool empty_slot = p.xpg && p.ids && live && __ldg(p.ids + t) < 0;
    if (live && !empty_slot && 8 * wi + 8 <= K) {
      if (p.x_f16) {
        const uint4 v =
            *reinterpret_cast<const uint4 *>(static_cast<const __half *>(p.x) + static_cast<size_t>(t) * K + 8 * wi);
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xv[2 * e] = __low2float(h[e]);
          xv[2 * e + 1] = __high2float(h[e]);
        }
      } else {
        const float4 *src =
            reinterpret_cast<const float4 *>(static_cast<const float *>(p.x) + static_cast<size_t>(t) * K + 8 * wi);
        const float4 a = src[0], b = src[1];
        xv[0] = a.x, xv[1] = a.y, xv[2] = a.z, xv[3] = a.w, xv[4] = b.x, xv[5] = b.y, xv[6] = b.z, xv[7] = b.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) xv[e] = 0.f;
    }
    float m = 0.f;
    int bad = 0;  // a non-finite x in the group: its scale becomes NaN
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      m = fmaxf(m, fabsf(xv[e]));
      bad |= !isfinite(xv[e]);
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (!live) continue;
    const float inv = m > 0.f && !bad ? kLimbMax / m : 0.f;
    if (j == 0)  // 1/16: weights enter as 16 * value
      xs[(t * kc + c) * 4 + q] = bad ? __int_as_float(0x7fc00000) : m / kLimbMax * (1.f / 16.f);
    int hi[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int v = static_cast<int>(rintf(xv[e] * inv));
      hi[e] = (v + 128) >> 8;
      lo[e] = v - (hi[e] << 8);
    }
    uint2 *dst = bfrag + (static_cast<size_t>(t) * nsteps + c * 4 + j) * 8;
    dst[2 * q] = make_uint2(pack_bytes(hi[0], hi[2], hi[4], hi[6]), pack_bytes(hi[1], hi[3], hi[5], hi[7]));
    dst[2 * q + 1] = make_uint2(pack_bytes(lo[0], lo[2], lo[4], lo[6]), pack_bytes(lo[1], lo[3], lo[5], lo[7]));
  }
  __syncthreads();

  // The staging warps' first loads go out only now: a TMA instruction holds lane 0's warp for
  // ~0.2 us, and issued before the staging they held the staging barrier back by up to 2 us
  // (traced); the tiles are L2-warm from the prefetch above.
  if (!early && !pre)
    for (int s = 0; s < S; ++s) issue(s);

  const int g = lane >> 2, q = lane & 3;
  const bool act = q == (g >> 1);  // lanes whose B fragment is non-zero (column g belongs to quad g / 2)
  const int pr = phys_row(g);      // physical rows pr, pr + 8, pr + 16, pr + 24 of the tile
  const int spr = K / G;
  const int BO = p.xpg ? 1 : B;    // output vectors (one per token; one in total for per-expert x)
  const uint2 *bl = bfrag + g;     // this lane's column of the B fragments
  constexpr uint32_t kHigh = 0xF0F0F0F0u;
  uint32_t u = 0, u_abort = 0;
  bool aborted = false;

  for (int r = blockIdx.x, j = 0; items.spread ? items.tile_of(j) - items.rtl * static_cast<int>(gridDim.x) < p.tiles
                                                : r < p.nrounds;
       r += gridDim.x, ++j) {
    const int tile = items.tile_of(j);
    const int tb = p.xpg ? min(tile, p.tiles - 1) / p.tpg : 0;  // x vector of this tile's expert slot
    const int wrow0 = weight_row0(p, min(tile, p.tiles - 1));
    float acc[NT][2][2];  // [token][row tile][row g, row g + 8], this lane's group
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0][0] = acc[t][0][1] = acc[t][1][0] = acc[t][1][1] = 0.f;
    // an empty expert slot: its loads were not issued (the barrier was only arrived on), so the
    // products are skipped too; its outputs are unused
    const bool skip = p.ids && tile < p.tiles && __ldg(p.ids + tile / p.tpg) < 0;
    if (tile < p.tiles) {
      for (int i = 0; i < items.per_round; ++i, ++u) {
        const int sk = items.kw * spw + i;
        const uint32_t slot = u % S;
        if (!aborted && !mbar_wait(&full[slot], (u / S) & 1)) {
          raise_status(kStatusGemvConsumerWait);
          aborted = true;  // the load never landed: no later load is issued into this ring
          u_abort = u;
        }
        const uint8_t *sb = ring + slot * p.slot_bytes;
        const int nchunk = min(2, (K - sk * kSlotK + 127) / 128);
        if (!aborted && !skip) {
#pragma unroll 1
          for (int c = 0; c < nchunk; ++c) {
            const int cg = sk * 2 + c;  // global 128-k chunk
            const uint8_t *rowp = sb + pr * 128 + (((c << 2) | q) ^ pr) * 16;
            const uint4 w0 = lds128(rowp), w1 = lds128(rowp + 1024), w2 = lds128(rowp + 2048), w3 = lds128(rowp + 3072);
            // Scales of rows pr + 8m (m = 0..3) for this lane's group (quad q of chunk cg).
            float sw[4];
            if (p.scales_tma) {
              const uint8_t *sc = sb + kWordBytes + pr * 16 + (4 * c + q) * 2;
#pragma unroll
              for (int m = 0; m < 4; ++m) sw[m] = __half2float(*reinterpret_cast<const __half *>(sc + m * 8 * 16));
            } else {
              const int gi = (cg * 128 + 32 * q) / G;
#pragma unroll
              for (int m = 0; m < 4; ++m) {
                const int row = p.gu    ? wrow0 + pr + 8 * (m & 1) + (m >> 1) * p.gu_off
                                : p.ids ? wrow0 + pr + 8 * m
                                        : min(tile * kRows + pr + 8 * m, N - 1);
                sw[m] = gi < spr ? __half2float(p.ws[static_cast<size_t>(row) * spr + gi]) : 0.f;
              }
            }
            int d[NT][2][4];
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int h = 0; h < 2; ++h) d[t][h][0] = d[t][h][1] = d[t][h][2] = d[t][h][3] = 0;
            const uint32_t v0[4] = {w0.x, w0.y, w0.z, w0.w}, v1[4] = {w1.x, w1.y, w1.z, w1.w};
            const uint32_t v2[4] = {w2.x, w2.y, w2.z, w2.w}, v3[4] = {w3.x, w3.y, w3.z, w3.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // int8 16 * value of the even (lo) and odd (hi) elements of each row's word j
              const uint32_t e0 = (v0[j] << 4) & kHigh, o0 = v0[j] & kHigh;  // row pr
              const uint32_t e1 = (v1[j] << 4) & kHigh, o1 = v1[j] & kHigh;  // row pr + 8
              const uint32_t e2 = (v2[j] << 4) & kHigh, o2 = v2[j] & kHigh;  // row pr + 16
              const uint32_t e3 = (v3[j] << 4) & kHigh, o3 = v3[j] & kHigh;  // row pr + 24
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                uint2 f = make_uint2(0u, 0u);
                if (act) f = bl[(static_cast<size_t>(tb + t) * nsteps + cg * 4 + j) * 8];
                mma_s8_16832(d[t][0], e0, e1, o0, o1, f.x, f.y);
                mma_s8_16832(d[t][1], e2, e3, o2, o3, f.x, f.y);
              }
            }
            // fp32 epilogue: this lane holds columns 2q (hi limb) and 2q + 1 (lo limb) of its group.
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              const float xsc = xs[((tb + t) * kc + cg) * 4 + q];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int r0 = d[t][h][0] * 256 + d[t][h][1], r1 = d[t][h][2] * 256 + d[t][h][3];
                acc[t][h][0] = fmaf(sw[2 * h] * xsc, static_cast<float>(r0), acc[t][h][0]);
                acc[t][h][1] = fmaf(sw[2 * h + 1] * xsc, static_cast<float>(r1), acc[t][h][1]);
              }
            }
          }
        }
        __syncwarp();  // every lane is done with the slot before lane 0 refills it
        if (!aborted) issue(u + S);
      }
    }
    // Reduce the quad's four groups, then (when K is split) the warps through shared memory.
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float v = acc[t][h][hh];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          acc[t][h][hh] = v;
        }
      if (q == 0 && t < BO && p.gu && p.ks == 1) {  // gate (h = 0) and up (h = 1) of outputs pr, pr + 8
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int j = tile * (kRows / 2) + pr + 8 * hh;
          if (tile < p.tiles && !aborted) p.y[static_cast<size_t>(t) * N + j] = silu_mul(acc[t][0][hh], acc[t][1][hh]);
        }
      } else if (q == 0 && t < BO) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {  // rows pr + 8m: (tile h = m / 2, row g or g + 8 = m % 2)
          const float v = acc[t][m >> 1][m & 1];
          if (p.ks == 1) {  // the warp owns whole rows: store directly, no barrier
            const int row = tile * kRows + pr + 8 * m;
            if (tile < p.tiles && row < N && !aborted) {
              float *out = p.y + static_cast<size_t>(t) * N + row;
              *out = p.add ? *out + v : v;
            }
          } else {
            red[(items.kw * kRows * p.rt + items.rtl * kRows + pr + 8 * m) * BO + t] = v;
          }
        }
      }
    }
    if (p.ks == 1) continue;
    __syncthreads();
    const int rows = kRows * p.rt;
    if (p.gu) {  // outputs of the round: 16 per tile, gate partials in tile rows 0..15, up in 16..31
      const int outs = rows / 2;
      for (int it = threadIdx.x; it < outs * BO; it += kThreads) {
        const int rl = it / BO, tok = it % BO;
        const int j = r * outs + rl, pb = (rl / 16) * kRows + rl % 16;
        if (j < N) {
          float gs = 0.f, us = 0.f;
          for (int w = 0; w < p.ks; ++w) {
            gs += red[(w * rows + pb) * BO + tok];
            us += red[(w * rows + pb + 16) * BO + tok];
          }
          p.y[static_cast<size_t>(tok) * N + j] = silu_mul(gs, us);
        }
      }
      __syncthreads();
      continue;
    }
    for (int it = threadIdx.x; it < rows * BO; it += kThreads) {
      const int rl = it / BO, tok = it % BO;
      const int row = r * rows + rl;
      if (row < N) {
        float v = 0.f;
        for (int w = 0; w < p.ks; ++w) v += red[(w * rows + rl) * BO + tok];
        float *out = p.y + static_cast<size_t>(tok) * N + row;
        *out = p.add ? *out + v : v;
      }
    }
    __syncthreads();
  }
  // Leave no copy in flight: after an abort, wait (bounded) for the loads issued before it.
  if (lane == 0 && aborted) {
    for (uint32_t v = u_abort; v < u_abort + S; ++v) {
      int tile, sk;
      if (items.get(v, tile, sk)) mbar_wait(&full[v % S], (v / S) & 1);
    }
  }
}

template <int G, int NT>
int launch(const uint32_t *wq, Params p, cudaStream_t stream, const DeviceInfo &dev) {
  p.scales_tma = G == 32 && (p.k / G) % 8 == 0 && aligned(p.ws, 16);
  p.slot_bytes = ((kWordBytes + (p.scales_tma ? kRows * kScaleHalvesTma * 2 : 0) + 1023) / 1024) * 1024;
  // Split K across warps (ks divides kWarps): the largest split whose rounds fit in one wave of the
  // SMs. A split that spills into a second, partly filled wave measured slower (16384 x 2048: ks = 4,
  // 128 rounds, 7.2 us; ks = 8, 256 rounds, 7.9 us), and so did splitting a matrix that already fills
  // the SMs more finely (lm_head: ks = 1, 251 rounds, 27.1 us; ks = 4, 30.4 us). ks may exceed K's
  // slots: the warps past them then have no items and add zeros, and a small matrix spreads over
  // more SMs (3072 x 2048, 8 slots: 96 CTAs of one tile instead of 48 of two).
  p.ks = 1;
  for (int ks = 2; ks <= kWarps; ks *= 2) {
    if ((p.tiles + kWarps / ks - 1) / (kWarps / ks) > dev.sms) break;
    p.ks = ks;
  }
  p.rt = kWarps / p.ks;
  p.nrounds = (p.tiles + p.rt - 1) / p.rt;
  Layout L{};
  for (p.slots = kMaxSlots; p.slots >= 1; --p.slots) {
    L = layout(p.k, p.batch, p.xpg ? p.batch : NT, p.slots, p.slot_bytes);
    if (L.total + 1024 <= dev.smem_optin) break;
  }
  const size_t smem = L.total + 1024;
  MQ_REQUIRE(p.slots >= 1 && smem <= dev.smem_optin, MQ_EUNSUPPORTED,
             "mq_gemv_q4: k=%d batch=%d needs %zu B of shared memory (max %zu)", p.k, p.batch, smem, dev.smem_optin);
  CUtensorMap wmap, smap;
  const uint64_t wrow_bytes = static_cast<uint64_t>(p.k) / 2, srow_bytes = static_cast<uint64_t>(p.k / G) * 2;
  if (p.gu) {  // planes: gate rows r and up rows r + gu_off, for r < wrows - gu_off
    const uint64_t rows = static_cast<uint64_t>(p.wrows - p.gu_off);
    if (int rc = encode_tmap_3d(&wmap, wq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.k / 8, rows, 2, wrow_bytes,
                                wrow_bytes * p.gu_off, 32, kRows / 2, 2, CU_TENSOR_MAP_SWIZZLE_128B, "mq_gate_up_q4 weights"))
      return rc;
    if (p.scales_tma)
      if (int rc = encode_tmap_3d(&smap, p.ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.k / G, rows, 2, srow_bytes,
                                  srow_bytes * p.gu_off, kScaleHalvesTma, kRows / 2, 2, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  "mq_gate_up_q4 scales"))
        return rc;
  } else {
    if (int rc = encode_tmap_2d(&wmap, wq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.k / 8, p.wrows, wrow_bytes, 32, kRows,
                                CU_TENSOR_MAP_SWIZZLE_128B, "mq_gemv_q4 weights"))
      return rc;
    if (p.scales_tma)
      if (int rc = encode_tmap_2d(&smap, p.ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.k / G, p.wrows, srow_bytes,
                                  kScaleHalvesTma, kRows, CU_TENSOR_MAP_SWIZZLE_NONE, "mq_gemv_q4 scales"))
        return rc;
  }
  if (!p.scales_tma) smap = wmap;  // not read
  auto kern = gemv_q4_kernel<G, NT>;
  static size_t configured[64] = {};
  if (int rc = ensure_smem(kern, smem, configured, "mq_gemv_q4")) return rc;
  const int grid = std::min(p.nrounds, dev.sms);
  return launch_overlapped(kern, dim3(grid), dim3(kThreads), smem, stream, "mq_gemv_q4", wmap, smap, p);
}

template <int G>
int dispatch_nt(const uint32_t *wq, const Params &p, cudaStream_t s, const DeviceInfo &dev) {
  if (p.batch == 1) return launch<G, 1>(wq, p, s, dev);
  if (p.batch == 2) return launch<G, 2>(wq, p, s, dev);
  return launch<G, 4>(wq, p, s, dev);
}

// One GEMV launch over [n, k] with batch <= 4 (also used by the MoE decode).
int gemv_q4_small(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y, int64_t n, int64_t k,
                  int group, int batch, int add, cudaStream_t stream) {
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  Params p{};
  p.ws = reinterpret_cast<const __half *>(ws);
  p.x = x;
  p.y = y;
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = batch;
  p.x_f16 = x_dtype == MQ_F16;
  p.add = add != 0;
  p.tiles = (p.n + kRows - 1) / kRows;
  p.wrows = p.n;
  switch (group) {
    case 32: return dispatch_nt<32>(wq, p, stream, dev);
    case 64: return dispatch_nt<64>(wq, p, stream, dev);
    default: return dispatch_nt<128>(wq, p, stream, dev);
  }
}

// a[t][j] = silu(W[j] . x_t) * (W[f + j] . x_t) for j < f, t < batch <= 4: the fused gate|up GEMV.
int gemv_q4_gate_up(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *a, int64_t f, int64_t k,
                    int group, int batch, cudaStream_t stream) {
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  Params p{};
  p.ws = reinterpret_cast<const __half *>(ws);
  p.x = x;
  p.y = a;
  p.n = static_cast<int>(f);
  p.k = static_cast<int>(k);
  p.batch = batch;
  p.x_f16 = x_dtype == MQ_F16;
  p.tiles = p.n / (kRows / 2);
  p.wrows = 2 * p.n;
  p.gu = 1;
  p.gu_off = p.n;
  switch (group) {
    case 32: return dispatch_nt<32>(wq, p, stream, dev);
    case 64: return dispatch_nt<64>(wq, p, stream, dev);
    default: return dispatch_nt<128>(wq, p, stream, dev);
  }
}

// The expert-indirect GEMV of the MoE decode: y[i * rows_per_group + r] = W[ids[i] * group_rows + r] . x_i
// for i < ngroups, r < rows_per_group, x_i = x (shared) or x + i * k (xpg); fp32 x, or fp16 with x_f16.
// With gate_up, y[i * rows_per_group + j] = silu(W[e_i * group_rows + j] . x_i) *
// (W[e_i * group_rows + rows_per_group + j] . x_i).
int gemv_q4_grouped(const uint32_t *wq, const uint16_t *ws, int64_t wrows, const void *x, float *y,
                    const int32_t *ids, int ngroups, int group_rows, int rows_per_group, int64_t k, int group, int xpg,
                    cudaStream_t stream, int gate_up, int x_f16, const int32_t *gate, int gate_max) {
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  Params p{};
  p.ws = reinterpret_cast<const __half *>(ws);
  p.x = x;
  p.y = y;
  p.n = ngroups * rows_per_group;
  p.k = static_cast<int>(k);
  p.batch = xpg ? ngroups : 1;
  p.x_f16 = x_f16 != 0;
  p.add = 0;
  p.wrows = static_cast<int>(wrows);
  p.ids = ids;
  p.group_rows = group_rows;
  p.xpg = xpg;
  p.gu = gate_up != 0;
  p.gu_off = rows_per_group;
  p.gate = gate;
  p.gate_max = gate_max;
  const int tr = p.gu ? kRows / 2 : kRows;
  p.tiles = p.n / tr;
  p.tpg = rows_per_group / tr;
  switch (group) {
    case 32: return launch<32, 1>(wq, p, stream, dev);
    case 64: return launch<64, 1>(wq, p, stream, dev);
    default: return launch<128, 1>(wq, p, stream, dev);
  }
}

}  // namespace gemv
}  // namespace mq

extern "C" int mq_moe_gemv_q4(const uint32_t *wq, const uint16_t *ws, int64_t wrows, const float *x, float *y,
                              const int32_t *ids, int ngroups, int group_rows, int rows_per_group, int64_t k, int group,
                              int x_per_group, void *stream) {
  MQ_REQUIRE(wq && ws && x && y && ids, MQ_EINVAL, "mq_moe_gemv_q4: null pointer");
  MQ_REQUIRE(ngroups >= 1 && ngroups <= 64 && group_rows > 0 && rows_per_group > 0 && rows_per_group <= group_rows,
             MQ_EINVAL, "mq_moe_gemv_q4: bad expert shape");
  MQ_REQUIRE(rows_per_group % 32 == 0, MQ_EINVAL, "mq_moe_gemv_q4: rows per expert must be a multiple of 32");
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL, "mq_moe_gemv_q4: group must be 32, 64 or 128");
  MQ_REQUIRE(k > 0 && k % 32 == 0 && k % group == 0 && wrows > 0 && wrows < (1LL << 31), MQ_EINVAL,
             "mq_moe_gemv_q4: bad k or weight rows");
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(x, 16) && mq::aligned(y, 4), MQ_EALIGN,
             "mq_moe_gemv_q4: wq and x must be 16-byte aligned");
  return mq::gemv::gemv_q4_grouped(wq, ws, wrows, x, y, ids, ngroups, group_rows, rows_per_group, k, group, x_per_group,
                                   static_cast<cudaStream_t>(stream), 0, 0, nullptr, 0);
}

extern "C" int mq_moe_gate_up_q4(const uint32_t *wq, const uint16_t *ws, int64_t wrows, const float *x, float *a,
                                 const int32_t *ids, int ngroups, int64_t fe, int64_t k, int group, void *stream) {
  MQ_REQUIRE(wq && ws && x && a && ids, MQ_EINVAL, "mq_moe_gate_up_q4: null pointer");
  MQ_REQUIRE(ngroups >= 1 && ngroups <= 64 && fe > 0 && fe % 16 == 0 && fe <= (1 << 20), MQ_EINVAL,
             "mq_moe_gate_up_q4: bad expert shape (fe %% 16 == 0)");
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL, "mq_moe_gate_up_q4: group must be 32, 64 or 128");
  MQ_REQUIRE(k > 0 && k % 32 == 0 && k % group == 0 && k <= (1 << 20) && wrows >= 2 * fe && wrows < (1LL << 31) &&
                 wrows % (2 * fe) == 0,
             MQ_EINVAL, "mq_moe_gate_up_q4: bad k or weight rows");
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(ws, 2) && mq::aligned(x, 16) && mq::aligned(a, 4), MQ_EALIGN,
             "mq_moe_gate_up_q4: wq and x must be 16-byte aligned");
  return mq::gemv::gemv_q4_grouped(wq, ws, wrows, x, a, ids, ngroups, static_cast<int>(2 * fe), static_cast<int>(fe), k,
                                   group, 0, static_cast<cudaStream_t>(stream), 1, 0, nullptr, 0);
}

extern "C" int mq_gate_up_q4(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *a, int64_t f,
                             int64_t k, int group, int batch, void *stream) {
  MQ_REQUIRE(wq && ws && x && a, MQ_EINVAL, "mq_gate_up_q4: null pointer");
  MQ_REQUIRE(f > 0 && k > 0 && 2 * f < (1LL << 31) && k <= (1 << 20), MQ_EINVAL, "mq_gate_up_q4: bad shape f=%lld k=%lld",
             static_cast<long long>(f), static_cast<long long>(k));
  MQ_REQUIRE(f % 16 == 0, MQ_EINVAL, "mq_gate_up_q4: f=%lld must be a multiple of 16", static_cast<long long>(f));
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL, "mq_gate_up_q4: group must be 32, 64 or 128 (got %d)",
             group);
  MQ_REQUIRE(k % 32 == 0 && k % group == 0, MQ_EINVAL, "mq_gate_up_q4: k=%lld must be a multiple of 32 and of group=%d",
             static_cast<long long>(k), group);
  MQ_REQUIRE(x_dtype == MQ_F32 || x_dtype == MQ_F16, MQ_EINVAL, "mq_gate_up_q4: x_dtype must be MQ_F32 or MQ_F16");
  MQ_REQUIRE(batch >= 1 && batch <= 4, MQ_EINVAL, "mq_gate_up_q4: batch must be in 1..4 (got %d)", batch);
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(ws, 2) && mq::aligned(x, 16) && mq::aligned(a, 4), MQ_EALIGN,
             "mq_gate_up_q4: wq and x must be 16-byte aligned, a 4-byte aligned");
  return mq::gemv::gemv_q4_gate_up(wq, ws, x, x_dtype, a, f, k, group, batch, static_cast<cudaStream_t>(stream));
}

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
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(ws, 2) && mq::aligned(x, 16) && mq::aligned(y, 4), MQ_EALIGN,
             "mq_gemv_q4: wq and x must be 16-byte aligned, y 4-byte aligned");
  if (batch > 4) {  // the tensor-core GEMM with the batch as its token dimension
    MQ_REQUIRE(x_dtype == MQ_F16, MQ_EUNSUPPORTED,
               "mq_gemv_q4: batch > 4 runs the tensor-core GEMM, which takes fp32 x only through mq_gemm_q4's workspace");
    MQ_REQUIRE(k % 256 == 0 && mq::aligned(ws, 16), MQ_EINVAL,
               "mq_gemv_q4: batch > 4 needs k %% 256 == 0 and 16-byte aligned scales");
    return mq::gemm_q4_run(wq, ws, x, x_dtype, y, n, k, batch, group, add, nullptr, 0, static_cast<cudaStream_t>(stream));
  }
  return mq::gemv::gemv_q4_small(wq, ws, x, x_dtype, y, n, k, group, batch, add, static_cast<cudaStream_t>(stream));
}
