// Prefill GEMM over int4 word-layout weights on the 5th-generation tensor cores (mq_gemm_q4).
//
// Replaces p_gemm_q4 (llama/kernels/prefill/p_gemm_q4.mojo:26-62) and gemm_q4 (lfm2/kernels/lk.mojo:
// 458-495): Y[m][r] (+)= sum_k X[m][k] * W[r][k], W int4 with an fp16 scale per `group` weights of a
// row, X fp16 [M][K], Y fp32 [M][N]. The reference stages X and the dequantised W slice in shared
// memory and multiplies on fp32 cooperative matrices; here:
//  * Up to 128 tokens (decode batches, MoE expert tiles): two CTAs per SM, each with at most half the
//    shared memory, so their pipelines hide each other's TMA, dequant and hand-off latencies. Larger
//    prefills: one CTA per SM with token tiles up to 256, dequantising each weight tile fewer times.
//  * The MMA sees W as the A operand (M = 128 weight rows per CTA) and the tokens as B (N = BN, a
//    multiple of 16 up to 256), so the accumulator tile in TMEM is [128 weight rows][BN tokens]
//    and the epilogue writes Y rows with consecutive threads on consecutive addresses.
//  * Warp 0 streams each 128-k stage with ONE multi-lane TMA instruction: the packed weights
//    (128 rows x 64 bytes) and the X tile as two 64-k sub-tiles (BN rows x 128 bytes each, 128-byte
//    swizzle, zero-filled past M).
//  * Warps 2-9 (two threads per weight row, 64 k each) dequantise the stage in registers -- byte permute,
//    mask into an fp16 mantissa (1024 + u), one fp16x2 FMA to q = u - 8 (exact), one fp16x2
//    multiply by the group scale (a single rounding) -- and store the fp16 A tile into TMEM with
//    tcgen05.st (a TMEM ring of A slots next to the accumulator; each warp writes its own lane
//    quarter). Shared memory then carries only the W/X ring. For the MoE products the activations
//    arrive in a permuted k order that needs no byte permute (dequant_word_perm).
//  * Warp 1 owns the TMEM allocation and one of its threads issues tcgen05.mma kind::f16 with A read
//    from TMEM (fp16 x fp16 -> fp32, M = 128, N = BN, K = 16, eight per stage), committing each stage
//    back to the producer (and the A slot back to the dequant warps) and the final one to the epilogue.
//  * Why 128 k per stage: the single issuing thread's per-stage work (a barrier wait, the MMAs, two
//    commits) set the pace of every mode. Timed alone, neither the dequantisation, the TMEM stores,
//    the MMAs themselves, the activation rows, the ring depth nor an L2 warm-up of the weights moved a
//    64-k-stage kernel; halving the stages per k did (431 x 8192 x 2048: 19.5 -> 16.8 us; MoE
//    gate|up at 404 tokens: 126 -> 107 us; batch-64 lm_head: 79 -> 62 us).
//  * Warps 2-9 then move the accumulator out of TMEM (tcgen05.ld 32x32b, one weight row per
//    thread, the two warps of a TMEM lane quarter taking alternate 32-column chunks), stage the fp32
//    tile in the freed ring and write it with one TMA store (a reduce-add with `add` or split K).
//  * Each CTA starts its K loop at its own 256-k offset (rotating through K): CTAs that share a
//    token tile then read different X tiles at any moment instead of all hitting the same L2 lines.
//  * Numerics: the product uses fp16 X and fp16 q*s (one rounding each); accumulation is fp32.
// Every wait on an mbarrier is bounded; on a time-out the kernel records a status code
// (mq_device_status), stops issuing work, drains what is in flight and frees its TMEM.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace mq {
namespace gemm {

constexpr int kBM = 128;  // weight rows per CTA tile (the UMMA M)
constexpr int kBK = 128;  // k per pipeline stage: two 128-byte fp16 rows of X (two swizzled sub-tiles)
constexpr int kMaxStages = 8;  // W/X ring slots in shared memory
constexpr int kACols = kBK / 2;  // TMEM columns of one dequantised A stage: 128 fp16 per row, as pairs
constexpr int kDeqWarps = 8;   // two per scheduler: one dequant warp alone cannot hide its latencies
constexpr int kThreads = 32 * (2 + kDeqWarps);  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 dequant + epilogue
constexpr int kWTileBytes = kBM * kBK / 2;  // int4 W per stage: 128 rows x 64 bytes

// MODE 0: dense Y = X W^T. MODE 1 (MoE gate|up): per expert e, rows e * 2fe + [0, fe) are gate and
// + [fe, 2fe) up; a CTA takes 64 gate rows and the 64 matching up rows and writes
// a = silu(gate) * up as fp16. MODE 2 (MoE down): per expert, a plain fp32 product. In MODE 1 and 2
// the tokens are rows of an expert-sorted X and the CTA's (expert, first row, rows) comes from a
// device tile table (mq_moe_group).
// MODE 3: dense Y = X W^T with ternary W in the transposed 2-bit layout of mq_tgemv (word
// (k / 16) * n + col holds codes k .. k + 15 of output col, weight (code - 1) * s[k / 128][col]):
// p_gemm_t2 (bonsai/kernels/prefill.mojo:155-164).
enum { kDense = 0, kGateUp = 1, kGrouped = 2, kTernary = 3 };
constexpr int kTWTileBytes = kBK / 16 * kBM * 4;  // ternary W per stage: 8 word rows x 128 outputs

struct Params {
  const __half *ws;
  float *y;
  __half *y16;            // MODE 1 output
  const int32_t *tiles;   // MODE 1, 2: (expert, first row, rows) per work tile
  const int32_t *ntiles;  // MODE 1, 2: number of work tiles (device)
  int rows_per_expert;    // MODE 1, 2: weight rows per expert (2fe or d)
  int n_out;              // MODE 1, 2: output columns per token (fe or d)
  int n, k, m;
  int bn;        // tokens per tile (multiple of 16, <= 256)
  int stages;    // pipeline depth: W/X ring slots (<= kMaxStages)
  int astages;   // dequantised A ring slots in TMEM (<= stages)
  int add;       // y += instead of y =
  int splitk;    // CTAs along K (red.add into y)
  int kb_split;  // 128-k blocks per split (a multiple of 2)
  int tiles_n, tiles_m;
  uint32_t tmem_cols;  // TMEM allocation: the fp32 accumulator, then the A ring
  uint32_t tmem_a;     // first TMEM column of the A ring
  int y_tma;  // MODE 0, 3: write y with TMA stores from a shared-memory tile (y 16-byte aligned, n % 4 == 0)
};

// Shared memory: the W/X ring (X tiles, then W tiles) and the barriers. The dequantised A tiles
// live in tensor memory, next to the accumulator, so they cost no shared-memory bandwidth: written
// with tcgen05.st, read by tcgen05.mma's A-from-TMEM form.
struct Layout {
  uint32_t x, w, bars, tmem_slot, total;
};

__host__ __device__ inline Layout layout(int bn, int stages) {
  Layout L;
  L.x = 0;
  L.w = L.x + stages * bn * kBK * 2;
  L.bars = L.w + stages * kWTileBytes;
  L.tmem_slot = L.bars + (4 * kMaxStages + 1) * 8;
  L.total = L.tmem_slot + 16;
  return L;
}

// fp16 (c - 1) * s for the 8 ternary codes in bits [shift, shift + 16) of w, in k order (16 bytes):
// codes c0, c1 of a nibble become the fp16 pair (1024 + c0, 1024 + c1), minus 1025, times s (exact).
__device__ __forceinline__ uint4 dequant_t2(uint32_t w, int shift, __half2 s2) {
  constexpr uint32_t kOne = 0x3C003C00u;   // fp16x2 (1, 1)
  constexpr uint32_t kOff = 0xE401E401u;   // fp16x2 (-1025, -1025)
  const __half2 one = *reinterpret_cast<const __half2 *>(&kOne);
  const __half2 off = *reinterpret_cast<const __half2 *>(&kOff);
  uint32_t out[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t t = w >> (shift + 4 * p);
    const uint32_t h = (t & 3u) | ((t & 0xCu) << 14) | 0x64006400u;
    __half2 f = __hfma2(*reinterpret_cast<const __half2 *>(&h), one, off);
    f = __hmul2(f, s2);
    out[p] = *reinterpret_cast<uint32_t *>(&f);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// fp16 (q - 8) * s for the 8 nibbles of a word, in k order, as 4 half2 (16 bytes).
__device__ __forceinline__ uint4 dequant_word(uint32_t w, __half2 s2) {
  constexpr uint32_t kMul = 0x2C003C00u;  // fp16x2 (1, 1/16)
  constexpr uint32_t kOff = 0xD480E408u;  // fp16x2 (-1032, -72)
  const __half2 mul = *reinterpret_cast<const __half2 *>(&kMul);
  const __half2 off = *reinterpret_cast<const __half2 *>(&kOff);
  uint32_t out[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    // byte b = nibbles 2b (low) and 2b + 1 (high), copied to both halves of the word
    const uint32_t t = __byte_perm(w, 0u, 0x4040u | b | (b << 8));
    // low half: 0x6400 | (nib ^ 8) = 1024 + u; high half: 0x6400 | (nib ^ 8) << 4 = 1024 + 16u
    const uint32_t h = (t & 0x00F0000Fu) ^ 0x64806408u;
    __half2 f = __hfma2(*reinterpret_cast<const __half2 *>(&h), mul, off);  // (u - 8, u' - 8), exact
    f = __hmul2(f, s2);
    out[b] = *reinterpret_cast<uint32_t *>(&f);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// fp16 (q - 8) * s for the 8 nibbles of a word as 4 half2 (16 bytes) in the k order
// 0, 4, 1, 5, 2, 6, 3, 7: nibbles j and j + 4 sit 16 bits apart, so one LOP3 masks both into fp16
// mantissas and flips the stored two's complement to the offset value u = q + 8 (1024 + u, or
// 1024 + 16u for the upper nibble of a byte), one fp16x2 FMA removes the offset exactly, one
// multiply applies the scale (the only rounding, as in dequant_word). No byte permute: 5 integer
// operations per word instead of 8. The activations must be stored in the same k order.
__device__ __forceinline__ uint4 dequant_word_perm(uint32_t w, __half2 s2) {
  constexpr uint32_t kOne = 0x3C003C00u;    // fp16x2 (1, 1)
  constexpr uint32_t kOff0 = 0xE408E408u;   // fp16x2 (-1032, -1032)
  constexpr uint32_t k16th = 0x2C002C00u;   // fp16x2 (1/16, 1/16)
  constexpr uint32_t kOff1 = 0xD480D480u;   // fp16x2 (-72, -72)
  const __half2 one = *reinterpret_cast<const __half2 *>(&kOne), off0 = *reinterpret_cast<const __half2 *>(&kOff0);
  const __half2 sixteenth = *reinterpret_cast<const __half2 *>(&k16th), off1 = *reinterpret_cast<const __half2 *>(&kOff1);
  const uint32_t t = w >> 8;
  const uint32_t h0 = (w & 0x000F000Fu) ^ 0x64086408u;  // (1024 + u0, 1024 + u4)
  const uint32_t h1 = (w & 0x00F000F0u) ^ 0x64806480u;  // (1024 + 16 u1, 1024 + 16 u5)
  const uint32_t h2 = (t & 0x000F000Fu) ^ 0x64086408u;  // (1024 + u2, 1024 + u6)
  const uint32_t h3 = (t & 0x00F000F0u) ^ 0x64806480u;  // (1024 + 16 u3, 1024 + 16 u7)
  uint32_t out[4];
  __half2 f;
  f = __hmul2(__hfma2(*reinterpret_cast<const __half2 *>(&h0), one, off0), s2);
  out[0] = *reinterpret_cast<uint32_t *>(&f);
  f = __hmul2(__hfma2(*reinterpret_cast<const __half2 *>(&h1), sixteenth, off1), s2);
  out[1] = *reinterpret_cast<uint32_t *>(&f);
  f = __hmul2(__hfma2(*reinterpret_cast<const __half2 *>(&h2), one, off0), s2);
  out[2] = *reinterpret_cast<uint32_t *>(&f);
  f = __hmul2(__hfma2(*reinterpret_cast<const __half2 *>(&h3), sixteenth, off1), s2);
  out[3] = *reinterpret_cast<uint32_t *>(&f);
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// Position of column j of a row stored in dequant_word_perm's k order (within each 8: 0, 4, 1, 5, 2, 6, 3, 7).
__host__ __device__ __forceinline__ int perm_col(int j) { return (j & ~7) | ((j & 3) << 1) | ((j >> 2) & 1); }

template <int G, int MODE, bool PERM = false>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_q4_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap ymap, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const Layout L = layout(p.bn, p.stages);
  // full / empty: W and X of a W/X ring slot landed / consumed by the MMA; deq / aempty: an A ring
  // slot (TMEM) written by the dequant warps / consumed by the MMA.
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
  uint64_t *deq = full + kMaxStages;
  uint64_t *empty = deq + kMaxStages;
  uint64_t *aempty = empty + kMaxStages;
  uint64_t *accum = aempty + kMaxStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.tmem_slot);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.tmem_slot + 8);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int S = p.stages, SA = p.astages;
  const bool split_rings = SA < S;  // otherwise full[s] already implies that A slot s % SA is free

  // Tile: token tiles fastest, so consecutive CTAs share (and L2-reuse) a weight tile.
  const int t = blockIdx.x;
  int tm = t % p.tiles_m, tn = (t / p.tiles_m) % p.tiles_n, split = t / (p.tiles_m * p.tiles_n);
  int n0 = tn * kBM, m0 = tm * p.bn, mcount = p.m - m0, expert = 0;
  griddep_launch_dependents();
  if (MODE == kGateUp || MODE == kGrouped) {  // grouped: work tile from the device table
    griddep_wait();      // the table is written by earlier work on the stream
    const int entry = t / p.tiles_n;
    tn = t % p.tiles_n;
    split = 0;
    if (entry >= *p.ntiles) return;  // the grid is sized for the most tiles the routing can produce
    expert = p.tiles[3 * entry];
    m0 = p.tiles[3 * entry + 1];
    mcount = p.tiles[3 * entry + 2];
    n0 = expert * p.rows_per_expert + tn * (MODE == kGateUp ? kBM / 2 : kBM);
  }
  const int nkb_total = p.k / kBK;
  const int kb0 = split * p.kb_split, nk = min(p.kb_split, nkb_total - kb0);
  // Stage i works on k-block kb0 + (i + rot) % nk; rot is a whole number of 2-block pairs.
  const int rot = 2 * (tn % max(1, nk / 2));
  auto kblock = [&](int i) { return kb0 + (i + rot) % nk; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full + i, 1);
      mbar_init(deq + i, 32 * kDeqWarps);
      mbar_init(empty + i, 1);
      mbar_init(aempty + i, 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  if (MODE == kDense || MODE == kTernary) griddep_wait();  // the set-up above touched no global memory

  if (warp == 0) {
    // ---------------- TMA producer ----------------------------------------------------------
    // A TMA instruction holds its warp for ~0.2 us on B200 whatever it copies, so the copies of a
    // stage (W, or gate and up halves of W, and X) go out as ONE instruction executed by lanes 0..2,
    // each lane with its own map, destination and coordinates.
    const int nload = MODE == kGateUp ? 4 : 3;  // W lanes (1 or 2), then the two X sub-tile lanes
    const int nwl = nload - 2;
    const CUtensorMap *lmap = lane >= nwl ? &xmap : &wmap;
    if (lane == 0) {
      prefetch_tmap(&wmap);
      prefetch_tmap(&xmap);
    }
    __syncwarp();
    const uint32_t bytes = (MODE == kTernary ? kTWTileBytes : kWTileBytes) + p.bn * kBK * 2;
    // The loops of all three roles keep their ring slot, phase and k block as running counters: a
    // single issuing thread retires only a few instructions per stage's worth of MMA time, so no
    // division or descriptor rebuild may sit in its path.
    int s = 0, round = 0, kb = kblock(0), issued = 0;
    const int kb_end = kb0 + nk;
    for (int i = 0; i < nk; ++i) {
      if (round > 0 && !__all_sync(0xffffffffu, mbar_wait(&empty[s], (round - 1) & 1))) {
        if (lane == 0) {
          raise_status(kStatusGemmTmaWait);
          *abort_flag = 1;
        }
        break;
      }
      if (lane == 0) mbar_expect_tx(&full[s], bytes);
      __syncwarp();
      if (lane < nload) {
        uint8_t *dst;
        int cx, cy;
        if (lane >= nwl) {  // X: bn token rows x 64 k, two sub-tiles per stage
          dst = smem + L.x + s * p.bn * kBK * 2 + (lane - nwl) * p.bn * 128;
          cx = kb * kBK + (lane - nwl) * 64;
          cy = m0;
        } else if (MODE == kTernary) {  // W: 4 word rows (64 k) x 128 outputs
          dst = smem + L.w + s * kWTileBytes;
          cx = n0;
          cy = kb * (kBK / 16);
        } else {  // W: 128 rows (dense), or 64 gate rows (lane 0) and the matching 64 up rows (lane 1)
          dst = smem + L.w + s * kWTileBytes + lane * (kWTileBytes / 2);
          cx = kb * (kBK / 8);
          cy = n0 + lane * (p.rows_per_expert / 2);
        }
        tma_load_2d(dst, lmap, &full[s], cx, cy);
      }
      issued = i + 1;
      if (++kb == kb_end) kb = kb0;
      if (++s == S) {
        s = 0;
        ++round;
      }
    }
    // Leave no copy in flight: wait (bounded) for the last load issued into each stage.
    if (lane == 0)
      for (int i = max(0, issued - S); i < issued; ++i) mbar_wait(&full[i % S], (i / S) & 1);
  } else if (warp == 1) {
    // ---------------- MMA issuer -------------------------------------------------------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kBM, p.bn);
      // X descriptor of slot 0; a slot further is + its byte size / 16 in the address field (the
      // field holds any shared-memory address of this CTA without carrying into bit 14).
      const uint64_t db0 = umma_desc_sw128(smem_u32(smem + L.x));
      const uint32_t da0 = tmem_d + p.tmem_a;  // A slot 0 in TMEM; a slot further is kACols columns on
      const uint32_t x_step = (p.bn * kBK * 2) >> 4;
      const uint32_t xsub = (p.bn * 128) >> 4;  // the second 64-k sub-tile of a stage
      uint32_t da = da0;
      uint64_t db = db0;
      uint32_t ph = 0;
      int s = 0, as = 0;
      for (int i = 0; i < nk; ++i) {
        // deq[as] completes only after every dequant thread saw full[s] (W and X landed) and
        // released its A writes: one acquire covers both.
        if (!mbar_wait(&deq[as], ph)) {
          raise_status(kStatusGemmMmaWait);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        // K + 16: 8 TMEM columns of A; +32 bytes = +2 in the X descriptor's address field
        umma_f16_ts(tmem_d, da, db, idesc, i != 0);
        umma_f16_ts(tmem_d, da + 8, db + 2, idesc, 1);
        umma_f16_ts(tmem_d, da + 16, db + 4, idesc, 1);
        umma_f16_ts(tmem_d, da + 24, db + 6, idesc, 1);
        umma_f16_ts(tmem_d, da + 32, db + xsub, idesc, 1);
        umma_f16_ts(tmem_d, da + 40, db + xsub + 2, idesc, 1);
        umma_f16_ts(tmem_d, da + 48, db + xsub + 4, idesc, 1);
        umma_f16_ts(tmem_d, da + 56, db + xsub + 6, idesc, 1);
        umma_commit(&empty[s]);
        if (split_rings) umma_commit(&aempty[as]);
        if (++s == S) {
          s = 0;
          db = db0;
        } else {
          db += x_step;
        }
        if (++as == SA) {
          as = 0;
          ph ^= 1;
          da = da0;
        } else {
          da += kACols;
        }
      }
      umma_commit(accum);  // also after an abort: it lands once the issued MMAs are done
    }
  } else {
    // ---------------- dequant (two threads per weight row), then the epilogue ----------------
    const int quarter = warp & 3;          // the TMEM lanes this warp may read: 32 * quarter ..
    const int half = (warp - 2) >> 2;      // which 64 k of each stage (and which column chunks) it owns
    const int row = quarter * 32 + lane;
    // the weight row this thread dequantises (rows past N are zero-filled by TMA; their scale is unused)
    const int grow = MODE == kGateUp ? n0 + (row < 64 ? row : p.rows_per_expert / 2 + row - 64)
                                     : min(n0 + row, p.n - 1);
    const int spr = p.k / G;
    // Scales: 2 stages (256 k) per vector load, prefetched one pair of stages ahead. The stages run
    // through k blocks kb0 + rot .. kb0 + nk - 1, then kb0 .. kb0 + rot - 1, a pair at a time.
    constexpr int kHalvesPerPair = 2 * kBK / G;  // 8, 4 or 2
    int qkb = kb0 + rot;  // first k block of the pair whose scales load_scales fetches next
    auto load_scales = [&](int pair, uint32_t (&dst)[4]) {
      dst[0] = dst[1] = dst[2] = dst[3] = 0u;
      if (2 * pair >= nk) return;
      const int kb = qkb;
      qkb += 2;
      if (qkb == kb0 + nk) qkb = kb0;
      if (MODE == kTernary) {  // scales [k/128][n]: this row's group of each stage of the pair
        const size_t g0 = static_cast<size_t>(kb * kBK / 128);
        const __half2 v = __halves2half2(p.ws[g0 * p.n + grow], p.ws[(g0 + 1) * p.n + grow]);
        dst[0] = *reinterpret_cast<const uint32_t *>(&v);
        return;
      }
      const __half *src = p.ws + static_cast<size_t>(grow) * spr + kb * kBK / G;
      if (kHalvesPerPair == 8) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src));
        dst[0] = v.x, dst[1] = v.y, dst[2] = v.z, dst[3] = v.w;
      } else if (kHalvesPerPair == 4) {
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(src));
        dst[0] = v.x, dst[1] = v.y;
      } else {
        dst[0] = __ldg(reinterpret_cast<const unsigned int *>(src));
      }
    };
    uint32_t cur[4], nxt[4];
    load_scales(0, cur);
    int ds = 0;        // W/X ring slot of the next stage
    uint32_t dph = 0;  // its phase parity
    int das = 0, dar = 0;  // A ring slot of the next stage and its round
    // This thread's 32 TMEM columns of A slot 0 (lane = its row; half h holds K 64h .. 64h + 63).
    const uint32_t a_t0 = tmem_d + (static_cast<uint32_t>(quarter * 32) << 16) + p.tmem_a + 32 * half;
    // This thread's 32 bytes of W in ring slot 0 (one-matrix and grouped int4 modes).
    const uint8_t *w_t0 = smem + L.w + row * (kBK / 2) + half * 32;
    for (int q2 = 0; q2 * 2 < nk; ++q2) {
      load_scales(q2 + 1, nxt);
      // The scale of word c (0..7) of this thread's 64 k in stage u of the pair, as a half2 pair.
      auto scale_of = [&](int u, int c) {
        uint32_t w;
        bool hi;
        if (G == 32) {
          w = half ? cur[2 * u + 1] : cur[2 * u];
          hi = (c >> 2) & 1;
        } else if (G == 64) {
          w = cur[u];
          hi = half;
        } else {
          w = cur[0];
          hi = u;
        }
        const __half2 pair = *reinterpret_cast<const __half2 *>(&w);
        return hi ? __high2half2(pair) : __low2half2(pair);
      };
      auto dq = [&](int u, int s, uint32_t (&r)[32]) {
        uint4 q[8];
        if (MODE == kTernary) {  // word rows 4 half .. 4 half + 3 of the stage's 8
          const __half2 s2 = scale_of(u, 0);
          const uint8_t *wt = smem + L.w + s * kWTileBytes + row * 4;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(wt + (4 * half + c) * kBM * 4);
            q[2 * c] = dequant_t2(w, 0, s2);
            q[2 * c + 1] = dequant_t2(w, 16, s2);
          }
        } else {
          const uint4 w0 = *reinterpret_cast<const uint4 *>(w_t0 + s * kWTileBytes);
          const uint4 w1 = *reinterpret_cast<const uint4 *>(w_t0 + s * kWTileBytes + 16);
          const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int c = 0; c < 8; ++c)
            q[c] = PERM ? dequant_word_perm(wv[c], scale_of(u, c)) : dequant_word(wv[c], scale_of(u, c));
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) r[4 * c] = q[c].x, r[4 * c + 1] = q[c].y, r[4 * c + 2] = q[c].z, r[4 * c + 3] = q[c].w;
      };
      auto wait_stage = [&](int s, uint32_t ph, int as, int ar) {
        bool ok = !*abort_flag;
        if (ok) ok = mbar_wait(&full[s], ph);
        if (ok && split_rings && ar > 0) ok = mbar_wait(&aempty[as], (ar - 1) & 1);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();  // the TMEM stores below come after the MMA that last read the slot
        if (!ok && lane == 0 && !*abort_flag) {
          raise_status(kStatusGemmDeqWait);
          *abort_flag = 1;
        }
        return ok;
      };
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (2 * q2 + u >= nk) break;
        if (wait_stage(ds, dph, das, dar)) {  // tcgen05.st is warp-collective: the whole warp or none
          uint32_t r[32];
          dq(u, ds, r);
          tmem_st32(a_t0 + das * kACols, r);
          tmem_wait_st();
        }
        tc_fence_before();  // orders the TMEM stores before the arrive that the MMA thread acquires
        mbar_arrive(&deq[das]);
        if (++ds == S) ds = 0, dph ^= 1;
        if (++das == SA) das = 0, ++dar;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) cur[j] = nxt[j];
    }

    // Epilogue: TMEM -> registers -> Y.
    bool ok = !*abort_flag;
    if (!mbar_wait(accum, 0)) {
      raise_status(kStatusGemmEpiWait);
      ok = false;
    }
    tc_fence_after();
    const bool live = __all_sync(0xffffffffu, ok && !*abort_flag && nk > 0);  // tcgen05.ld is warp-collective
    const uint32_t taddr = tmem_d + (static_cast<uint32_t>(quarter * 32) << 16);
    if ((MODE == kDense || MODE == kTernary) && p.y_tma) {
      // The tile goes to shared memory as [token][128 rows] fp32 (the rings are free: every copy landed
      // and every MMA finished), then one TMA store -- or an fp32 reduce-add with add or split K --
      // writes it; the tensor map clips tokens past m and rows past n. Far fewer instructions than a
      // warp store per 32 values, which left the write-out as a third of the kernel's time.
      float *tile = reinterpret_cast<float *>(smem + L.x);  // [bn][kBM]
      if (live) {
        for (int c0 = 32 * half; c0 < p.bn; c0 += 64) {
          float v[32];
          tmem_ld32(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < p.bn) tile[(c0 + j) * kBM + row] = v[j];
        }
      }
      fence_proxy_async_smem();  // each thread orders its tile writes before the TMA's reads
      named_bar_sync(1, 32 * kDeqWarps);
      if (warp == 2 && lane == 0 && live) {  // live is the same in every epilogue warp
        tma_store_2d(&ymap, tile, n0, m0, p.add || p.splitk > 1);
        bulk_commit_and_wait();
      }
    } else if ((MODE == kDense || MODE == kTernary) && live) {
      const int r = n0 + row;
      for (int c0 = 32 * half; c0 < p.bn; c0 += 64) {
        float v[32];
        tmem_ld32(taddr + c0, v);
        if (r < p.n) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int tok = m0 + c0 + j;
            if (c0 + j < p.bn && tok < p.m) {
              float *out = p.y + static_cast<size_t>(tok) * p.n + r;
              if (p.splitk > 1)
                atomicAdd(out, v[j]);
              else
                *out = p.add ? *out + v[j] : v[j];
            }
          }
        }
      }
    } else if (MODE == kGrouped && live) {
      const int r = tn * kBM + row;  // output column within the expert
      for (int c0 = 32 * half; c0 < p.bn; c0 += 64) {
        float v[32];
        tmem_ld32(taddr + c0, v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < mcount) p.y[static_cast<size_t>(m0 + c0 + j) * p.n_out + r] = v[j];
      }
    } else if (MODE == kGateUp) {
      // Up rows (TMEM lanes 64-127) go through shared memory (the W/X ring is free now) to the
      // threads holding the matching gate rows (lanes 0-63): a = silu(gate) * up, fp16. Row r's
      // column c sits at c ^ (r & 15) (bn is a multiple of 16), so the 32 rows a warp writes or reads
      // at one column fall in 16 different banks instead of one.
      float *up = reinterpret_cast<float *>(smem + L.x);  // [64 rows][bn]
      if (live && row >= 64) {
        const int ur = row - 64;
        for (int c0 = 32 * half; c0 < p.bn; c0 += 64) {
          float v[32];
          tmem_ld32(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < p.bn) up[ur * p.bn + ((c0 + j) ^ (ur & 15))] = v[j];
        }
      }
      named_bar_sync(1, 32 * kDeqWarps);
      if (live && row < 64) {
        const int col = tn * (kBM / 2) + row;  // output column within the expert
        for (int c0 = 32 * half; c0 < p.bn; c0 += 64) {
          float v[32];
          tmem_ld32(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j < mcount) {
              const float g = v[j], u = up[row * p.bn + ((c0 + j) ^ (row & 15))];
              p.y16[static_cast<size_t>(m0 + c0 + j) * p.n_out + (PERM ? perm_col(col) : col)] =
                  __float2half_rn(g / (1.f + expf(-g)) * u);
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_d, p.tmem_cols);
  }
}

__global__ void f32_to_f16_kernel(const float4 *__restrict__ x, uint2 *__restrict__ out, int64_t n4) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = x[i];
    out[i] = make_uint2(pack_half2(v.x, v.y), pack_half2(v.z, v.w));
  }
}

// TMEM of one CTA (`budget` columns: 512, or 256 with two CTAs per SM): the accumulator's bn
// columns (rounded to 32), then as many A stages as fit, at most one per W/X slot.
inline void plan_tmem(Params &p, uint32_t budget) {
  p.tmem_a = (static_cast<uint32_t>(p.bn) + 31) / 32 * 32;  // bn <= 128 when budget is 256
  p.astages = std::min<int>(p.stages, (budget - p.tmem_a) / kACols);
  p.tmem_cols = 32;
  while (p.tmem_cols < p.tmem_a + p.astages * kACols) p.tmem_cols *= 2;
}

template <int G, int MODE = kDense>
int launch(const uint32_t *wq, const __half *x16, Params p, cudaStream_t stream, const DeviceInfo &dev) {
  // Tiles: tokens split as evenly as possible into tiles of a multiple of 16. Up to 128 tokens: one
  // tile, two CTAs per SM (two independent pipelines hide each other's latencies). More: tiles of up
  // to 256 tokens and one CTA per SM, so each weight tile is dequantised as few times as possible.
  const bool two_per_sm = p.m <= 128;
  p.tiles_n = (p.n + kBM - 1) / kBM;
  // Split K (in pairs of 128-k blocks) into as many parts as one wave of the SMs holds (two CTAs per
  // SM when they share it): the longest part sets the time (431 tokens x 3072 x 2048: 48 tiles x 3
  // parts of at most 12 blocks).
  const int nkb = p.k / kBK, pairs = nkb / 2;
  const int slots = two_per_sm ? 2 * dev.sms : dev.sms;
  auto plan_k = [&](int tiles_m, int &kb_split, int &splitk) {
    const int tiles = tiles_m * p.tiles_n;
    const int s = std::max(1, std::min(pairs, slots / std::max(tiles, 1)));
    kb_split = ((pairs + s - 1) / s) * 2;
    splitk = (nkb + kb_split - 1) / kb_split;
  };
  // Token tiles: the fewest of at most 256 tokens, or one more when that fills the waves of SMs
  // better. A 128 x N x 16 MMA costs about 96 cycles for N <= 128 and 138 at N = 256 (measured), so
  // a wave of narrower tiles can finish sooner than a part-filled extra wave of wide ones
  // (512 x 12288 x 4096 ternary: 3 tiles of 176 tokens, 288 CTAs in two full waves, +4 % over
  // 2 tiles of 256, 192 CTAs in a wave and a third).
  auto cost = [&](int tiles_m) {
    int kb_split, splitk;
    plan_k(tiles_m, kb_split, splitk);
    const int bn = ((p.m + tiles_m - 1) / tiles_m + 15) / 16 * 16;
    const int64_t waves = (static_cast<int64_t>(tiles_m) * p.tiles_n * splitk + slots - 1) / slots;
    return waves * kb_split * (96 + std::max(0, bn - 128) * 42 / 128);
  };
  p.tiles_m = two_per_sm ? 1 : (p.m + 255) / 256;
  if (!two_per_sm && cost(p.tiles_m + 1) < cost(p.tiles_m)) ++p.tiles_m;
  p.bn = ((p.m + p.tiles_m - 1) / p.tiles_m + 15) / 16 * 16;
  const int tiles = p.tiles_m * p.tiles_n;
  plan_k(p.tiles_m, p.kb_split, p.splitk);
  // Pipeline depth: as many stages as the SM's shared memory (or half of it) holds.
  const size_t budget = two_per_sm ? dev.smem_optin / 2 - 1024 : dev.smem_optin;
  Layout L{};
  for (p.stages = kMaxStages; p.stages >= 2; --p.stages) {
    L = layout(p.bn, p.stages);
    if (L.total + 1024 <= budget) break;
  }
  plan_tmem(p, two_per_sm ? 256 : 512);
  const size_t smem = L.total + 1024;
  MQ_REQUIRE(smem <= dev.smem_optin, MQ_EUNSUPPORTED, "mq_gemm_q4: tile of %d tokens needs %zu B of shared memory", p.bn,
             smem);
  CUtensorMap wmap, xmap;
  if (MODE == kTernary) {  // [k/16][n] words: boxes of 128 outputs x 4 word rows
    if (int rc = encode_tmap_2d(&wmap, wq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.n, p.k / 16, static_cast<uint64_t>(p.n) * 4,
                                kBM, kBK / 16, CU_TENSOR_MAP_SWIZZLE_NONE, "mq_gemm_t2 weights"))
      return rc;
  } else if (int rc = encode_tmap_2d(&wmap, wq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.k / 8, p.n,
                                     static_cast<uint64_t>(p.k) / 2, kBK / 8, kBM, CU_TENSOR_MAP_SWIZZLE_NONE,
                                     "mq_gemm_q4 weights")) {
    return rc;
  }
  if (int rc = encode_tmap_2d(&xmap, x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.k, p.m, static_cast<uint64_t>(p.k) * 2, 64,
                              p.bn, CU_TENSOR_MAP_SWIZZLE_128B, "mq_gemm_q4 activations"))
    return rc;
  if (p.splitk > 1 && !p.add) {
    cudaError_t e = cudaMemsetAsync(p.y, 0, static_cast<size_t>(p.m) * p.n * sizeof(float), stream);
    if (e != cudaSuccess) return fail(MQ_ECUDA, "mq_gemm_q4: zeroing y: %s", cudaGetErrorString(e));
  }
  auto kern = gemm_q4_kernel<G, MODE>;
  static size_t configured[64] = {};
  if (int rc = ensure_smem(kern, smem, configured, "mq_gemm_q4")) return rc;
  // y through TMA stores when the tensor map can describe it (16-byte base and row stride) and the
  // [bn][128] fp32 staging tile fits where the rings were.
  CUtensorMap ymap = xmap;  // not read unless y_tma
  p.y_tma = aligned(p.y, 16) && p.n % 4 == 0 && static_cast<size_t>(p.bn) * kBM * 4 <= L.bars;
  if (p.y_tma) {
    if (int rc = encode_tmap_2d(&ymap, p.y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.n, p.m, static_cast<uint64_t>(p.n) * 4,
                                kBM, p.bn, CU_TENSOR_MAP_SWIZZLE_NONE, "mq_gemm_q4 output"))
      return rc;
  }
  return launch_overlapped(kern, dim3(tiles * p.splitk), dim3(kThreads), smem, stream, "mq_gemm_q4", wmap, xmap, ymap, p);
}

template <int G, int MODE, bool PERM>
int launch_grouped(const uint32_t *wq, const __half *ws, const __half *xs, int64_t pairs, int64_t k, int experts,
                   int rows_per_expert, const int32_t *tiles, const int32_t *ntiles, int max_tiles, int bn, void *out,
                   cudaStream_t stream, const DeviceInfo &dev) {
  Params p{};
  p.ws = ws;
  p.y = MODE == kGrouped ? static_cast<float *>(out) : nullptr;
  p.y16 = MODE == kGateUp ? static_cast<__half *>(out) : nullptr;
  p.tiles = tiles;
  p.ntiles = ntiles;
  p.rows_per_expert = rows_per_expert;
  p.n_out = MODE == kGateUp ? rows_per_expert / 2 : rows_per_expert;
  p.n = experts * rows_per_expert;
  p.k = static_cast<int>(k);
  p.m = static_cast<int>(pairs);
  p.bn = bn;
  p.tiles_m = 1;
  p.tiles_n = MODE == kGateUp ? (rows_per_expert / 2) / (kBM / 2) : rows_per_expert / kBM;
  p.splitk = 1;
  p.kb_split = p.k / kBK;
  // Two CTAs per SM while both fit their accumulators and A rings in half of TMEM.
  const bool two_per_sm = bn <= 128;
  const size_t budget = two_per_sm ? dev.smem_optin / 2 - 1024 : dev.smem_optin;
  Layout L{};
  for (p.stages = kMaxStages; p.stages >= 2; --p.stages) {
    L = layout(p.bn, p.stages);
    if (L.total + 1024 <= budget) break;
  }
  plan_tmem(p, two_per_sm ? 256 : 512);
  const size_t smem = L.total + 1024;
  CUtensorMap wmap, xmap;
  if (int rc = encode_tmap_2d(&wmap, wq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.k / 8, p.n, static_cast<uint64_t>(p.k) / 2,
                              kBK / 8, MODE == kGateUp ? kBM / 2 : kBM, CU_TENSOR_MAP_SWIZZLE_NONE, "mq_moe_gemm_q4 weights"))
    return rc;
  if (int rc = encode_tmap_2d(&xmap, xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.k, p.m, static_cast<uint64_t>(p.k) * 2, 64,
                              p.bn, CU_TENSOR_MAP_SWIZZLE_128B, "mq_moe_gemm_q4 activations"))
    return rc;
  auto kern = gemm_q4_kernel<G, MODE, PERM>;
  static size_t configured[64] = {};
  if (int rc = ensure_smem(kern, smem, configured, "mq_moe_gemm_q4")) return rc;
  p.y_tma = 0;
  return launch_overlapped(kern, dim3(max_tiles * p.tiles_n), dim3(kThreads), smem, stream, "mq_moe_gemm_q4", wmap, xmap,
                           xmap, p);
}

}  // namespace gemm

// Grouped expert product (MoE): mode 1 = gate|up with SiLU (fp16 out), mode 2 = plain (fp32 out).
// perm: xs rows (and mode 1's output rows) are stored in dequant_word_perm's k order.
int moe_gemm_run(int mode, const uint32_t *wq, const uint16_t *ws, const uint16_t *xs, int64_t pairs, int64_t k,
                 int experts, int64_t rows_per_expert, int group, const int32_t *tiles, const int32_t *ntiles,
                 int max_tiles, int tile_m, void *out, cudaStream_t stream, int perm) {
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  const __half *w16 = reinterpret_cast<const __half *>(ws);
  const __half *x16 = reinterpret_cast<const __half *>(xs);
  const int rpe = static_cast<int>(rows_per_expert);
#define MQ_GROUPED(G, P)                                                                                               \
  return mode == 1 ? gemm::launch_grouped<G, gemm::kGateUp, P>(wq, w16, x16, pairs, k, experts, rpe, tiles, ntiles,    \
                                                              max_tiles, tile_m, out, stream, dev)                    \
                   : gemm::launch_grouped<G, gemm::kGrouped, P>(wq, w16, x16, pairs, k, experts, rpe, tiles, ntiles,   \
                                                               max_tiles, tile_m, out, stream, dev)
  if (perm) {
    switch (group) {
      case 32: MQ_GROUPED(32, true);
      case 64: MQ_GROUPED(64, true);
      default: MQ_GROUPED(128, true);
    }
  }
  switch (group) {
    case 32: MQ_GROUPED(32, false);
    case 64: MQ_GROUPED(64, false);
    default: MQ_GROUPED(128, false);
  }
#undef MQ_GROUPED
}

// Shared by mq_gemm_q4 and the batched decode path of mq_gemv_q4.
int gemm_q4_run(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y, int64_t n, int64_t k,
                int64_t m, int group, int add, void *workspace, size_t workspace_bytes, cudaStream_t stream) {
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  const __half *x16 = static_cast<const __half *>(x);
  if (x_dtype == MQ_F32) {
    const size_t need = static_cast<size_t>(m) * k * 2;
    MQ_REQUIRE(workspace && workspace_bytes >= need, MQ_EINVAL,
               "mq_gemm_q4: fp32 activations need a workspace of %zu bytes (got %zu)", need, workspace_bytes);
    MQ_REQUIRE(aligned(workspace, 16), MQ_EALIGN, "mq_gemm_q4: workspace must be 16-byte aligned");
    const int64_t n4 = m * k / 4;
    const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(dev.sms) * 8));
    gemm::f32_to_f16_kernel<<<grid, 256, 0, stream>>>(static_cast<const float4 *>(x), static_cast<uint2 *>(workspace), n4);
    if (int rc = check_launch("mq_gemm_q4 (fp32 -> fp16)")) return rc;
    x16 = static_cast<const __half *>(workspace);
  }
  gemm::Params p{};
  p.ws = reinterpret_cast<const __half *>(ws);
  p.y = y;
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.m = static_cast<int>(m);
  p.add = add != 0;
  switch (group) {
    case 32: return gemm::launch<32>(wq, x16, p, stream, dev);
    case 64: return gemm::launch<64>(wq, x16, p, stream, dev);
    default: return gemm::launch<128>(wq, x16, p, stream, dev);
  }
}

// mq_gemm_q4_noalloc keeps its fp16 copy of the fp32 activations in this module's own device memory,
// for callers that have no device allocator to hand: a binding that can pass only (wq, ws, x, y, n, k)
// and no scratch buffer, or a host whose memory manager owns every device allocation. One copy per
// CUDA context (normally one per device), shared by every call in that context.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // m * k * 2 bytes at most
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the current context's copy of g_noalloc_scratch, looked up once per context
// (a caller that makes its own, non-primary context current gets that context's copy) and cached.
int noalloc_scratch(void **out) {
  typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
  static std::mutex mu;
  static CtxGetCurrentFn ctx_fn = nullptr;
  static CUcontext keys[64] = {};
  static void *cache[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);  // also makes the device's primary context current if none is
  if (e != cudaSuccess) return fail(MQ_ECUDA, "mq_gemm_q4_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  if (!ctx_fn) {
    void *fp = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fp, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fp)
      return fail(MQ_ECUDA, "mq_gemm_q4_noalloc: cuCtxGetCurrent is not available from the driver");
    ctx_fn = reinterpret_cast<CtxGetCurrentFn>(fp);
  }
  CUcontext ctx = nullptr;
  if (ctx_fn(&ctx) != CUDA_SUCCESS || !ctx) {
    e = cudaFree(nullptr);  // no context current yet: let the runtime make the primary one current
    if (e != cudaSuccess || ctx_fn(&ctx) != CUDA_SUCCESS || !ctx)
      return fail(MQ_ECUDA, "mq_gemm_q4_noalloc: no current CUDA context");
  }
  int slot = 0;
  while (slot < 64 && keys[slot] && keys[slot] != ctx) ++slot;
  if (slot == 64) return fail(MQ_EUNSUPPORTED, "mq_gemm_q4_noalloc: more than 64 CUDA contexts");
  if (!keys[slot]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(MQ_ECUDA, "mq_gemm_q4_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    cache[slot] = p;
    keys[slot] = ctx;
  }
  *out = cache[slot];
  return MQ_OK;
}

int gemm_q4_noalloc_run(const uint32_t *wq, const uint16_t *ws, const float *x, float *y, int64_t n, int64_t k,
                        int64_t m, int group, int add, cudaStream_t stream) {
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  void *scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // The conversion writes all m * k halves the product reads, so nothing in the scratch needs to start at zero.
  const int64_t n4 = m * k / 4;
  const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(dev.sms) * 8));
  gemm::f32_to_f16_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const float4 *>(x), static_cast<uint2 *>(scratch), n4);
  if (int rc = check_launch("mq_gemm_q4_noalloc (fp32 -> fp16)")) return rc;
  const __half *x16 = static_cast<const __half *>(scratch);
  gemm::Params p{};
  p.ws = reinterpret_cast<const __half *>(ws);
  p.y = y;
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.m = static_cast<int>(m);
  p.add = add != 0;
  switch (group) {
    case 32: return gemm::launch<32>(wq, x16, p, stream, dev);
    case 64: return gemm::launch<64>(wq, x16, p, stream, dev);
    default: return gemm::launch<128>(wq, x16, p, stream, dev);
  }
}

}  // namespace mq

extern "C" size_t mq_gemm_q4_workspace_size(int64_t m, int64_t k, int x_dtype) {
  return x_dtype == MQ_F32 && m > 0 && k > 0 ? static_cast<size_t>(m) * k * 2 : 0;
}

extern "C" int mq_gemm_q4(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y, int64_t n,
                          int64_t k, int64_t m, int group, int add, void *workspace, size_t workspace_bytes, void *stream) {
  MQ_REQUIRE(wq && ws && x && y, MQ_EINVAL, "mq_gemm_q4: null pointer");
  MQ_REQUIRE(n > 0 && k > 0 && m > 0 && n < (1LL << 31) && k <= (1 << 20) && m < (1LL << 24), MQ_EINVAL,
             "mq_gemm_q4: bad shape n=%lld k=%lld m=%lld", static_cast<long long>(n), static_cast<long long>(k),
             static_cast<long long>(m));
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL, "mq_gemm_q4: group must be 32, 64 or 128 (got %d)", group);
  MQ_REQUIRE(k % 256 == 0, MQ_EINVAL, "mq_gemm_q4: k=%lld must be a multiple of 256", static_cast<long long>(k));
  MQ_REQUIRE(x_dtype == MQ_F32 || x_dtype == MQ_F16, MQ_EINVAL, "mq_gemm_q4: x_dtype must be MQ_F32 or MQ_F16");
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(ws, 16) && mq::aligned(x, 16) && mq::aligned(y, 4), MQ_EALIGN,
             "mq_gemm_q4: wq, ws and x must be 16-byte aligned, y 4-byte aligned");
  return mq::gemm_q4_run(wq, ws, x, x_dtype, y, n, k, m, group, add, workspace, workspace_bytes,
                         static_cast<cudaStream_t>(stream));
}

extern "C" int mq_gemm_q4_noalloc(const uint32_t *wq, const uint16_t *ws, const float *x, float *y, int64_t n,
                                  int64_t k, int64_t m, int group, int add, void *stream) {
  MQ_REQUIRE(wq && ws && x && y, MQ_EINVAL, "mq_gemm_q4_noalloc: null pointer");
  MQ_REQUIRE(n > 0 && k > 0 && m > 0 && n < (1LL << 31) && k <= (1 << 20) && m < (1LL << 24), MQ_EINVAL,
             "mq_gemm_q4_noalloc: bad shape n=%lld k=%lld m=%lld", static_cast<long long>(n), static_cast<long long>(k),
             static_cast<long long>(m));
  MQ_REQUIRE(static_cast<size_t>(m) * static_cast<size_t>(k) * 2 <= mq::kNoAllocScratchBytes, MQ_EINVAL,
             "mq_gemm_q4_noalloc: m * k = %lld activations need %lld bytes of scratch, above its fixed %zu "
             "(m * k <= %zu); use mq_gemm_q4 with a workspace",
             static_cast<long long>(m * k), static_cast<long long>(m * k * 2), mq::kNoAllocScratchBytes,
             mq::kNoAllocScratchBytes / 2);
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL,
             "mq_gemm_q4_noalloc: group must be 32, 64 or 128 (got %d)", group);
  MQ_REQUIRE(k % 256 == 0, MQ_EINVAL, "mq_gemm_q4_noalloc: k=%lld must be a multiple of 256", static_cast<long long>(k));
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(ws, 16) && mq::aligned(x, 16) && mq::aligned(y, 4), MQ_EALIGN,
             "mq_gemm_q4_noalloc: wq, ws and x must be 16-byte aligned, y 4-byte aligned");
  return mq::gemm_q4_noalloc_run(wq, ws, x, y, n, k, m, group, add, static_cast<cudaStream_t>(stream));
}

extern "C" int mq_gemm_t2(const void *x, int x_dtype, const uint32_t *w, const uint16_t *s, float *y, int64_t n, int64_t k,
                          int64_t m, int add, void *workspace, size_t workspace_bytes, void *stream) {
  MQ_REQUIRE(x && w && s && y, MQ_EINVAL, "mq_gemm_t2: null pointer");
  MQ_REQUIRE(n > 0 && k > 0 && m > 0 && n < (1LL << 31) && k <= (1 << 20) && m < (1LL << 24), MQ_EINVAL,
             "mq_gemm_t2: bad shape n=%lld k=%lld m=%lld", static_cast<long long>(n), static_cast<long long>(k),
             static_cast<long long>(m));
  MQ_REQUIRE(k % 256 == 0 && n % 4 == 0, MQ_EINVAL, "mq_gemm_t2: k must be a multiple of 256 and n of 4");
  MQ_REQUIRE(x_dtype == MQ_F32 || x_dtype == MQ_F16, MQ_EINVAL, "mq_gemm_t2: x_dtype must be MQ_F32 or MQ_F16");
  MQ_REQUIRE(mq::aligned(w, 16) && mq::aligned(s, 2) && mq::aligned(x, 16) && mq::aligned(y, 4), MQ_EALIGN,
             "mq_gemm_t2: w and x must be 16-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __half *x16 = static_cast<const __half *>(x);
  if (x_dtype == MQ_F32) {
    const size_t need = static_cast<size_t>(m) * k * 2;
    MQ_REQUIRE(workspace && workspace_bytes >= need && mq::aligned(workspace, 16), MQ_EINVAL,
               "mq_gemm_t2: fp32 activations need a 16-byte aligned workspace of %zu bytes (got %zu)", need,
               workspace_bytes);
    const int64_t n4 = m * k / 4;
    const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(dev.sms) * 8));
    mq::gemm::f32_to_f16_kernel<<<grid, 256, 0, st>>>(static_cast<const float4 *>(x), static_cast<uint2 *>(workspace), n4);
    if (int rc = mq::check_launch("mq_gemm_t2 (fp32 -> fp16)")) return rc;
    x16 = static_cast<const __half *>(workspace);
  }
  mq::gemm::Params p{};
  p.ws = reinterpret_cast<const __half *>(s);
  p.y = y;
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.m = static_cast<int>(m);
  p.add = add != 0;
  return mq::gemm::launch<128, mq::gemm::kTernary>(w, x16, p, st, dev);
}

extern "C" int mq_moe_gemm_q4(int mode, const uint32_t *wq, const uint16_t *ws, const uint16_t *xs, int64_t pairs,
                              int64_t k, int experts, int64_t rows_per_expert, int group, const int32_t *tiles,
                              const int32_t *ntiles, int max_tiles, int tile_m, void *out, void *stream) {
  MQ_REQUIRE(wq && ws && xs && tiles && ntiles && out, MQ_EINVAL, "mq_moe_gemm_q4: null pointer");
  MQ_REQUIRE(mode == 1 || mode == 2, MQ_EINVAL, "mq_moe_gemm_q4: mode must be 1 (gate|up, SiLU) or 2 (plain)");
  MQ_REQUIRE(pairs > 0 && k > 0 && k % 256 == 0, MQ_EINVAL, "mq_moe_gemm_q4: k=%lld must be a multiple of 256",
             static_cast<long long>(k));
  MQ_REQUIRE(experts >= 1 && rows_per_expert > 0 && static_cast<int64_t>(experts) * rows_per_expert < (1LL << 31), MQ_EINVAL,
             "mq_moe_gemm_q4: bad expert shape");
  MQ_REQUIRE(mode == 1 ? rows_per_expert % 128 == 0 : rows_per_expert % 128 == 0, MQ_EINVAL,
             "mq_moe_gemm_q4: rows per expert must be a multiple of 128 (gate|up: 2fe with fe %% 64 == 0)");
  MQ_REQUIRE(group == 32 || group == 64 || group == 128, MQ_EINVAL, "mq_moe_gemm_q4: group must be 32, 64 or 128");
  MQ_REQUIRE(tile_m >= 16 && tile_m <= (mode == 1 ? 128 : 256) && tile_m % 16 == 0, MQ_EINVAL,
             "mq_moe_gemm_q4: tile_m must be a multiple of 16 in 16..%d", mode == 1 ? 128 : 256);
  MQ_REQUIRE(max_tiles >= 1, MQ_EINVAL, "mq_moe_gemm_q4: max_tiles must be >= 1");
  MQ_REQUIRE(mq::aligned(wq, 16) && mq::aligned(ws, 16) && mq::aligned(xs, 16), MQ_EALIGN,
             "mq_moe_gemm_q4: wq, ws and xs must be 16-byte aligned");
  return mq::moe_gemm_run(mode, wq, ws, xs, pairs, k, experts, rows_per_expert, group, tiles, ntiles, max_tiles, tile_m,
                          out, static_cast<cudaStream_t>(stream), 0);
}
