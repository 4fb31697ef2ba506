// Top-k MoE on int4 experts: routing, grouping by expert, gathering, the SwiGLU product and the
// weighted combine (the expert products themselves run on the grouped tcgen05 GEMM, gemm_q4.cu,
// and for one token on the grouped GEMV, gemv_q4.cu).
//
// Reference functions (qwen3moe/kernels/moek.mojo): route / p_route (:156-197, :385-425),
// p_expert_lists / p_expert_items (:432-442, :548-557), t_moe_gate_up / t_moe_down (:560-608),
// moe_gate_up / moe_down (:200-223), p_moe_sum (:479-488); the grouped design follows
// lfm2moe/kernels/mk.mojo:123-199 (p_group, p_gather, p_silu_mul, p_combine).
#include <algorithm>

#include "common.cuh"

namespace mq {
namespace moe {

// ---- routing: one warp per token -----------------------------------------------------------
// Top-k experts by logit (the lowest index among equals), then softmax over the k chosen logits
// (max-subtracted, fp32), as route / p_route compute it. E <= 256 (each lane holds E / 32 logits).
// One token's routing by one warp: v[i] is the logit of expert i * 32 + lane (-inf past experts).
// route_kernel and the fused router chain (route_group_kernel) both use it, so the two route alike.
template <int PER>
__device__ __forceinline__ void route_row(float (&v)[PER], int lane, int experts, int topk, int32_t *__restrict__ ids_row,
                                          float *__restrict__ weights_row) {
  float top[32];
  int32_t idx[32];
  for (int k = 0; k < topk; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      if (e < experts && (v[i] > best || (v[i] == best && e < bi))) {
        best = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    top[k] = best;
    idx[k] = bi;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i * 32 + lane == bi) v[i] = -INFINITY;
  }
  if (lane == 0) {
    float total = 0.f;
    for (int k = 0; k < topk; ++k) total += expf(top[k] - top[0]);
    for (int k = 0; k < topk; ++k) {
      ids_row[k] = idx[k];
      weights_row[k] = expf(top[k] - top[0]) / total;
    }
  }
}

template <int PER>  // logits per lane
__global__ void route_kernel(const float *__restrict__ logits, int32_t *__restrict__ ids, float *__restrict__ weights,
                             int tokens, int experts, int topk) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= tokens) return;
  const float *lg = logits + static_cast<size_t>(warp) * experts;
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < experts ? lg[e] : -INFINITY;
  }
  route_row<PER>(v, lane, experts, topk, ids + static_cast<size_t>(warp) * topk, weights + static_cast<size_t>(warp) * topk);
}

// ---- grouping: a stable counting sort of the (token, slot) pairs by expert, one CTA ---------
// offsets[e] = number of pairs routed to experts < e; order[offsets[e] + r] = the r-th pair (in
// increasing pair index t * topk + k) whose expert is e -- p_expert_lists' lists, concatenated;
// slot_of[pair] = its position in that order; tiles = (expert, first row, rows) work items of at
// most `tile` rows per expert -- p_expert_items' items, over the concatenated lists.
constexpr int kGroupThreads = 1024;

// Pairs are bucketed by ids[i] / div (div = 1: by expert; div = experts per rank: by owning rank,
// the expert-parallel dispatch order). tiles / ntiles may be null (no work tiles). local, when not
// null, receives ids[i] - bucket * div at the pair's sorted position. A negative id means "no
// expert" (the padding of a fixed-capacity exchange): the pair is left out silently.
// cap > 0: the fixed-capacity layout of an exchange with static split sizes. Bucket b's pairs sit at
// b * cap .. in pair order, every other position of order and local holds -1, offsets[b] = b * cap,
// and pairs past a bucket's capacity are reported (kStatusEpOverflow) and left out.
__global__ void __launch_bounds__(kGroupThreads) group_kernel(const int32_t *__restrict__ ids, int div, int pairs,
                                                              int experts, int tile, int32_t *__restrict__ counts,
                                                              int32_t *__restrict__ offsets, int32_t *__restrict__ order,
                                                              int32_t *__restrict__ slot_of, int32_t *__restrict__ tiles,
                                                              int32_t *__restrict__ ntiles, int32_t *__restrict__ local,
                                                              int cap, FlagWait wait = FlagWait(), int small_limit = 0) {
  griddep_launch_dependents();
  griddep_wait();    // programmatic dependent launch (behind the fused router, or an exchange step): ids are written
  wait_flags(wait);  // an expert-parallel owner: the senders' rows and ids have arrived
  extern __shared__ int32_t sh[];
  int32_t *warp_cnt = sh;                    // [32 warps][experts]: pairs of the warp's range, then their start
  int32_t *start = warp_cnt + 32 * experts;  // [experts + 1]: bucket totals, then offsets
  int32_t *tstart = start + experts + 1;     // [experts + 1]: first work tile of each bucket
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const unsigned lt_mask = (1u << lane) - 1u;
  // Warp w owns the contiguous pairs [lo, hi): ranks within a bucket follow pair index because the
  // warps' ranges are in pair order and each warp walks its own range in order.
  const int per = (pairs + 31) / 32;
  const int lo = min(pairs, warp * per), hi = min(pairs, lo + per);
  // Bucket of pair i, or -1 (left out) for a negative id and (reported) for an id past experts * div.
  auto bucket = [&](int i) {
    const int id = ids[i];
    if (id < 0) return -1;
    if (id >= experts * div) {
      raise_status(kStatusMoeBadExpertId);
      return -1;
    }
    return id / div;
  };
  auto tiles_of = [&](int c) { return tiles ? (c + tile - 1) / tile : 0; };

  // Each lane's first kCache pairs' buckets stay in registers for both passes (their ids are loaded
  // once, all at the same time); pairs past them (more than 32 x 32 x kCache) are read again.
  constexpr int kCache = 8;
  int bc[kCache];
#pragma unroll
  for (int j = 0; j < kCache; ++j) {
    const int i = lo + lane + 32 * j;
    bc[j] = i < hi ? bucket(i) : -1;
  }
  // Pass 1: per-warp histograms.
  for (int j = threadIdx.x; j < 32 * experts; j += kGroupThreads) warp_cnt[j] = 0;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kCache; ++j)
    if (bc[j] >= 0) atomicAdd(&warp_cnt[warp * experts + bc[j]], 1);
  for (int i = lo + lane + 32 * kCache; i < hi; i += 32) {
    const int b = bucket(i);
    if (b >= 0) atomicAdd(&warp_cnt[warp * experts + b], 1);
  }
  __syncthreads();
  // Per bucket: each warp's start within the bucket (exclusive over warps) and the bucket total.
  for (int e = threadIdx.x; e < experts; e += kGroupThreads) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = warp_cnt[w * experts + e];
      warp_cnt[w * experts + e] = run;
      run += c;
    }
    start[e] = run;
  }
  __syncthreads();
  // Exclusive scans over buckets of the totals and of the work tiles (warp 0, chunk of buckets per lane).
  if (warp == 0) {
    const int chunk = (experts + 31) / 32;
    int csum = 0, ctiles = 0;
    for (int j = 0; j < chunk; ++j) {
      const int e = lane * chunk + j;
      if (e < experts) csum += start[e], ctiles += tiles_of(start[e]);
    }
    int inc = csum, tinc = ctiles;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o), tv = __shfl_up_sync(0xffffffffu, tinc, o);
      if (lane >= o) inc += v, tinc += tv;
    }
    int run = inc - csum, trun = tinc - ctiles;
    for (int j = 0; j < chunk; ++j) {
      const int e = lane * chunk + j;
      if (e < experts) {
        const int c = start[e];
        counts[e] = c;
        offsets[e] = run;
        start[e] = run;
        tstart[e] = trun;
        run += c;
        trun += tiles_of(c);
      }
    }
    if (lane == 31) {
      start[experts] = run;
      offsets[experts] = run;
      tstart[experts] = trun;
      // small_limit: at most that many kept pairs run on the per-pair GEMVs, so no tile is handed out
      if (ntiles) *ntiles = small_limit > 0 && run <= small_limit ? 0 : trun;
    }
  }
  __syncthreads();
  if (cap > 0) {  // fixed-capacity layout: every position empty until pass 2 fills it
    for (int e = threadIdx.x; e <= experts; e += kGroupThreads) offsets[e] = e * cap;
    for (int pos = threadIdx.x; pos < experts * cap; pos += kGroupThreads) {
      order[pos] = -1;
      if (local) local[pos] = -1;
    }
    __syncthreads();
  }
  // Work tiles (expert, first row, rows), bucket by bucket.
  if (tiles) {
    for (int e = threadIdx.x; e < experts; e += kGroupThreads) {
      const int c = start[e + 1] - start[e];
      for (int r = 0, t = tstart[e]; r < c; r += tile, ++t) {
        tiles[3 * t] = e;
        tiles[3 * t + 1] = start[e] + r;
        tiles[3 * t + 2] = min(tile, c - r);
      }
    }
  }
  // Positions past the pairs that were kept (only when ids were left out) point at pair 0, so every
  // entry of order stays a valid pair index.
  for (int pos = start[experts] + threadIdx.x; cap == 0 && pos < pairs; pos += kGroupThreads) {
    order[pos] = 0;
    if (local) local[pos] = 0;
  }

  // Pass 2: each warp places its own pairs, 32 at a time, in pair order.
  int32_t *my_cnt = warp_cnt + warp * experts;
  for (int base = lo, j = 0; base < hi; base += 32, ++j) {
    const int i = base + lane;
    int b = -1;
    if (j < kCache) {
#pragma unroll
      for (int c = 0; c < kCache; ++c)
        if (c == j) b = bc[c];
    } else if (i < hi) {
      b = bucket(i);
    }
    const unsigned same = __match_any_sync(0xffffffffu, b);
    const int rank = __popc(same & lt_mask);
    int pos = b >= 0 ? start[b] + my_cnt[b] + rank : 0;
    if (cap > 0 && b >= 0) {
      pos = my_cnt[b] + rank < cap ? b * cap + my_cnt[b] + rank : -1;
      if (pos < 0) raise_status(kStatusEpOverflow);
    }
    __syncwarp();
    if (b >= 0 && rank == 0) my_cnt[b] += __popc(same);
    __syncwarp();
    if (i < hi && (b < 0 || pos < 0)) slot_of[i] = -1;  // left out
    if (b >= 0 && pos >= 0) {
      order[pos] = i;
      slot_of[i] = pos;
      if (local) local[pos] = ids[i] - b * div;
    }
  }
}

// ---- gather: expert-sorted fp16 copies of the tokens' rows ---------------------------------------
// xg[s] = fp16(x[order[s] / topk]) (p_gather of lfm2moe/kernels/mk.mojo:164-176); order null: s / topk.
// perm: each 8 consecutive columns are stored in the k order 0, 4, 1, 5, 2, 6, 3, 7, the order in which
// the grouped products dequantise a weight word (gemm_q4.cu, dequant_word_perm).
__device__ __forceinline__ uint4 perm8(uint4 v) {  // halves 0..7 -> 0, 4, 1, 5, 2, 6, 3, 7
  return make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632), __byte_perm(v.y, v.w, 0x5410),
                    __byte_perm(v.y, v.w, 0x7632));
}

// valid (may be null): only the first *valid positions are copied (the pairs the grouping kept).
__global__ void gather_kernel(const void *__restrict__ x, int x_f16, const int32_t *__restrict__ order, int pairs,
                              int topk, int d, __half *__restrict__ xg, int perm = 0, const int32_t *valid = nullptr,
                              FlagWait wait = FlagWait()) {
  griddep_launch_dependents();
  griddep_wait();    // programmatic dependent launch: earlier work on the stream is complete
  wait_flags(wait);  // an expert-parallel owner: the senders' rows and ids have arrived
  const int vec = d / 8;  // 8 values per thread step
  const int64_t n = static_cast<int64_t>(valid ? min(*valid, pairs) : pairs) * vec;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < n;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(it / vec), c = static_cast<int>(it % vec) * 8;
    const int o = order ? order[s] : s;  // no order: the pairs in their own order
    if (o < 0) {  // an empty position of a fixed-capacity layout
      *reinterpret_cast<uint4 *>(xg + static_cast<size_t>(s) * d + c) = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    const int t = o / topk;
    uint4 out;
    if (x_f16) {
      out = *reinterpret_cast<const uint4 *>(static_cast<const __half *>(x) + static_cast<size_t>(t) * d + c);
    } else {
      const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(x) + static_cast<size_t>(t) * d + c);
      const float4 a = src[0], b = src[1];
      out = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y), pack_half2(b.z, b.w));
    }
    if (perm) out = perm8(out);
    *reinterpret_cast<uint4 *>(xg + static_cast<size_t>(s) * d + c) = out;
  }
}

// ---- the per-pair path of an expert-parallel owner: the first pairs of the grouped order, compacted --
// For s < n_out: xs[s] = rows[order[s]] (fp16, natural k order) and cid[s] = ids[order[s]] when s < *valid,
// cid[s] = -1 after. Does nothing when *valid > n_out (the grouped products have the work).
__global__ void small_gather_kernel(const __half *__restrict__ rows, const int32_t *__restrict__ order,
                                    const int32_t *__restrict__ ids, const int32_t *__restrict__ valid, int n_out, int d,
                                    __half *__restrict__ xs, int32_t *__restrict__ cid) {
  griddep_launch_dependents();
  griddep_wait();
  const int nv = *valid;
  if (nv > n_out) return;
  const int vec = d / 8;
  for (int it = blockIdx.x * blockDim.x + threadIdx.x; it < n_out * vec; it += gridDim.x * blockDim.x) {
    const int s = it / vec, c = (it % vec) * 8;
    if (c == 0) cid[s] = s < nv ? ids[order[s]] : -1;
    if (s < nv)
      *reinterpret_cast<uint4 *>(xs + static_cast<size_t>(s) * d + c) =
          *reinterpret_cast<const uint4 *>(rows + static_cast<size_t>(order[s]) * d + c);
  }
}

// ---- SwiGLU for the one-token path: a[k][j] = silu(h[k][j]) * h[k][fe + j] (moe_gate_up) -------
__global__ void silu_mul_kernel(const float *__restrict__ h, float *__restrict__ a, int rows, int fe) {
  griddep_launch_dependents();
  griddep_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows * fe; i += gridDim.x * blockDim.x) {
    const int r = i / fe, j = i % fe;
    const float g = h[static_cast<size_t>(r) * 2 * fe + j], u = h[static_cast<size_t>(r) * 2 * fe + fe + j];
    a[i] = g / (1.f + expf(-g)) * u;
  }
}

// ---- combine: y[t][c] (+)= sum_k w[t][k] * z[slot_of[t * topk + k]][c] (p_moe_sum, p_combine) -----
// The k terms are added in order k = 0 .. topk - 1, then added to y: deterministic.
__global__ void combine_kernel(const float *__restrict__ z, const int32_t *__restrict__ slot_of,
                               const float *__restrict__ w, int tokens, int topk, int d, int add, float *__restrict__ y,
                               FlagWait wait = FlagWait()) {
  griddep_launch_dependents();
  griddep_wait();
  wait_flags(wait);  // an expert-parallel sender: every owner's outputs have come back
  const int vec = d / 4;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < static_cast<int64_t>(tokens) * vec;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(it / vec), c = static_cast<int>(it % vec) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < topk; ++k) {
      const float wk = w[static_cast<size_t>(t) * topk + k];
      const int row = slot_of ? slot_of[static_cast<size_t>(t) * topk + k] : t * topk + k;
      if (row < 0) continue;  // a pair left out of the grouping (invalid expert id)
      const float4 v = *reinterpret_cast<const float4 *>(z + static_cast<size_t>(row) * d + c);
      acc.x += wk * v.x;
      acc.y += wk * v.y;
      acc.z += wk * v.z;
      acc.w += wk * v.w;
    }
    float4 *out = reinterpret_cast<float4 *>(y + static_cast<size_t>(t) * d + c);
    if (add) {
      const float4 o = *out;
      acc.x += o.x, acc.y += o.y, acc.z += o.z, acc.w += o.w;
    }
    *out = acc;
  }
}

inline int grid_for(int64_t work, int threads, const DeviceInfo &dev) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads, static_cast<int64_t>(dev.sms) * 8)));
}


// ---- router: logits[t][e] = W[e] . x[t], fp32 (gemv_f32 / p_gemv_f32, moek.mojo:143-153, 284-295) ----
// A CTA takes kRouterTokens tokens x 4 * PER experts; x arrives in shared memory 1024 k at a time;
// each warp owns PER experts. Per chunk a lane first loads its eight float4 of a W row (so their
// latencies overlap), then multiplies them with the chunk's tokens; the warp sums its lanes in a
// fixed order at the end. PER = 1 for a handful of tokens (more CTAs), 4 otherwise.
constexpr int kRouterTokens = 8, kRouterChunk = 1024, kRouterThreads = 128;

template <int PER>
__global__ void __launch_bounds__(kRouterThreads) router_kernel(const float *__restrict__ w, const float *__restrict__ x,
                                                                 float *__restrict__ logits, int tokens, int experts, int d) {
  __shared__ __align__(16) float xs[kRouterTokens][kRouterChunk];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int t0 = blockIdx.x * kRouterTokens, e0 = (blockIdx.y * (kRouterThreads / 32) + warp) * PER;
  float acc[PER][kRouterTokens];
#pragma unroll
  for (int e = 0; e < PER; ++e)
#pragma unroll
    for (int t = 0; t < kRouterTokens; ++t) acc[e][t] = 0.f;
  griddep_wait();
  for (int k0 = 0; k0 < d; k0 += kRouterChunk) {
    const int kn = min(kRouterChunk, d - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < kRouterTokens * kRouterChunk / 4; i += kRouterThreads) {
      const int t = i / (kRouterChunk / 4), k = (i % (kRouterChunk / 4)) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t0 + t < tokens && k < kn) v = *reinterpret_cast<const float4 *>(x + static_cast<size_t>(t0 + t) * d + k0 + k);
      *reinterpret_cast<float4 *>(&xs[t][k]) = v;
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const bool live = e0 + e < experts;
      const float *wr = w + static_cast<size_t>(live ? e0 + e : 0) * d + k0;
      float4 wv[kRouterChunk / 128];
#pragma unroll
      for (int j = 0; j < kRouterChunk / 128; ++j) {
        const int k = lane * 4 + 128 * j;
        wv[j] = live && k < kn ? __ldg(reinterpret_cast<const float4 *>(wr + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < kRouterChunk / 128; ++j) {
        const int k = lane * 4 + 128 * j;
#pragma unroll
        for (int t = 0; t < kRouterTokens; ++t) {
          const float4 xv = *reinterpret_cast<const float4 *>(&xs[t][k]);
          acc[e][t] = fmaf(wv[j].x, xv.x, fmaf(wv[j].y, xv.y, fmaf(wv[j].z, xv.z, fmaf(wv[j].w, xv.w, acc[e][t]))));
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < PER; ++e)
#pragma unroll
    for (int t = 0; t < kRouterTokens; ++t) {
      float v = acc[e][t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && e0 + e < experts && t0 + t < tokens) logits[static_cast<size_t>(t0 + t) * experts + e0 + e] = v;
    }
}

// ---- the fused router chain: router GEMV + top-k + softmax in one cluster kernel -------------
// A cluster of 8 CTAs takes TOK tokens (16, or 4 for a few tokens); CTA r computes the logits of
// experts [r * epc, (r + 1) * epc) (epc = ceil(E / 8) <= 32) for them and keeps them in its shared
// memory; after a cluster barrier each token is routed by one warp that reads its E logits from the
// eight CTAs' shared memory (distributed shared memory), so the logits never round-trip through
// global memory (they are written out only when asked for). The grouping (group_kernel) follows as
// a programmatic dependent launch. The router follows gemv_f32 / p_gemv_f32 (moek.mojo:143-153,
// 284-295), the routing route / p_route (moek.mojo:156-197, 385-425).
// The GEMV is register-blocked: a warp owns 8 tokens x 8 experts over a k range; per 128 k its lanes
// read 4 k of the 8 tokens and of the 8 expert rows from shared memory, so each load feeds 32 fused
// multiply-adds. x and the CTA's expert rows stream into shared memory 256 k at a time through a
// 3-stage ring of cp.async copies (the copies of later stages fly while a stage is multiplied). The
// CTA's warps split its experts into groups of 8 and each stage's k into kKG ranges; a warp's 64 sums
// are reduced across its lanes by a transposing butterfly, then the kKG partial sums of each logit
// are added in a fixed order.
constexpr int kRgCluster = 8, kRgThreads = 256, kRgTokens = 16, kRgChunk = 256, kRgStages = 3;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster: shared-memory writes before it are visible to the
// cluster's reads after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A float at the same shared-memory offset as `p` in CTA `rank` of this cluster.
__device__ __forceinline__ float ld_cluster_f32(const float *p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}
// 16 bytes global -> shared, asynchronously; src_bytes 0 fills the 16 bytes with zeros (src unread).
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 32 partial sums per lane -> lane l holds the warp total of sum l (a transposing butterfly: 31 shuffles).
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16, half = 16; o >= 1; o >>= 1, half >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = up ? v[i] : v[i + half];
      const float keep = up ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// Dynamic shared memory of route_group_kernel<XG>: the ring of (x, w) stages.
__host__ __device__ constexpr size_t rg_ring_bytes(int xg) {
  return static_cast<size_t>(kRgStages) * (kRgTokens + 8 * xg) * kRgChunk * sizeof(float);
}

template <int XG, int PER>  // expert groups of 8 per CTA (epc <= 8 * XG); logits per lane in routing (E <= 32 * PER)
__global__ void __cluster_dims__(kRgCluster, 1, 1) __launch_bounds__(kRgThreads)
    route_group_kernel(const float *__restrict__ w, const float *__restrict__ x, float *__restrict__ logits,
                       int32_t *__restrict__ ids, float *__restrict__ weights, int tokens, int experts, int topk, int d) {
  constexpr int kTG = kRgTokens / 8;                   // token groups of 8
  constexpr int kKG = (kRgThreads / 32) / (kTG * XG);  // k ranges (warps = kTG x XG x kKG)
  static_assert(kKG >= 1 && kTG * XG * kKG == kRgThreads / 32 && kRgChunk / kKG >= 128, "warp layout");
  constexpr int kRows = kRgTokens + 8 * XG;            // rows of a stage: the tokens, then the experts
  extern __shared__ __align__(16) float ring[];        // [stage][kRows][kRgChunk]
  __shared__ float part[kKG][kRgTokens][8 * XG];       // per k range: this CTA's logits
  __shared__ float lg[kRgTokens][32];                  // this CTA's experts' logits
  const uint32_t rank = cluster_ctarank();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tg = warp % kTG, xg = (warp / kTG) % XG, kg = warp / (kTG * XG);
  const int t0 = static_cast<int>(blockIdx.x / kRgCluster) * kRgTokens;
  const int epc = (experts + kRgCluster - 1) / kRgCluster, e_lo = static_cast<int>(rank) * epc;
  const int nchunks = (d + kRgChunk - 1) / kRgChunk;
  griddep_launch_dependents();
  griddep_wait();  // x may come from the previous kernel on the stream
  // Stage c of the ring: row r < kRgTokens is token t0 + r of x, row kRgTokens + j expert e_lo + j of w;
  // rows past the tokens, the CTA's experts or d are zero-filled.
  auto issue = [&](int c) {
    float *st = ring + static_cast<size_t>(c % kRgStages) * kRows * kRgChunk;
    const int k0 = c * kRgChunk;
    for (int i = threadIdx.x; i < kRows * (kRgChunk / 4); i += kRgThreads) {
      const int r = i / (kRgChunk / 4), k = (i % (kRgChunk / 4)) * 4;
      const float *src = x;
      bool live = k0 + k < d;
      if (r < kRgTokens) {
        live = live && t0 + r < tokens;
        if (live) src = x + static_cast<size_t>(t0 + r) * d + k0 + k;
      } else {
        const int le = r - kRgTokens, e = e_lo + le;
        live = live && le < epc && e < experts;
        if (live) src = w + static_cast<size_t>(e) * d + k0 + k;
      }
      cp_async16(st + r * kRgChunk + k, src, live ? 16u : 0u);
    }
  };
#pragma unroll
  for (int c = 0; c < kRgStages - 1; ++c) {
    if (c < nchunks) issue(c);
    cp_async_commit();
  }
  float acc[8][8];  // [expert][token]
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[j][t] = 0.f;
  constexpr int kSpan = kRgChunk / kKG;  // k of a stage per k range
  for (int c = 0; c < nchunks; ++c) {
    if (c + kRgStages - 1 < nchunks) issue(c + kRgStages - 1);
    cp_async_commit();
    cp_async_wait<kRgStages - 1>();  // this thread's copies of stage c landed
    __syncthreads();                 // ... and every thread's
    const float *st = ring + static_cast<size_t>(c % kRgStages) * kRows * kRgChunk;
#pragma unroll
    for (int q = 0; q < kSpan / 128; ++q) {
      const int k = kg * kSpan + lane * 4 + 128 * q;
      float4 wv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = *reinterpret_cast<const float4 *>(st + (kRgTokens + xg * 8 + j) * kRgChunk + k);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float4 xv = *reinterpret_cast<const float4 *>(st + (tg * 8 + t) * kRgChunk + k);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          acc[j][t] = fmaf(wv[j].x, xv.x, fmaf(wv[j].y, xv.y, fmaf(wv[j].z, xv.z, fmaf(wv[j].w, xv.w, acc[j][t]))));
      }
    }
    __syncthreads();  // stage c is free for the copies issued next
  }
  cp_async_wait<0>();
  // lanes -> one sum per (expert, token): two transposing butterflies of 32
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = acc[4 * h + i / 8][i % 8];
    const float total = warp_transpose_sum32(v, lane);  // expert 4 h + lane / 8, token lane % 8
    part[kg][tg * 8 + lane % 8][xg * 8 + 4 * h + lane / 8] = total;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kRgTokens * epc; i += kRgThreads) {
    const int t = i / epc, le = i % epc, e = e_lo + le;
    if (e >= experts) continue;
    float v = part[0][t][le];
#pragma unroll
    for (int g = 1; g < kKG; ++g) v += part[g][t][le];
    lg[t][le] = v;
    if (logits && t0 + t < tokens) logits[static_cast<size_t>(t0 + t) * experts + e] = v;
  }
  cluster_sync();
  // Routing: token t0 + tt by warp tt / 8 of CTA tt % 8, its logits gathered from the eight CTAs.
  const int tt = static_cast<int>(rank) + kRgCluster * warp;
  if (tt < kRgTokens && t0 + tt < tokens) {
    float v[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      v[i] = e < experts ? ld_cluster_f32(&lg[tt][e % epc], static_cast<uint32_t>(e / epc)) : -INFINITY;
    }
    route_row<PER>(v, lane, experts, topk, ids + static_cast<size_t>(t0 + tt) * topk,
                   weights + static_cast<size_t>(t0 + tt) * topk);
  }
  cluster_sync();  // no CTA leaves while another may still read its logits
}

}  // namespace moe
}  // namespace mq

extern "C" int mq_moe_router(const float *w, const float *x, float *logits, int64_t tokens, int experts, int64_t d,
                             void *stream) {
  MQ_REQUIRE(w && x && logits, MQ_EINVAL, "mq_moe_router: null pointer");
  MQ_REQUIRE(tokens > 0 && tokens < (1 << 24) && experts >= 1 && experts <= 4096 && d > 0 && d % 4 == 0 && d < (1 << 24),
             MQ_EINVAL, "mq_moe_router: bad shape (d must be a multiple of 4)");
  MQ_REQUIRE(mq::aligned(w, 16) && mq::aligned(x, 16) && mq::aligned(logits, 4), MQ_EALIGN,
             "mq_moe_router: w and x must be 16-byte aligned");
  const unsigned tt = static_cast<unsigned>((tokens + mq::moe::kRouterTokens - 1) / mq::moe::kRouterTokens);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int warps = mq::moe::kRouterThreads / 32;
  if (tokens <= 4 * mq::moe::kRouterTokens)  // few tokens: one expert per warp, more CTAs
    return mq::launch_overlapped(mq::moe::router_kernel<1>, dim3(tt, (experts + warps - 1) / warps),
                                 dim3(mq::moe::kRouterThreads), 0, st, "mq_moe_router", w, x, logits,
                                 static_cast<int>(tokens), experts, static_cast<int>(d));
  return mq::launch_overlapped(mq::moe::router_kernel<4>, dim3(tt, (experts + 4 * warps - 1) / (4 * warps)),
                               dim3(mq::moe::kRouterThreads), 0, st, "mq_moe_router", w, x, logits,
                               static_cast<int>(tokens), experts, static_cast<int>(d));
}

extern "C" int mq_moe_route(const float *logits, int32_t *ids, float *weights, int64_t tokens, int experts, int topk,
                            void *stream) {
  MQ_REQUIRE(logits && ids && weights, MQ_EINVAL, "mq_moe_route: null pointer");
  MQ_REQUIRE(tokens > 0 && tokens < (1 << 24), MQ_EINVAL, "mq_moe_route: bad token count %lld", static_cast<long long>(tokens));
  MQ_REQUIRE(experts >= 1 && experts <= 256, MQ_EINVAL, "mq_moe_route: experts must be in 1..256 (got %d)", experts);
  MQ_REQUIRE(topk >= 1 && topk <= 32 && topk <= experts, MQ_EINVAL, "mq_moe_route: topk must be in 1..min(32, experts)");
  const int threads = 256, per_block = threads / 32;
  const int grid = static_cast<int>((tokens + per_block - 1) / per_block);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int per = (experts + 31) / 32;
  if (per <= 4)
    mq::moe::route_kernel<4><<<grid, threads, 0, s>>>(logits, ids, weights, static_cast<int>(tokens), experts, topk);
  else
    mq::moe::route_kernel<8><<<grid, threads, 0, s>>>(logits, ids, weights, static_cast<int>(tokens), experts, topk);
  return mq::check_launch("mq_moe_route");
}

namespace mq {
namespace moe {
// The fused router chain on `stream`: route_group_kernel, then (counts != null) group_kernel as a
// programmatic dependent launch. Shapes are checked by the callers.
int route_cluster(const float *w, const float *x, float *logits, int32_t *ids, float *weights, int64_t tokens,
                  int experts, int topk, int64_t d, cudaStream_t s);

// scratch (may be null): room for tokens x experts fp32 logits. A few tokens (decode) with somewhere
// to put the logits run the router GEMV over more CTAs (router_kernel: one expert per warp, 32 CTAs
// for 128 experts) and route_kernel instead of the cluster kernel, which would spend a 16-token tile
// of work and one 8-SM cluster on them.
int route_group(const float *w, const float *x, float *logits, int32_t *ids, float *weights, int64_t tokens,
                int experts, int topk, int64_t d, int tile, int32_t *counts, int32_t *offsets, int32_t *order,
                int32_t *slot_of, int32_t *tiles, int32_t *ntiles, cudaStream_t s, float *scratch = nullptr) {
  float *lbuf = logits ? logits : scratch;
  if (tokens <= 4 && lbuf) {
    const int warps = kRouterThreads / 32;
    if (int rc = launch_overlapped(router_kernel<1>, dim3(static_cast<unsigned>((tokens + kRouterTokens - 1) / kRouterTokens),
                                                         (experts + warps - 1) / warps),
                                   dim3(kRouterThreads), 0, s, "mq_moe_route_group (router)", w, x, lbuf,
                                   static_cast<int>(tokens), experts, static_cast<int>(d)))
      return rc;
    const int per_block = 256 / 32, grid = static_cast<int>((tokens + per_block - 1) / per_block);
    if (experts <= 128)
      route_kernel<4><<<grid, 256, 0, s>>>(lbuf, ids, weights, static_cast<int>(tokens), experts, topk);
    else
      route_kernel<8><<<grid, 256, 0, s>>>(lbuf, ids, weights, static_cast<int>(tokens), experts, topk);
    if (int rc = check_launch("mq_moe_route_group (route)")) return rc;
  } else {
    if (int rc = route_cluster(w, x, logits, ids, weights, tokens, experts, topk, d, s)) return rc;
  }
  if (!counts) return MQ_OK;
  const size_t smem = (32 * experts + 2 * (experts + 1)) * sizeof(int32_t);
  const int32_t *cids = ids;
  int32_t *no_local = nullptr;
  return launch_overlapped(group_kernel, dim3(1), dim3(kGroupThreads), smem, s, "mq_moe_route_group (grouping)", cids, 1,
                           static_cast<int>(tokens * topk), experts, tile, counts, offsets, order, slot_of, tiles, ntiles,
                           no_local, 0, FlagWait(), 0);
}

// The cluster kernel: router GEMV, top-k and softmax in one launch.
int route_cluster(const float *w, const float *x, float *logits, int32_t *ids, float *weights, int64_t tokens,
                  int experts, int topk, int64_t d, cudaStream_t s) {
  const int epc = (experts + kRgCluster - 1) / kRgCluster;  // <= 32
  const unsigned grid = static_cast<unsigned>((tokens + kRgTokens - 1) / kRgTokens) * kRgCluster;
  const int ti = static_cast<int>(tokens), ei = experts, di = static_cast<int>(d);
  const char *what = "mq_moe_route_group";
  int rc;
  auto go = [&](auto kern, int xg) {
    const size_t smem = rg_ring_bytes(xg);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
      return fail(MQ_ECUDA, "mq_moe_route_group: shared memory attribute");
    return launch_overlapped(kern, dim3(grid), dim3(kRgThreads), smem, s, what, w, x, logits, ids, weights, ti, ei, topk,
                             di);
  };
  if (epc <= 16 && experts <= 128)  // (fewer experts leave rows of the CTA's two groups of 8 empty)
    rc = go(route_group_kernel<2, 4>, 2);
  else
    rc = go(route_group_kernel<4, 8>, 4);
  return rc;
}
}  // namespace moe
}  // namespace mq

extern "C" int mq_moe_route_group(const float *w, const float *x, float *logits, int32_t *ids, float *weights,
                                  int64_t tokens, int experts, int topk, int64_t d, int tile, int32_t *counts,
                                  int32_t *offsets, int32_t *order, int32_t *slot_of, int32_t *tiles, int32_t *ntiles,
                                  void *stream) {
  MQ_REQUIRE(w && x && ids && weights, MQ_EINVAL, "mq_moe_route_group: null pointer");
  MQ_REQUIRE(!counts || (offsets && order && slot_of && tiles && ntiles), MQ_EINVAL,
             "mq_moe_route_group: the grouping outputs are all given or counts is null");
  MQ_REQUIRE(tokens > 0 && tokens < (1 << 24) && tokens * topk < (1 << 30), MQ_EINVAL, "mq_moe_route_group: bad token count");
  MQ_REQUIRE(experts >= 1 && experts <= 256, MQ_EINVAL, "mq_moe_route_group: experts must be in 1..256 (got %d)", experts);
  MQ_REQUIRE(topk >= 1 && topk <= 32 && topk <= experts, MQ_EINVAL, "mq_moe_route_group: topk must be in 1..min(32, experts)");
  MQ_REQUIRE(d > 0 && d % 4 == 0 && d < (1 << 24), MQ_EINVAL, "mq_moe_route_group: d must be a positive multiple of 4");
  MQ_REQUIRE(tile >= 1, MQ_EINVAL, "mq_moe_route_group: tile must be >= 1");
  MQ_REQUIRE(mq::aligned(w, 16) && mq::aligned(x, 16), MQ_EALIGN, "mq_moe_route_group: w and x must be 16-byte aligned");
  return mq::moe::route_group(w, x, logits, ids, weights, tokens, experts, topk, d, tile, counts, offsets, order,
                              slot_of, tiles, ntiles, static_cast<cudaStream_t>(stream));
}

extern "C" int mq_moe_group(const int32_t *ids, int64_t tokens, int topk, int experts, int tile, int32_t *counts,
                            int32_t *offsets, int32_t *order, int32_t *slot_of, int32_t *tiles, int32_t *ntiles,
                            void *stream) {
  MQ_REQUIRE(ids && counts && offsets && order && slot_of && tiles && ntiles, MQ_EINVAL, "mq_moe_group: null pointer");
  MQ_REQUIRE(tokens > 0 && topk >= 1 && tokens * topk < (1 << 30), MQ_EINVAL, "mq_moe_group: bad tokens / topk");
  MQ_REQUIRE(experts >= 1 && experts <= 256, MQ_EINVAL, "mq_moe_group: experts must be in 1..256");
  MQ_REQUIRE(tile >= 1, MQ_EINVAL, "mq_moe_group: tile must be >= 1");
  const size_t smem = (32 * experts + 2 * (experts + 1)) * sizeof(int32_t);
  mq::moe::group_kernel<<<1, mq::moe::kGroupThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      ids, 1, static_cast<int>(tokens * topk), experts, tile, counts, offsets, order, slot_of, tiles, ntiles, nullptr, 0);
  return mq::check_launch("mq_moe_group");
}

extern "C" int mq_ep_plan(const int32_t *ids, int64_t tokens, int topk, int experts, int world, int capacity,
                          int32_t *counts, int32_t *offsets, int32_t *order, int32_t *slot_of, int32_t *local_ids,
                          void *stream) {
  MQ_REQUIRE(ids && counts && offsets && order && slot_of && local_ids, MQ_EINVAL, "mq_ep_plan: null pointer");
  MQ_REQUIRE(tokens > 0 && topk >= 1 && tokens * topk < (1 << 30), MQ_EINVAL, "mq_ep_plan: bad tokens / topk");
  MQ_REQUIRE(world >= 1 && world <= 256 && experts >= world && experts % world == 0, MQ_EINVAL,
             "mq_ep_plan: experts (%d) must be a positive multiple of world (%d)", experts, world);
  MQ_REQUIRE(capacity >= 0 && static_cast<int64_t>(capacity) * world < (1 << 30), MQ_EINVAL,
             "mq_ep_plan: bad capacity %d", capacity);
  const size_t smem = (32 * world + 2 * (world + 1)) * sizeof(int32_t);
  int32_t *no_tiles = nullptr;
  return mq::launch_overlapped(mq::moe::group_kernel, dim3(1), dim3(mq::moe::kGroupThreads), smem,
                               static_cast<cudaStream_t>(stream), "mq_ep_plan", ids, experts / world,
                               static_cast<int>(tokens * topk), world, 1, counts, offsets, order, slot_of, no_tiles,
                               no_tiles, local_ids, capacity, mq::FlagWait(), 0);
}

extern "C" int mq_moe_gather(const void *x, int x_dtype, const int32_t *order, int64_t pairs, int topk, int64_t d,
                             uint16_t *xg, void *stream) {
  MQ_REQUIRE(x && order && xg, MQ_EINVAL, "mq_moe_gather: null pointer");
  MQ_REQUIRE(pairs > 0 && d > 0 && d % 8 == 0 && topk >= 1, MQ_EINVAL, "mq_moe_gather: d must be a multiple of 8");
  MQ_REQUIRE(mq::aligned(x, 16) && mq::aligned(xg, 16), MQ_EALIGN, "mq_moe_gather: x and xg must be 16-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  mq::moe::gather_kernel<<<mq::moe::grid_for(pairs * (d / 8), 256, dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_dtype == MQ_F16, order, static_cast<int>(pairs), topk, static_cast<int>(d), reinterpret_cast<__half *>(xg));
  return mq::check_launch("mq_moe_gather");
}

extern "C" int mq_moe_silu_mul(const float *h, float *a, int64_t rows, int64_t fe, void *stream) {
  MQ_REQUIRE(h && a && rows > 0 && fe > 0, MQ_EINVAL, "mq_moe_silu_mul: bad arguments");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  mq::moe::silu_mul_kernel<<<mq::moe::grid_for(rows * fe, 256, dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      h, a, static_cast<int>(rows), static_cast<int>(fe));
  return mq::check_launch("mq_moe_silu_mul");
}

extern "C" int mq_moe_combine(const float *z, const int32_t *slot_of, const float *weights, int64_t tokens, int topk,
                              int64_t d, int add, float *y, void *stream) {
  MQ_REQUIRE(z && weights && y, MQ_EINVAL, "mq_moe_combine: null pointer");
  MQ_REQUIRE(tokens > 0 && topk >= 1 && d > 0 && d % 4 == 0, MQ_EINVAL, "mq_moe_combine: d must be a multiple of 4");
  MQ_REQUIRE(mq::aligned(z, 16) && mq::aligned(y, 16), MQ_EALIGN, "mq_moe_combine: z and y must be 16-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  return mq::launch_overlapped(mq::moe::combine_kernel, dim3(mq::moe::grid_for(tokens * (d / 4), 256, dev)), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), "mq_moe_combine", z, slot_of, weights,
                               static_cast<int>(tokens), topk, static_cast<int>(d), static_cast<int>(add != 0), y,
                               mq::FlagWait());
}

namespace mq {
namespace moe {

constexpr int kTileM = 64;  // tokens per expert work tile in the grouped GEMMs
constexpr int kSmallPairs = 16;  // up to this many (token, expert) pairs the layer runs on the streaming GEMVs

struct Work {
  int32_t *counts, *offsets, *order, *slot_of, *tiles, *ntiles;
  __half *xg, *a;
  float *z;
  size_t bytes;
  int max_tiles;
};

inline size_t align_up(size_t v) { return (v + 255) / 256 * 256; }

// Carves the caller's workspace (pointer may be null to only size it).
inline Work carve(uint8_t *base, int64_t tokens, int experts, int topk, int64_t d, int64_t fe) {
  Work w{};
  const int64_t P = tokens * topk;
  // tiles = sum over the touched experts of ceil(count / kTileM) <= touched + P / kTileM, touched <= min(experts, P)
  w.max_tiles = static_cast<int>(std::min<int64_t>(experts, P) + (P + kTileM - 1) / kTileM);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t *p = base ? base + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  w.counts = reinterpret_cast<int32_t *>(take(experts * 4));
  w.offsets = reinterpret_cast<int32_t *>(take((experts + 1) * 4));
  w.order = reinterpret_cast<int32_t *>(take(P * 4));
  w.slot_of = reinterpret_cast<int32_t *>(take(P * 4));
  w.tiles = reinterpret_cast<int32_t *>(take(static_cast<size_t>(w.max_tiles) * 3 * 4));
  w.ntiles = reinterpret_cast<int32_t *>(take(4));
  w.xg = reinterpret_cast<__half *>(take(P * d * 2));
  w.a = reinterpret_cast<__half *>(take(P * fe * 4));  // fp16 between the grouped GEMMs; fp32 on the decode path
  w.z = reinterpret_cast<float *>(take(P * (d > 2 * fe ? d : 2 * fe) * 4));
  w.bytes = off;
  return w;
}

}  // namespace moe
}  // namespace mq

extern "C" size_t mq_moe_workspace_size(int64_t tokens, int experts, int topk, int64_t d, int64_t fe) {
  if (tokens <= 0 || experts <= 0 || topk <= 0 || d <= 0 || fe <= 0) return 0;
  return mq::moe::carve(nullptr, tokens, experts, topk, d, fe).bytes;
}

namespace mq {
namespace moe {

// The experts of the layer on P = tokens * topk pairs (ids -1: no expert, skipped): z_out receives the
// expert outputs (fp32 rows of d) and slot_of_out the row of pair p in them (null: row p). Up to
// small_pairs pairs run on the streaming GEMVs (each pair's own x), more on grouping + gather + the
// two grouped tensor-core products (the activations in their dequantisation k order).
int experts(const void *x, int x_dtype, const int32_t *ids, const uint32_t *gu_wq, const uint16_t *gu_ws,
            const uint32_t *dn_wq, const uint16_t *dn_ws, int64_t tokens, int experts_n, int topk, int64_t d, int64_t fe,
            int group, const Work &w, cudaStream_t s, int64_t small_pairs, const float **z_out,
            const int32_t **slot_of_out, FlagWait wait = FlagWait(), bool grouped = false) {
  const int64_t P = tokens * topk;
  DeviceInfo dev;
  if (int rc = device_info(&dev)) return rc;
  if (P <= small_pairs) {
    float *a = reinterpret_cast<float *>(w.a), *z = w.z;
    const int32_t *no_order = nullptr;
    if (int rc = launch_overlapped(gather_kernel, dim3(grid_for(P * (d / 8), 256, dev)), dim3(256), 0, s,
                                   "mq_moe_forward gather", x, static_cast<int>(x_dtype == MQ_F16), no_order,
                                   static_cast<int>(P), topk, static_cast<int>(d), w.xg, 0, no_order, wait))
      return rc;
    if (int rc = gemv::gemv_q4_grouped(gu_wq, gu_ws, experts_n * 2 * fe, w.xg, a, ids, static_cast<int>(P),
                                       static_cast<int>(2 * fe), static_cast<int>(fe), d, group, 1, s, 1, 1))
      return rc;
    if (int rc = gemv::gemv_q4_grouped(dn_wq, dn_ws, experts_n * d, a, z, ids, static_cast<int>(P), static_cast<int>(d),
                                       static_cast<int>(d), fe, group, 1, s, 0, 0))
      return rc;
    *z_out = z;
    *slot_of_out = nullptr;
    return MQ_OK;
  }
  if (!grouped) {  // grouped: the fused router chain already wrote the grouping into w
    const size_t smem = (32 * experts_n + 2 * (experts_n + 1)) * sizeof(int32_t);
    int32_t *no_local = nullptr;
    if (int rc = launch_overlapped(group_kernel, dim3(1), dim3(kGroupThreads), smem, s, "mq_moe_forward group", ids, 1,
                                   static_cast<int>(P), experts_n, kTileM, w.counts, w.offsets, w.order, w.slot_of,
                                   w.tiles, w.ntiles, no_local, 0, wait, 0))
      return rc;
  }
  // The activations and the SwiGLU outputs travel in the products' dequantisation k order (perm); only
  // the pairs the grouping kept are gathered (offsets[experts] of them).
  if (int rc = launch_overlapped(gather_kernel, dim3(grid_for(P * (d / 8), 256, dev)), dim3(256), 0, s,
                                 "mq_moe_forward gather", x, static_cast<int>(x_dtype == MQ_F16), w.order,
                                 static_cast<int>(P), topk, static_cast<int>(d), w.xg, 1, w.offsets + experts_n,
                                 FlagWait()))
    return rc;
  if (int rc = moe_gemm_run(1, gu_wq, gu_ws, reinterpret_cast<const uint16_t *>(w.xg), P, d, experts_n, 2 * fe, group,
                            w.tiles, w.ntiles, w.max_tiles, kTileM, w.a, s, 1))
    return rc;
  if (int rc = moe_gemm_run(2, dn_wq, dn_ws, reinterpret_cast<const uint16_t *>(w.a), P, fe, experts_n, d, group, w.tiles,
                            w.ntiles, w.max_tiles, kTileM, w.z, s, 1))
    return rc;
  *z_out = w.z;
  *slot_of_out = w.slot_of;
  return MQ_OK;
}

}  // namespace moe
}  // namespace mq

extern "C" int mq_moe_forward(const void *x, int x_dtype, const int32_t *ids, const float *weights, const uint32_t *gu_wq,
                              const uint16_t *gu_ws, const uint32_t *dn_wq, const uint16_t *dn_ws, float *y, int64_t tokens,
                              int experts, int topk, int64_t d, int64_t fe, int group, int add, void *workspace,
                              size_t workspace_bytes, void *stream) {
  MQ_REQUIRE(x && ids && weights && gu_wq && gu_ws && dn_wq && dn_ws && y, MQ_EINVAL, "mq_moe_forward: null pointer");
  MQ_REQUIRE(tokens > 0 && experts >= 1 && experts <= 256 && topk >= 1 && topk <= experts, MQ_EINVAL,
             "mq_moe_forward: bad tokens / experts / topk");
  MQ_REQUIRE(d % 256 == 0 && fe % 256 == 0, MQ_EINVAL, "mq_moe_forward: d and fe must be multiples of 256");
  MQ_REQUIRE(x_dtype == MQ_F32 || x_dtype == MQ_F16, MQ_EINVAL, "mq_moe_forward: x_dtype must be MQ_F32 or MQ_F16");
  const mq::moe::Work need = mq::moe::carve(nullptr, tokens, experts, topk, d, fe);
  MQ_REQUIRE(workspace && workspace_bytes >= need.bytes, MQ_EINVAL, "mq_moe_forward: needs a workspace of %zu bytes (got %zu)",
             need.bytes, workspace_bytes);
  MQ_REQUIRE(mq::aligned(workspace, 256), MQ_EALIGN, "mq_moe_forward: workspace must be 256-byte aligned");
  const mq::moe::Work w = mq::moe::carve(static_cast<uint8_t *>(workspace), tokens, experts, topk, d, fe);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (tokens == 1 && x_dtype == MQ_F32) {
    // One token (decode): the streaming GEMV over the selected experts' rows, as moe_gate_up /
    // moe_down do (moek.mojo:200-223): a = silu(gate_e x) * (up_e x) in one launch, z_k = down_e a_k,
    // y (+)= sum_k w_k z_k.
    float *a = reinterpret_cast<float *>(w.a), *z = w.z;
    if (int rc = mq::gemv::gemv_q4_grouped(gu_wq, gu_ws, experts * 2 * fe, x, a, ids, topk, static_cast<int>(2 * fe),
                                           static_cast<int>(fe), d, group, 0, s, 1, 0))
      return rc;
    if (int rc = mq::gemv::gemv_q4_grouped(dn_wq, dn_ws, experts * d, a, z, ids, topk, static_cast<int>(d),
                                           static_cast<int>(d), fe, group, 1, s, 0, 0))
      return rc;
    return mq_moe_combine(z, nullptr, weights, 1, topk, d, add, y, s);
  }
  // Up to kSmallPairs pairs (a small decode batch, an expert-parallel rank's share of one token) run
  // on the streaming GEMVs with each pair's own fp16 x instead of tensor-core tiles they would barely fill.
  const float *z = nullptr;
  const int32_t *slot_of = nullptr;
  if (int rc = mq::moe::experts(x, x_dtype, ids, gu_wq, gu_ws, dn_wq, dn_ws, tokens, experts, topk, d, fe, group, w, s,
                                mq::moe::kSmallPairs, &z, &slot_of))
    return rc;
  return mq_moe_combine(z, slot_of, weights, tokens, topk, d, add, y, s);
}

extern "C" int mq_moe_layer(const float *x, const float *router_w, const uint32_t *gu_wq, const uint16_t *gu_ws,
                            const uint32_t *dn_wq, const uint16_t *dn_ws, float *y, int32_t *ids, float *weights,
                            float *logits, int64_t tokens, int experts, int topk, int64_t d, int64_t fe, int group, int add,
                            void *workspace, size_t workspace_bytes, void *stream) {
  MQ_REQUIRE(x && router_w && gu_wq && gu_ws && dn_wq && dn_ws && y && ids && weights, MQ_EINVAL, "mq_moe_layer: null pointer");
  MQ_REQUIRE(tokens > 0 && tokens < (1 << 24) && experts >= 1 && experts <= 256 && topk >= 1 && topk <= 32 && topk <= experts,
             MQ_EINVAL, "mq_moe_layer: bad tokens / experts / topk");
  MQ_REQUIRE(d % 256 == 0 && fe % 256 == 0 && d < (1 << 24), MQ_EINVAL, "mq_moe_layer: d and fe must be multiples of 256");
  MQ_REQUIRE(mq::aligned(x, 16) && mq::aligned(router_w, 16), MQ_EALIGN, "mq_moe_layer: x and router_w must be 16-byte aligned");
  const mq::moe::Work need = mq::moe::carve(nullptr, tokens, experts, topk, d, fe);
  MQ_REQUIRE(workspace && workspace_bytes >= need.bytes, MQ_EINVAL, "mq_moe_layer: needs a workspace of %zu bytes (got %zu)",
             need.bytes, workspace_bytes);
  MQ_REQUIRE(mq::aligned(workspace, 256), MQ_EALIGN, "mq_moe_layer: workspace must be 256-byte aligned");
  const mq::moe::Work w = mq::moe::carve(static_cast<uint8_t *>(workspace), tokens, experts, topk, d, fe);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t P = tokens * topk;
  // The grouping is needed only by the grouped tensor-core products (more than kSmallPairs pairs).
  const bool grouped = tokens > 1 && P > mq::moe::kSmallPairs;
  if (int rc = mq::moe::route_group(router_w, x, logits, ids, weights, tokens, experts, topk, d, mq::moe::kTileM,
                                    grouped ? w.counts : nullptr, w.offsets, w.order, w.slot_of, w.tiles, w.ntiles, s,
                                    w.z))
    return rc;
  if (tokens == 1) {  // decode: the streaming GEMVs over the selected experts' rows (as mq_moe_forward)
    float *a = reinterpret_cast<float *>(w.a), *z = w.z;
    if (int rc = mq::gemv::gemv_q4_grouped(gu_wq, gu_ws, experts * 2 * fe, x, a, ids, topk, static_cast<int>(2 * fe),
                                           static_cast<int>(fe), d, group, 0, s, 1, 0))
      return rc;
    if (int rc = mq::gemv::gemv_q4_grouped(dn_wq, dn_ws, experts * d, a, z, ids, topk, static_cast<int>(d),
                                           static_cast<int>(d), fe, group, 1, s, 0, 0))
      return rc;
    return mq_moe_combine(z, nullptr, weights, 1, topk, d, add, y, s);
  }
  const float *z = nullptr;
  const int32_t *slot_of = nullptr;
  if (int rc = mq::moe::experts(x, MQ_F32, ids, gu_wq, gu_ws, dn_wq, dn_ws, tokens, experts, topk, d, fe, group, w, s,
                                mq::moe::kSmallPairs, &z, &slot_of, mq::FlagWait(), grouped))
    return rc;
  return mq_moe_combine(z, slot_of, weights, tokens, topk, d, add, y, s);
}

namespace mq {
namespace moe {
constexpr int kEpSmall = 16;  // an owner with at most this many pairs runs them on per-pair GEMVs
// The per-pair path's buffers after the layer's workspace: compacted rows [kEpSmall][d] fp16, their
// expert ids [kEpSmall], SwiGLU outputs [kEpSmall][fe] fp32.
inline size_t ep_small_bytes(int64_t d, int64_t fe) {
  return align_up(kEpSmall * d * 2) + align_up(kEpSmall * 4) + align_up(kEpSmall * fe * 4);
}
}  // namespace moe
}  // namespace mq

extern "C" size_t mq_ep_workspace_size(int64_t rows, int experts, int64_t d, int64_t fe) {
  if (rows <= 0 || experts <= 0 || d <= 0 || fe <= 0) return 0;
  return mq_moe_workspace_size(rows, experts, 1, d, fe) + mq::moe::ep_small_bytes(d, fe);
}

extern "C" int mq_ep_expert_step(const uint16_t *rows, const int32_t *ids, const uint32_t *gu_wq, const uint16_t *gu_ws,
                                 const uint32_t *dn_wq, const uint16_t *dn_ws, int64_t nrows, int experts, int64_t d,
                                 int64_t fe, int group, int world, int rank, int cap, float *const *peer_ret,
                                 const int *flags, int *const *peer_flags, const int *epoch, int *done, void *workspace,
                                 size_t workspace_bytes, void *stream) {
  MQ_REQUIRE(rows && ids && gu_wq && gu_ws && dn_wq && dn_ws && peer_ret && flags && peer_flags && epoch && done,
             MQ_EINVAL, "mq_ep_expert_step: null pointer");
  MQ_REQUIRE(nrows == static_cast<int64_t>(world) * cap && nrows > 0, MQ_EINVAL,
             "mq_ep_expert_step: nrows must be world * cap");
  MQ_REQUIRE(experts >= 1 && experts <= 256 && d % 256 == 0 && fe % 256 == 0, MQ_EINVAL,
             "mq_ep_expert_step: bad experts, d or fe");
  const mq::moe::Work need = mq::moe::carve(nullptr, nrows, experts, 1, d, fe);
  const size_t total = need.bytes + mq::moe::ep_small_bytes(d, fe);
  MQ_REQUIRE(workspace && workspace_bytes >= total && mq::aligned(workspace, 256), MQ_EINVAL,
             "mq_ep_expert_step: needs a 256-byte aligned workspace of %zu bytes", total);
  const mq::moe::Work w = mq::moe::carve(static_cast<uint8_t *>(workspace), nrows, experts, 1, d, fe);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Both paths of the layer are on the stream, chosen on the device by the number of pairs that
  // arrived (the host cannot know it): the grouping hands out no tiles when at most kEpSmall pairs
  // came (the grouped products then exit at once), and the per-pair GEMVs exit when more came. A few
  // pairs (decode) thus cost per-pair GEMVs over only the real rows; many cost the tensor-core tiles.
  using mq::moe::kEpSmall;
  const int64_t P = nrows;
  mq::FlagWait wait;  // the senders' rows: the grouping (the first kernel) waits for them
  wait.flags = flags;
  wait.which = 0;
  wait.world = world;
  wait.epoch = epoch;
  const int32_t *valid = w.offsets + experts;
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  {
    const size_t smem = (32 * experts + 2 * (experts + 1)) * sizeof(int32_t);
    int32_t *no_local = nullptr;
    if (int rc = mq::launch_overlapped(mq::moe::group_kernel, dim3(1), dim3(mq::moe::kGroupThreads), smem, s,
                                       "mq_ep_expert_step group", ids, 1, static_cast<int>(P), experts, mq::moe::kTileM,
                                       w.counts, w.offsets, w.order, w.slot_of, w.tiles, w.ntiles, no_local, 0, wait,
                                       kEpSmall))
      return rc;
  }
  // per-pair path: its buffers after the layer's workspace
  uint8_t *small = static_cast<uint8_t *>(workspace) + need.bytes;
  __half *xs = reinterpret_cast<__half *>(small);
  int32_t *cid = reinterpret_cast<int32_t *>(small + mq::moe::align_up(kEpSmall * d * 2));
  float *a32 = reinterpret_cast<float *>(small + mq::moe::align_up(kEpSmall * d * 2) + mq::moe::align_up(kEpSmall * 4));
  if (int rc = mq::launch_overlapped(mq::moe::small_gather_kernel,
                                     dim3(mq::moe::grid_for(std::min<int64_t>(kEpSmall, P) * (d / 8), 256, dev)), dim3(256),
                                     0, s, "mq_ep_expert_step small gather", reinterpret_cast<const __half *>(rows),
                                     w.order, ids, valid, static_cast<int>(std::min<int64_t>(kEpSmall, P)),
                                     static_cast<int>(d), xs, cid))
    return rc;
  const int nsmall = static_cast<int>(std::min<int64_t>(kEpSmall, P));
  if (int rc = mq::gemv::gemv_q4_grouped(gu_wq, gu_ws, experts * 2 * fe, xs, a32, cid, nsmall, static_cast<int>(2 * fe),
                                         static_cast<int>(fe), d, group, 1, s, 1, 1, valid, nsmall))
    return rc;
  if (int rc = mq::gemv::gemv_q4_grouped(dn_wq, dn_ws, experts * d, a32, w.z, cid, nsmall, static_cast<int>(d),
                                         static_cast<int>(d), fe, group, 1, s, 0, 0, valid, nsmall))
    return rc;
  if (P <= kEpSmall) {  // never more than kEpSmall pairs: the grouped path has nothing to do
    return mq_ep_return(w.z, w.slot_of, ids, d, world, rank, cap, peer_ret, peer_flags, epoch, done, s);
  }
  // grouped path (no tiles when the per-pair path ran): activations in the products' k order
  if (int rc = mq::launch_overlapped(mq::moe::gather_kernel, dim3(mq::moe::grid_for(P * (d / 8), 256, dev)), dim3(256), 0,
                                     s, "mq_ep_expert_step gather", rows, 1, w.order, static_cast<int>(P), 1,
                                     static_cast<int>(d), w.xg, 1, valid, mq::FlagWait()))
    return rc;
  if (int rc = mq::moe_gemm_run(1, gu_wq, gu_ws, reinterpret_cast<const uint16_t *>(w.xg), P, d, experts, 2 * fe, group,
                                w.tiles, w.ntiles, w.max_tiles, mq::moe::kTileM, w.a, s, 1))
    return rc;
  if (int rc = mq::moe_gemm_run(2, dn_wq, dn_ws, reinterpret_cast<const uint16_t *>(w.a), P, fe, experts, d, group,
                                w.tiles, w.ntiles, w.max_tiles, mq::moe::kTileM, w.z, s, 1))
    return rc;
  // both paths leave the outputs at the pairs' grouped positions (slot_of)
  const float *z = w.z;
  const int32_t *slot_of = w.slot_of;
  return mq_ep_return(z, slot_of, ids, d, world, rank, cap, peer_ret, peer_flags, epoch, done, s);
}

extern "C" int mq_ep_combine(const float *ret, const int32_t *slot_of, const float *weights, int64_t tokens, int topk,
                             int64_t d, int add, float *y, const int *flags, int world, const int *epoch, void *stream) {
  MQ_REQUIRE(ret && slot_of && weights && y && flags && epoch, MQ_EINVAL, "mq_ep_combine: null pointer");
  MQ_REQUIRE(tokens > 0 && topk >= 1 && d > 0 && d % 4 == 0 && world >= 1 && world <= 256, MQ_EINVAL,
             "mq_ep_combine: bad shape (d must be a multiple of 4)");
  MQ_REQUIRE(mq::aligned(ret, 16) && mq::aligned(y, 16), MQ_EALIGN, "mq_ep_combine: ret and y must be 16-byte aligned");
  mq::DeviceInfo dev;
  if (int rc = mq::device_info(&dev)) return rc;
  mq::FlagWait wait;  // every owner's outputs: each CTA waits for them
  wait.flags = flags;
  wait.which = 1;
  wait.world = world;
  wait.epoch = epoch;
  return mq::launch_overlapped(mq::moe::combine_kernel, dim3(mq::moe::grid_for(tokens * (d / 4), 256, dev)), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), "mq_ep_combine", ret, slot_of, weights,
                               static_cast<int>(tokens), topk, static_cast<int>(d), static_cast<int>(add != 0), y, wait);
}
