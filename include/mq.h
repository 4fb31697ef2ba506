/*
 * mq.h - C ABI of the B200 (sm_100a) weight-quantised matmul library (libmq.so).
 *
 * Every entry point is stream-ordered and asynchronous: it validates its arguments on the host,
 * enqueues its kernels on `stream` (a cudaStream_t, NULL = the legacy default stream) and returns.
 * The caller allocates and owns every buffer (device pointers, as from cudaMalloc or
 * torch.Tensor.data_ptr()); no entry point allocates device memory. Where an operator needs
 * scratch memory the caller passes it, sized by the matching *_workspace_size() call.
 *
 * Return value: MQ_OK (0) or a negative MQ_E* code; the message of the most recent failure on the
 * calling thread is returned by mq_last_error(). This mirrors the reference's status-code
 * convention: an int status, 0 = success, plus a first-error string
 * (driver/executor.h:13-26, driver/protocol.h:36-40).
 *
 * Storage formats (the reference's own bytes, read unchanged):
 *   int4 "word layout": W[n][k] row-major as uint32 wq[n][k/8]; element 8w+j of a row sits in
 *     bits 4j..4j+3 of word w as a 4-bit two's complement nibble (value = (nib ^ 8) - 8);
 *     one fp16 scale per `group` consecutive weights of a row, ws[n][k/group]
 *     (llama/kernels/gemv_q4.mojo:1-4,18-27; lfm2/convert.c:4-7; qwen3moe/export.py:152-176).
 *   ternary transposed layout: codes c in {0,1,2} (value c - 1), 16 per uint32; the code of
 *     (k, n) is (w[(k/16)*n_total + n] >> 2*(k%16)) & 3; one fp16 scale per 128 k of an output,
 *     s[k/128][n] (qwen3/convert.cpp:39-74, bonsai/kernels/kernels.mojo:190-223).
 */
#ifndef MQ_H
#define MQ_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MQ_API __attribute__((visibility("default")))
#else
#define MQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MQ_OK 0
#define MQ_EINVAL (-1)       /* bad shape, group, batch or null pointer */
#define MQ_EALIGN (-2)       /* a pointer is not aligned as the operator needs */
#define MQ_ECUDA (-3)        /* a CUDA call failed (launch error, no device, ...) */
#define MQ_EUNSUPPORTED (-4) /* the device is not sm_100 or the size is above a stated maximum */
#define MQ_ETIMEOUT (-5)     /* a kernel's bounded wait ran out (see mq_device_status) */
#define MQ_EIO (-6)          /* a file could not be opened or read */

/* Activation dtypes. */
#define MQ_F32 0
#define MQ_F16 1
#define MQ_BF16 2 /* weights for the packers only */

/* Quantisation methods of mq_quantize_q4. */
#define MQ_Q4_MAX7 0   /* scale = fp16(max|w| / 7) */
#define MQ_Q4_SEARCH 1 /* scale searched over max|w| / d, d = 6.5 .. 9 */

/* The message of the last failure on this thread ("" when none). */
MQ_API const char *mq_last_error(void);

/* Library ABI version (major * 100 + minor). */
MQ_API int mq_version(void);

/* Reads the device-side status word that kernels with bounded waits set when a wait runs out
 * (0 = none, else the code of the first wait that gave up). Synchronises `stream`. When `reset`
 * is nonzero the word is cleared afterwards. Returns the word (>= 0) or a negative MQ_E* code. */
MQ_API int mq_device_status(int reset, void *stream);

/*
 * q[r][c] = ((nib ^ 8) - 8) as int8 and s_out = ws unchanged, for the int4 word layout: the
 * bit-exact unpack hook. Replaces the nibble decode inside gemv_q4 (llama/kernels/gemv_q4.mojo:23-25)
 * and the host dequantiser's integer step (qwen3moe/reference.py:53-65).
 * wq: [n][k/8] u32, ws: [n][k/group] f16, q: [n][k] i8, s_out: [n][k/group] f16 (may be NULL).
 */
MQ_API int mq_unpack_q4(const uint32_t *wq, const uint16_t *ws, int8_t *q, uint16_t *s_out, int64_t n,
                 int64_t k, int group, void *stream);

/*
 * Decode GEMV over int4 weights: y[b][r] (+)= sum_c W[r][c] * x[b][c] for b < batch.
 * Replaces gemv_q4 / gemv_add_q4 (llama/kernels/gemv_q4.mojo:13-30,
 * llama/kernels/gemv_add_q4.mojo:13-30; the G=32 Q4_0 variant lfm2/kernels/lk.mojo:56-72,134-143;
 * the G=128 expert rows qwen3moe/kernels/moek.mojo:29-45) and the batched t_gemv_q4 / p_gemv_q4
 * (qwen3moe/kernels/moek.mojo:273-281,528-545) with the argument order wq, ws, x, y, cols.
 * x: [batch][k] fp32 (x_dtype MQ_F32) or fp16 (MQ_F16); y: [batch][n] fp32.
 * group in {32, 64, 128}; k % 32 == 0 and k % group == 0; add != 0 adds into y (gemv_add_q4).
 * 1 <= batch <= 64: batch <= 4 runs the streaming GEMV; batch > 4 runs the tensor-core GEMM
 * (mq_gemm_q4), which needs fp16 x here (fp32 x needs mq_gemm_q4's workspace) and k % 256 == 0.
 * wq and x 16-byte aligned (ws too for batch > 4), y 4-byte aligned. The streaming GEMV stages x
 * as 15-bit fixed point per 32-k group (two int8 limbs, step 1/65024 of the group's largest |x|) and
 * multiplies exactly in integers; a NaN or an infinity in x makes the outputs of that token NaN,
 * where the reference's fp32 sums are Inf or NaN.
 */
MQ_API int mq_gemv_q4(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y,
               int64_t n, int64_t k, int group, int batch, int add, void *stream);

/*
 * Fused gate|up decode GEMV: a[b][j] = silu(W[j] . x[b]) * (W[f + j] . x[b]) for j < f, b < batch,
 * silu(g) = g / (1 + exp(-g)). Replaces gate_up_q4 (lfm2/kernels/lk.mojo:154-167; argument order
 * wq, ws, x, a, cols, f): W is the fused [2f][k] gate|up matrix in mq_gemv_q4's layout (gate rows
 * 0..f-1, up rows f..2f-1), so the SwiGLU costs no extra launch and no fp32 round trip of gate|up.
 * Each product is computed exactly as mq_gemv_q4 computes that row. f % 16 == 0, 1 <= batch <= 4;
 * other limits as mq_gemv_q4.
 */
MQ_API int mq_gate_up_q4(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *a, int64_t f,
                         int64_t k, int group, int batch, void *stream);

/*
 * Prefill GEMM over int4 weights on the tcgen05 tensor cores: y[t][r] (+)= sum_c W[r][c] * x[t][c]
 * for t < m tokens. Replaces p_gemm_q4 (llama/kernels/prefill/p_gemm_q4.mojo:26-62, argument order
 * wq, ws, x, y, n, k) and gemm_q4 (lfm2/kernels/lk.mojo:458-495), without their rows % 128 and
 * n % 128 restrictions. x: [m][k] fp16 (MQ_F16) or fp32 (MQ_F32, converted to fp16 in `workspace`,
 * mq_gemm_q4_workspace_size() bytes); y: [m][n] fp32. group in {32, 64, 128}; k % 256 == 0.
 * The product uses fp16 x and fp16 q*scale with fp32 accumulation. wq, ws, x and workspace 16-byte
 * aligned, y 4-byte aligned. When K is split across CTAs (small n * m) y is zeroed first unless add,
 * and the parts are added into y in an order that varies from run to run: y is then not bitwise
 * reproducible (it differs in the last bits of fp32 between runs).
 */
MQ_API size_t mq_gemm_q4_workspace_size(int64_t m, int64_t k, int x_dtype);
MQ_API int mq_gemm_q4(const uint32_t *wq, const uint16_t *ws, const void *x, int x_dtype, float *y, int64_t n,
                      int64_t k, int64_t m, int group, int add, void *workspace, size_t workspace_bytes, void *stream);

/*
 * mq_gemm_q4 for fp32 x without a caller workspace. This entry point has no counterpart in the
 * reference. Its fp16 copy of x lives in a fixed 4 MiB buffer inside libmq's own device memory
 * (m * k <= 2097152 activations; larger calls return MQ_EINVAL), so it allocates nothing: for callers
 * that cannot allocate device memory, such as a binding that can pass only (wq, ws, x, y, n, k) and no
 * scratch buffer, or a host whose own allocator owns the device. The first call in each CUDA context
 * (normally one per device) looks the buffer's address up (cudaGetSymbolAddress) with that context
 * current; make that first call before any stream capture. Every call in a context shares the one
 * buffer: calls that overlap in time (on two streams or two host threads) race and must be
 * serialised by the caller. Other arguments, limits and numerics as mq_gemm_q4.
 */
MQ_API int mq_gemm_q4_noalloc(const uint32_t *wq, const uint16_t *ws, const float *x, float *y, int64_t n, int64_t k,
                              int64_t m, int group, int add, void *stream);

/*
 * Ternary GEMV: y[b][i] = sum_k s[k/128][i] * (code(k, i) - 1) * x[b][k], b < batch <= 4.
 * Replaces packed_linear + packed_reduce and the GEMV part of packed_head
 * (bonsai/kernels/kernels.mojo:283-325,437-448,451-489) as called by qwen3/model.mojo:128-135,170-181.
 * w: [k/16][n] u32, s: [k/128][n] f16, x: [batch][k] fp16 (the reference's fp16 pairs,
 * qwen3/kernels/qwen3k.mojo:17-20, are the same bytes), y: [batch][n] fp32.
 * k % 128 == 0; any n >= 1 (n % 4 == 0 streams w with TMA; other widths, such as the reference's
 * second head half of 75893 outputs, with 4-byte copies); w and x 16-byte aligned, s 2-byte, y 4-byte.
 * A NaN or an infinity in x makes every output of that token NaN (the reference's fp32 sums are then
 * Inf or NaN: the same outputs are not finite).
 */
MQ_API int mq_tgemv(const uint16_t *x, const uint32_t *w, const uint16_t *s, float *y, int64_t n, int64_t k,
             int batch, void *stream);

/*
 * mq_tgemv plus packed_head's argmax candidates (bonsai/kernels/kernels.mojo:490-517, select != 0):
 * for each token b and each block of 512 consecutive outputs c (ncand = ceil(n / 512) blocks),
 * candidates[(b * ncand + c) * 3 + 0..2] = (largest y in the block, its index as a float, 1.0 if any
 * y in the block is not finite else 0.0); among equal values the lowest index wins. Only outputs
 * i < n compete (the reference's lanes past n compete with the value 0 at an index >= n).
 * n <= 4718592; other arguments and limits as mq_tgemv.
 */
MQ_API int mq_tgemv_head(const uint16_t *x, const uint32_t *w, const uint16_t *s, float *y, float *candidates,
                         int64_t n, int64_t k, int batch, void *stream);

/*
 * Greedy token from head candidates, on the device: index[b] = the index of the best of the ncand
 * candidates (value, index, flag) of token b, the lowest index among equal values (best_of,
 * lfm2/kernels/dsk.mojo:442-465; the host loop greedy() of bonsai/bonsai_vk.c:506-515), or -1 when a
 * candidate's non-finite flag is set (where greedy() stops with "nonfinite logits").
 */
MQ_API int mq_head_argmax(const float *candidates, int64_t ncand, int batch, int32_t *index, void *stream);

/*
 * Prefill GEMM over ternary weights on the tcgen05 tensor cores: y[t][c] (+)= sum_k x[t][k] * W[c][k]
 * for t < m, W in mq_tgemv's transposed layout (w [k/16][n] 2-bit codes, s [k/128][n] fp16 scales).
 * Replaces p_gemm_t2 (bonsai/kernels/prefill.mojo:155-164, argument order x, w, params, y, n, k).
 * x: [m][k] fp16 (MQ_F16) or fp32 (MQ_F32, converted to fp16 in `workspace`,
 * mq_gemm_q4_workspace_size(m, k, MQ_F32) bytes); y: [m][n] fp32. k % 256 == 0, n % 4 == 0.
 * The weights are exact in fp16; x is rounded to fp16; accumulation is fp32.
 */
MQ_API int mq_gemm_t2(const void *x, int x_dtype, const uint32_t *w, const uint16_t *s, float *y, int64_t n, int64_t k,
                      int64_t m, int add, void *workspace, size_t workspace_bytes, void *stream);

/* ---- top-k MoE on int4 experts (Qwen3-MoE layout) ------------------------------------------------
 * Expert weights are one word-layout matrix each: gate|up [experts * 2fe][d/8] (expert e's gate rows
 * e*2fe .. e*2fe+fe-1, its up rows the next fe; qwen3moe/export.py:166-169) and down [experts * d][fe/8],
 * with fp16 scales per `group` weights of a row. */

/* Router logits in fp32: logits[t][e] = W[e] . x[t] for W [experts][d], x [tokens][d] (gemv_f32 and
 * p_gemv_f32, qwen3moe/kernels/moek.mojo:143-153, 284-295). d % 4 == 0; w and x 16-byte aligned. */
MQ_API int mq_moe_router(const float *w, const float *x, float *logits, int64_t tokens, int experts, int64_t d,
                         void *stream);

/* ids[t][k], weights[t][k]: the top-k experts of each token (the lowest index among equal logits)
 * and softmax over the k chosen logits. Replaces route / p_route (qwen3moe/kernels/moek.mojo:156-197,
 * 385-425). logits: [tokens][experts] fp32, experts <= 256, topk <= 32. */
MQ_API int mq_moe_route(const float *logits, int32_t *ids, float *weights, int64_t tokens, int experts, int topk,
                        void *stream);

/* Stable grouping of the tokens * topk (token, slot) pairs by expert. Replaces p_expert_lists and
 * p_expert_items (moek.mojo:432-442, 548-557): counts[e]; offsets[e] (exclusive prefix, offsets[experts]
 * = pairs); order[offsets[e] + r] = the r-th pair t * topk + k routed to e, in increasing pair index;
 * slot_of[pair] = its position in order; tiles[3 * i ..] = (expert, first sorted row, rows <= tile)
 * work items in expert order and *ntiles their count (at most experts + ceil(pairs / tile)).
 * A pair whose id is outside [0, experts) is left out (slot_of = -1, the unused tail of order = 0)
 * and reported through mq_device_status. */
MQ_API int mq_moe_group(const int32_t *ids, int64_t tokens, int topk, int experts, int tile, int32_t *counts,
                        int32_t *offsets, int32_t *order, int32_t *slot_of, int32_t *tiles, int32_t *ntiles,
                        void *stream);

/* The router chain fused: mq_moe_router, mq_moe_route and (counts != NULL) mq_moe_group in two
 * launches. A cluster of 8 CTAs computes the router logits of 16 tokens (each CTA an eighth of the
 * experts), keeps them in shared memory and routes each token from the cluster's distributed shared
 * memory; the grouping follows as a programmatic dependent launch. ids and weights are those of
 * mq_moe_route on the logits this chain computes, and the grouping that of mq_moe_group on those
 * ids. logits (may be NULL): receives the router logits [tokens][experts]. Replaces gemv_f32 + route
 * + p_expert_lists / p_expert_items (qwen3moe/kernels/moek.mojo:143-197, 432-442, 548-557).
 * experts <= 256, topk <= 32, d % 4 == 0; w and x 16-byte aligned. counts == NULL skips the grouping
 * (the other grouping outputs are then ignored). */
MQ_API int mq_moe_route_group(const float *w, const float *x, float *logits, int32_t *ids, float *weights,
                              int64_t tokens, int experts, int topk, int64_t d, int tile, int32_t *counts,
                              int32_t *offsets, int32_t *order, int32_t *slot_of, int32_t *tiles, int32_t *ntiles,
                              void *stream);

/* Expert-parallel dispatch plan: experts are split into `world` equal contiguous ranges, range r owned
 * by rank r. The tokens * topk pairs are grouped stably by owning rank: counts[r], offsets[r]
 * (offsets[world] = pairs), order[offsets[r] + i] = the i-th pair sent to rank r, slot_of[pair] = its
 * send position, local_ids[pos] = the pair's expert id within its owner (ids - r * experts / world).
 * capacity > 0 gives the fixed-capacity layout of an exchange with static split sizes: rank r's
 * pairs sit at r * capacity + i, offsets[r] = r * capacity, and the other positions of order and
 * local_ids (world * capacity entries each) hold -1; pairs past a rank's capacity are reported
 * through mq_device_status (9) and left out (slot_of -1). A negative id means "no expert" and is
 * left out silently; an id >= experts is reported (8). No counterpart kernel in the reference
 * (which runs on one device). */
MQ_API int mq_ep_plan(const int32_t *ids, int64_t tokens, int topk, int experts, int world, int capacity,
                      int32_t *counts, int32_t *offsets, int32_t *order, int32_t *slot_of, int32_t *local_ids,
                      void *stream);

/* xg[s] = fp16(x[order[s] / topk]) for s < pairs: the expert-sorted activation rows (p_gather,
 * lfm2moe/kernels/mk.mojo:164-176); a row of zeros where order[s] < 0 (an empty position of a
 * fixed-capacity layout). x: [tokens][d] fp32 or fp16; d % 8 == 0. */
MQ_API int mq_moe_gather(const void *x, int x_dtype, const int32_t *order, int64_t pairs, int topk, int64_t d,
                         uint16_t *xg, void *stream);

/* Grouped expert product on the tcgen05 tensor cores over the work tiles of mq_moe_group (tile_m rows
 * per tile, grid sized for max_tiles). mode 1: gate|up with the SwiGLU fused, out = fp16 a[pairs][fe]
 * with a = silu(gate . x) * (up . x), rows_per_expert = 2fe (t_moe_gate_up, moek.mojo:560-583);
 * mode 2: out = fp32 z[pairs][rows_per_expert] (t_moe_down, moek.mojo:586-608). xs: expert-sorted fp16
 * rows [pairs][k]. k % 256 == 0, rows_per_expert % 128 == 0, tile_m % 16 == 0 (<= 128 for mode 1). */
MQ_API int mq_moe_gemm_q4(int mode, const uint32_t *wq, const uint16_t *ws, const uint16_t *xs, int64_t pairs,
                          int64_t k, int experts, int64_t rows_per_expert, int group, const int32_t *tiles,
                          const int32_t *ntiles, int max_tiles, int tile_m, void *out, void *stream);

/* The expert-indirect decode GEMV (moe_gate_up / moe_down's products, moek.mojo:200-223):
 * y[i * rows_per_group + r] = W[ids[i] * group_rows + r] . x_i for i < ngroups, r < rows_per_group,
 * with x_i = x (x_per_group == 0) or x + i * k. W: [wrows][k/8] words; x fp32; rows_per_group % 32 == 0.
 * An id outside the matrix is reported through mq_device_status (and its rows read as expert 0's). */
MQ_API int mq_moe_gemv_q4(const uint32_t *wq, const uint16_t *ws, int64_t wrows, const float *x, float *y,
                          const int32_t *ids, int ngroups, int group_rows, int rows_per_group, int64_t k, int group,
                          int x_per_group, void *stream);

/* moe_gate_up in one launch (qwen3moe/kernels/moek.mojo:200-210): a[i][j] = silu(W[e_i * 2fe + j] . x) *
 * (W[e_i * 2fe + fe + j] . x) for i < ngroups, j < fe, e_i = ids[i]; the fused form of mq_moe_gemv_q4
 * (rows_per_group 2fe) followed by mq_moe_silu_mul, with the same products. fe % 16 == 0, fp32 x. */
MQ_API int mq_moe_gate_up_q4(const uint32_t *wq, const uint16_t *ws, int64_t wrows, const float *x, float *a,
                             const int32_t *ids, int ngroups, int64_t fe, int64_t k, int group, void *stream);

/* a[r][j] = silu(h[r][j]) * h[r][fe + j] in fp32 (moe_gate_up's SwiGLU, moek.mojo:200-210). */
MQ_API int mq_moe_silu_mul(const float *h, float *a, int64_t rows, int64_t fe, void *stream);

/* y[t][c] (+)= sum_k weights[t][k] * z[slot_of[t * topk + k]][c], k in order (p_moe_sum,
 * moek.mojo:479-488); slot_of NULL means row t * topk + k; a negative slot_of adds nothing. z, y 16-byte aligned, d % 4 == 0. */
MQ_API int mq_moe_combine(const float *z, const int32_t *slot_of, const float *weights, int64_t tokens, int topk,
                          int64_t d, int add, float *y, void *stream);

/* The whole MoE layer for precomputed routing: y (+)= sum_k w[t][k] * down_e(silu(gate_e x_t) * up_e x_t).
 * Up to 16 (token, expert) pairs run on the streaming GEMVs (gate|up with the SwiGLU fused, then down,
 * each pair with its own x); more run group, gather, the two grouped tensor-core products and the
 * combine. All on `stream`, with a caller workspace of mq_moe_workspace_size() bytes (256-byte
 * aligned). d % 256 == 0, fe % 256 == 0. An expert id outside [0, experts) is reported through
 * mq_device_status; the grouped path leaves its pair out, the GEMV path reads expert 0's rows for it. */
MQ_API size_t mq_moe_workspace_size(int64_t tokens, int experts, int topk, int64_t d, int64_t fe);
MQ_API int mq_moe_forward(const void *x, int x_dtype, const int32_t *ids, const float *weights, const uint32_t *gu_wq,
                          const uint16_t *gu_ws, const uint32_t *dn_wq, const uint16_t *dn_ws, float *y, int64_t tokens,
                          int experts, int topk, int64_t d, int64_t fe, int group, int add, void *workspace,
                          size_t workspace_bytes, void *stream);

/* The MoE layer with its router on the device, as the model runs it (qwen3moe/model.mojo:208-274:
 * gemv_f32 router, route, the experts): the fused router chain (mq_moe_route_group) writes ids,
 * weights (and logits, when not NULL) and the grouping into the workspace, then the layer runs as
 * mq_moe_forward does on those ids. x fp32 [tokens][d]; router_w fp32 [experts][d]; the workspace
 * is mq_moe_workspace_size(tokens, experts, topk, d, fe) bytes, 256-byte aligned. */
MQ_API int mq_moe_layer(const float *x, const float *router_w, const uint32_t *gu_wq, const uint16_t *gu_ws,
                        const uint32_t *dn_wq, const uint16_t *dn_ws, float *y, int32_t *ids, float *weights,
                        float *logits, int64_t tokens, int experts, int topk, int64_t d, int64_t fe, int group, int add,
                        void *workspace, size_t workspace_bytes, void *stream);

/* ---- expert parallelism over NVLink peer memory ------------------------------------------------------
 * No counterpart in the reference, which runs every expert on one device (qwen3moe/model.mojo:256-267).
 * One process per GPU; rank r owns the experts [r E / world, (r + 1) E / world). Each rank exports one
 * device buffer (mq_ipc_handle) and maps its peers' (mq_ipc_open); the exchange then runs as kernels
 * on the stream, with no host read, so a whole layer can be captured in a CUDA graph:
 *   mq_ep_plan (capacity cap) -> mq_ep_dispatch -> mq_ep_expert_step -> mq_ep_combine
 * (mq_ep_expert_step waits for the rows, mq_ep_combine for the returned outputs; mq_ep_wait is the
 * same wait on its own).
 * Buffers of rank r (each rank's own, mapped by the others; pointer tables are device arrays of world
 * pointers, entry r = the local buffer): rows fp16 [world * cap][d] (received rows), ids int32
 * [world * cap], ret fp32 [world * cap][d] (returned outputs, row d * cap + i for send slot i to owner
 * d), flags int32 [2][world], epoch int32 and two arrival counters int32, all zero-initialised. Every
 * wait is bounded: a rank that does not answer within 2 s is reported through mq_device_status
 * (10: dispatch, 11: return) and the layer goes on without it. */

/* Exports the device allocation holding ptr: a 64-byte handle and ptr's offset within it. */
MQ_API int mq_ipc_handle(const void *ptr, void *handle, int64_t *offset);
/* Maps a peer's exported allocation into the current device (peer access enabled): *ptr = its base + offset. */
MQ_API int mq_ipc_open(const void *handle, int64_t offset, void **ptr);
/* Unmaps what mq_ipc_open mapped (the same ptr and offset). */
MQ_API int mq_ipc_close(void *ptr, int64_t offset);
/* Starts a layer: epoch += 1 (every rank runs the same layers, so the epochs agree), and writes this rank's pairs into their owners' receive buffers: send slot d * cap + i (the fixed-capacity
 * plan of mq_ep_plan: order, local_ids) becomes row rank * cap + i of owner d's rows, with id
 * local_ids[slot] (-1 for an empty slot); then raises flag [0][rank] on every owner to the epoch.
 * x: [tokens][d] fp32 or fp16 (may be NULL when tokens == 0); done: this rank's dispatch counter. */
MQ_API int mq_ep_dispatch(const void *x, int x_dtype, const int32_t *order, const int32_t *local_ids, int64_t tokens,
                          int topk, int64_t d, int world, int rank, int cap, uint16_t *const *peer_rows,
                          int32_t *const *peer_ids, int *const *peer_flags, int *epoch, int *done, void *stream);
/* Waits (one CTA, bounded) until flags[which][s] >= epoch for every rank s. */
MQ_API int mq_ep_wait(const int *flags, int which, int world, const int *epoch, void *stream);
/* Sends expert outputs back: row slot = s * cap + i with ids[slot] >= 0 goes from z (its row slot_of[slot],
 * or slot when slot_of is NULL) to sender s's ret row rank * cap + i; then raises flag [1][rank] on
 * every sender. done: this rank's return counter. */
MQ_API int mq_ep_return(const float *z, const int32_t *slot_of, const int32_t *ids, int64_t d, int world, int rank,
                        int cap, float *const *peer_ret, int *const *peer_flags, const int *epoch, int *done,
                        void *stream);
/* Waits for every rank's rows (flags [0]), then this rank's experts on its received rows (rows, ids; nrows = world * cap, ids -1
 * skipped), then mq_ep_return. Expert weights are this rank's slices (experts = its expert count) in
 * mq_moe_forward's layout. Workspace: mq_ep_workspace_size(nrows, experts, d, fe) bytes, 256-byte aligned. */
MQ_API size_t mq_ep_workspace_size(int64_t rows, int experts, int64_t d, int64_t fe);
MQ_API int mq_ep_expert_step(const uint16_t *rows, const int32_t *ids, const uint32_t *gu_wq, const uint16_t *gu_ws,
                             const uint32_t *dn_wq, const uint16_t *dn_ws, int64_t nrows, int experts, int64_t d,
                             int64_t fe, int group, int world, int rank, int cap, float *const *peer_ret,
                             const int *flags, int *const *peer_flags, const int *epoch, int *done, void *workspace,
                             size_t workspace_bytes, void *stream);
/* Waits for every owner's returned outputs (flags [1]), then y[t] (+)= sum_k weights[t][k] * ret[slot_of[t * topk + k]]
 * (mq_moe_combine over the plan's slot_of). */
MQ_API int mq_ep_combine(const float *ret, const int32_t *slot_of, const float *weights, int64_t tokens, int topk,
                         int64_t d, int add, float *y, const int *flags, int world, const int *epoch, void *stream);

/* ---- weight files -------------------------------------------------------------------------------- */

/* Reads nbytes at byte `offset` of the file at `path` into device memory at dst, through two pinned
 * staging buffers whose host-to-device copies run on `stream` while the next chunk is read; returns
 * when every copy has finished. Replaces M_driver_remote_file (qwen3moe/model.mojo:156-158), which
 * the reference's manifest loaders call once per tensor. MQ_EIO when the file cannot be opened or
 * read; MQ_EINVAL when the range passes the end of the file. */
MQ_API int mq_read_file_to_device(void *dst, int64_t nbytes, const char *path, int64_t offset, void *stream);

/* ---- packers: the byte layouts above, produced on the device -------------------------------------- */

/* w [n][k] (fp32, fp16 or bf16 bits) -> int4 words wq [n][k/8] and fp16 scales ws [n][k/group].
 * MQ_Q4_MAX7 replaces quantize4 (llama/run.py:56-70) and st2bin's q4 (llama/st2bin.c:54-70): values
 * rounded to fp16 first, scale fp16(max|w| / 7), q = clip(rint(w / scale), -8, 7). MQ_Q4_SEARCH
 * replaces qwen3moe/convert.c:124-157 (values used as given; scale = the first of fp16(max|w| / d),
 * d = 6.5, 6.75, .., 9, with the least fp32 squared error). Bytes equal the reference converters'. */
MQ_API int mq_quantize_q4(const void *w, int w_dtype, int64_t n, int64_t k, int group, int method, uint32_t *wq,
                          uint16_t *ws, void *stream);

/* GGUF Q4_0 blocks (18 bytes each: fp16 d, 16 bytes of nibbles) -> 4 words and one fp16 scale per
 * block, G = 32 (lfm2/convert.c:58-71). A row of a [rows][cols] matrix is cols / 32 consecutive blocks. */
MQ_API int mq_q4_0_to_words(const uint8_t *blocks, int64_t nblocks, uint32_t *wq, uint16_t *ws, void *stream);

/* MLX 2-bit rows (codes [n][k/16], scales and biases [n][k/128] fp16) -> the ternary GEMV's transposed
 * w [k/16][n] and s [k/128][n] (qwen3/convert.cpp:39-74). With biases, every group must be ternary
 * (bias == -scale) or MQ_EINVAL "not ternary" is returned and nothing is written; that check
 * synchronises `stream`. biases may be NULL (no check). */
MQ_API int mq_pack_ternary(const uint32_t *codes, const uint16_t *scales, const uint16_t *biases, int64_t n, int64_t k,
                           uint32_t *w, uint16_t *s, void *stream);

/* q[i] = fp16 pair (x[2i], x[2i+1]) (pack_half, qwen3/kernels/qwen3k.mojo:17-20,45-48): fp32
 * activations -> the ternary GEMV's x. n even. */
MQ_API int mq_pack_half(const float *x, uint32_t *q, int64_t n, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MQ_H */
