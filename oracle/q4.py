"""int4 word layout: decode, dequantise, GEMV/GEMM and the packers (numpy restatements).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
import numpy as np

SHIFTS = np.arange(8, dtype=np.uint32) * 4


def unpack(wq):
    """int8 values of a word-layout matrix [n, k/8] -> [n, k]: ((nib ^ 8) - 8), element 8w + j in
    bits 4j..4j+3 of word w. Restates qwen3moe/reference.py:60-61 (Weights.int4) and the decode of
    llama/kernels/gemv_q4.mojo:23-25."""
    wq = np.asarray(wq, np.uint32)
    nib = (wq[..., None] >> SHIFTS) & 15
    return ((nib.astype(np.int32) ^ 8) - 8).astype(np.int8).reshape(*wq.shape[:-1], wq.shape[-1] * 8)


def dequant(wq, ws, group):
    """q * scale in fp32, a scale per `group` weights of a row: qwen3moe/reference.py:53-65."""
    q = unpack(wq).astype(np.float32)
    n, k = q.shape
    s = np.asarray(ws, np.float16).astype(np.float32).reshape(n, k // group, 1)
    return (q.reshape(n, k // group, group) * s).reshape(n, k)


def gemv(wq, ws, x, group):
    """y[b, r] = sum_c W[r, c] x[b, c] in float64 on the dequantised weights (the exact value the
    reference's fp32 kernels approximate: llama/kernels/gemv_q4.mojo:13-30)."""
    w = dequant(wq, ws, group).astype(np.float64)
    x = np.atleast_2d(np.asarray(x, np.float64))
    return x @ w.T


def gate_up(wq, ws, x, f, group):
    """a[b, j] = silu(W[j] . x_b) * (W[f + j] . x_b) in float64 for the fused [2f, k] gate|up matrix:
    gate_up_q4 of lfm2/kernels/lk.mojo:154-167 (silu(g) = g / (1 + exp(-g)), lk.mojo:33-34)."""
    h = gemv(wq, ws, x, group)
    g, u = h[:, :f], h[:, f:2 * f]
    return g / (1.0 + np.exp(-g)) * u


def gemv_reference_order(wq, ws, x, group):
    """fp32, in gemv_q4's own order: per word part = sum_j q_j x_j (fp32), acc += part * scale,
    then a sum over the 64 lanes' accumulators (llama/kernels/gemv_q4.mojo:18-30). Small sizes only."""
    q = unpack(wq).astype(np.float32)
    n, k = q.shape
    x = np.asarray(x, np.float32).reshape(k)
    s = np.asarray(ws, np.float16).astype(np.float32)
    words = k // 8
    part = (q.reshape(n, words, 8) * x.reshape(words, 8)).sum(-1, dtype=np.float32)
    return (part * s[:, np.arange(words) // (group // 8)]).sum(-1, dtype=np.float32)


def pack_words(q):
    """int values in -8..7 [n, k] -> uint32 words [n, k/8], low nibble first (4-bit two's complement)."""
    q = np.asarray(q, np.int32)
    n, k = q.shape
    nib = (q.reshape(n, k // 8, 8) & 15).astype(np.uint32)
    return (nib << SHIFTS).sum(-1, dtype=np.uint64).astype(np.uint32)


def quantize_max7(w16, group):
    """Symmetric int4 with scale = fp16(max|w| / 7) per group, q = clip(rint(w / scale), -8, 7):
    llama/run.py:56-70 (quantize4) and llama/st2bin.c:54-70, fp32 math. Returns (wq, ws)."""
    w = np.asarray(w16, np.float16).astype(np.float32)
    n, k = w.shape
    wg = w.reshape(n, k // group, group)
    s16 = (np.abs(wg).max(-1) / np.float32(7)).astype(np.float16)
    sf = s16.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(sf > 0, np.rint(wg / sf), np.float32(0))
    q = np.clip(q, -8, 7).astype(np.int32).reshape(n, k)
    return pack_words(q), s16


def quantize_search(wbf, group):
    """int4 with the searched scale of qwen3moe/convert.c:124-157: for d = 6.5, 6.75, ..., 9 the
    candidate t = fp16(m / d) (m = max|w| of the group, fp32), error sum (w - clip(rint(w/t)) t)^2
    in fp32; the first least error wins; q = clip(rint(w / s), -8, 7). `wbf` holds bf16 values as
    fp32. Returns (wq, ws)."""
    w = np.asarray(wbf, np.float32)
    n, k = w.shape
    wg = w.reshape(-1, group)
    m = np.abs(wg).max(-1)
    best = np.full(m.shape, np.inf, np.float32)
    sf = np.zeros(m.shape, np.float32)
    alive = np.ones(m.shape, bool)
    d = np.float32(6.5)
    while d <= np.float32(9.0):
        t = (m / d).astype(np.float32).astype(np.float16).astype(np.float32)
        alive &= t > 0  # the C loop breaks at the first non-positive candidate
        with np.errstate(divide="ignore", invalid="ignore"):
            v = np.clip(np.rint(wg / t[:, None]), -8, 7).astype(np.float32)
        diff = (wg - v * t[:, None]).astype(np.float32)
        e = np.zeros(m.shape, np.float32)
        for j in range(group):  # fp32 accumulation in the C order
            e = (e + diff[:, j] * diff[:, j]).astype(np.float32)
        better = alive & (e < best)
        best = np.where(better, e, best)
        sf = np.where(better, t, sf)
        d = np.float32(d + np.float32(0.25))
    s16 = sf.astype(np.float16)
    sfx = s16.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(sfx > 0, np.clip(np.rint(wg / sfx), -8, 7), 0).astype(np.int32)
    return pack_words(q.reshape(n, k)), s16.reshape(n, k // group)


def q4_0_to_words(blocks):
    """GGUF Q4_0 blocks (18 B: fp16 d, 16 bytes; element j = lo nibble of byte j, element j + 16 =
    hi nibble, value nibble - 8) -> 4 words each (nibble ^ 8 at element 8w + k) and the fp16 d
    unchanged: lfm2/convert.c:58-71 (q4_block). `blocks` uint8 [nblocks, 18] -> (words u32
    [nblocks, 4], d f16 [nblocks])."""
    b = np.asarray(blocks, np.uint8).reshape(-1, 18)
    d = b[:, :2].copy().view(np.float16).reshape(-1)
    qs = b[:, 2:]
    nib = np.concatenate([qs & 15, qs >> 4], axis=1).astype(np.uint32)  # element order 0..31
    words = ((nib ^ 8).reshape(-1, 4, 8) << SHIFTS).sum(-1, dtype=np.uint64).astype(np.uint32)
    return words, d


def dequant_q4_0(blocks, rows, cols):
    """ggml's Q4_0 dequantisation as lfm2/weights.py:61-68 restates it: (nibble - 8) * d, fp32."""
    b = np.asarray(blocks, np.uint8).reshape(-1, 18)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    qs = b[:, 2:]
    q = np.concatenate([(qs & 15).astype(np.int8) - 8, (qs >> 4).astype(np.int8) - 8], axis=1)
    return (q.astype(np.float32) * d).reshape(rows, cols)
