"""Ternary (2-bit) transposed layout: codes, GEMV (exact and fp16-chain emulation), packer.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
import numpy as np

SHIFTS2 = np.arange(16, dtype=np.uint32) * 2


def codes(w, n, k):
    """codes [n, k] of the transposed layout: code(k, i) = (w[k/16, i] >> 2 (k % 16)) & 3
    (bonsai/kernels/kernels.mojo:201-208, qwen3/convert.cpp:39-74). `w` is [k/16, n] uint32."""
    w = np.asarray(w, np.uint32).reshape(k // 16, n)
    c = (w[:, None, :] >> SHIFTS2[None, :, None]) & 3  # [k/16, 16, n]
    return c.reshape(k, n).T.astype(np.int8)


def tgemv(x16, w, s, n, k, cols=4096):
    """Exact y[b, i] = sum_g s[g, i] sum_{k in g} (code - 1) x[b, k] (float64), the value
    packed_linear + packed_reduce approximate (bonsai/kernels/kernels.mojo:283-325,437-448).
    Computed `cols` outputs at a time, so that full-size heads fit in host memory."""
    w = np.asarray(w, np.uint32).reshape(k // 16, n)
    sc = np.asarray(s, np.float16).reshape(k // 128, n)
    x = np.atleast_2d(np.asarray(x16, np.float16)).astype(np.float64)
    y = np.empty((x.shape[0], n), np.float64)
    for c0 in range(0, n, cols):
        c1 = min(n, c0 + cols)
        c = codes(np.ascontiguousarray(w[:, c0:c1]), c1 - c0, k).astype(np.float64) - 1.0
        scl = sc[:, c0:c1].astype(np.float64)
        wd = (c.reshape(c1 - c0, k // 128, 128) * scl.T[:, :, None]).reshape(c1 - c0, k)
        y[:, c0:c1] = x @ wd.T
    return y


CAND_BLOCK = 512  # logits of a candidate: 64 lanes x 8 (bonsai/kernels/kernels.mojo:491-517)


def head_candidates(y):
    """packed_head's argmax candidates for logits y [batch, n] (bonsai/kernels/kernels.mojo:490-517):
    per block of 512 consecutive logits (value, index, non-finite flag) as float32 [batch, ceil(n/512), 3],
    the lowest index among equal values. Only logits i < n compete (the reference's lanes past n
    compete with 0 at an index >= n). The value and index of a flagged block are unspecified."""
    y = np.atleast_2d(np.asarray(y, np.float32))
    b, n = y.shape
    nc = -(-n // CAND_BLOCK)
    out = np.zeros((b, nc, 3), np.float32)
    for t in range(b):
        for c in range(nc):
            blk = y[t, c * CAND_BLOCK:(c + 1) * CAND_BLOCK]
            bad = not np.isfinite(blk).all()
            i = int(np.argmax(np.where(np.isnan(blk), -np.inf, blk)))  # first maximum = lowest index
            out[t, c] = (blk[i], c * CAND_BLOCK + i, 1.0 if bad else 0.0)
    return out


def greedy(cand):
    """The greedy token of each row of candidates [batch, ncand, 3]: greedy() of bonsai/bonsai_vk.c:506-515
    (lowest index among equal values) and best_of of lfm2/kernels/dsk.mojo:442-465; -1 where a flag is
    set (greedy() stops there with "nonfinite logits")."""
    cand = np.asarray(cand, np.float32).reshape(-1, np.asarray(cand).shape[-2], 3)
    res = []
    for c in cand:
        if (c[:, 2] != 0).any():
            res.append(-1)
            continue
        best = 0
        for i in range(1, len(c)):
            if c[i, 0] > c[best, 0] or (c[i, 0] == c[best, 0] and c[i, 1] < c[best, 1]):
                best = i
        res.append(int(c[best, 1]))
    return np.array(res, np.int32)


def tgemv_fp16_chains(x16, w, s, n, k):
    """The reference's own arithmetic (batch 1): per 128-group, _group_dot's four fp16 FMA chains
    per activation half (pair % 4), each step rounded to fp16, joined in fp32 as
    ((d0lo + d0hi) + (d1lo + d1hi)) + ((d2lo + d2hi) + (d3lo + d3hi)), times the fp32 scale,
    groups summed in fp32 (bonsai/kernels/kernels.mojo:190-223,227-280). Small sizes only."""
    c = codes(w, n, k).astype(np.float32) - 1.0  # [n, k]
    x = np.asarray(x16, np.float16).reshape(k).astype(np.float32)
    sc = np.asarray(s, np.float16).astype(np.float32).reshape(k // 128, n)
    y = np.zeros(n, np.float32)
    for g in range(k // 128):
        d = np.zeros((4, 2, n), np.float16)
        for word in range(8):
            for pair in range(8):
                kk = g * 128 + word * 16 + 2 * pair
                for h in range(2):
                    prod = c[:, kk + h] * x[kk + h]
                    d[pair % 4, h] = (d[pair % 4, h].astype(np.float32) + prod).astype(np.float16)
        df = d.astype(np.float32)
        tot = ((df[0, 0] + df[0, 1]) + (df[1, 0] + df[1, 1])) + ((df[2, 0] + df[2, 1]) + (df[3, 0] + df[3, 1]))
        y = (y + tot * sc[g]).astype(np.float32)
    return y


def pack_transposed(w_rows, s_rows, b_rows=None):
    """MLX 2-bit rows -> the kernels' transposed layout, as qwen3/convert.cpp:39-74 (addPacked):
    codes [n, k/16] -> [k/16, n] words, scales [n, k/128] -> [k/128, n]; every group must be
    ternary (bias == -scale) or ValueError."""
    w_rows = np.asarray(w_rows, np.uint32)
    s_rows = np.asarray(s_rows, np.float16)
    if b_rows is not None:
        b = np.asarray(b_rows, np.float16).astype(np.float32)
        if np.any(b != -s_rows.astype(np.float32)):
            raise ValueError("not ternary (bias != -scale)")
    return np.ascontiguousarray(w_rows.T), np.ascontiguousarray(s_rows.T)
