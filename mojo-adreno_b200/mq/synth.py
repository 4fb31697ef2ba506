"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configurations.

There are no checkpoints offline; these stand in for them. numpy default_rng(seed), drawn in a
fixed order per matrix: activations, then scales, then codes.
  int4: per group an fp16 scale |N(0, 0.02)| and uniform nibbles (value = nibble - 8), stored in
        the word layout as the two's complement nibble (= nibble ^ 8). Drawing whole uint32 words
        uniformly gives exactly those uniform nibbles.
  ternary: codes {0, 1, 2} with probabilities 1/4, 1/2, 1/4 (value code - 1), 16 per word in the
        transposed [k/16, n] layout; fp16 scale per 128 weights |N(0, 0.05)|. A code is the sum
        of two fair bits, so a word is (r & 0x55555555) + ((r >> 1) & 0x55555555) for uniform r.
"""
import numpy as np

# Llama-3.2-1B decode layer + head (hidden 2048, 32 q / 8 kv heads of 64, FFN 8192).
LLAMA_LAYER = [("qkv", 3072, 2048), ("o", 2048, 2048), ("gate_up", 16384, 2048), ("down", 2048, 8192),
               ("lm_head", 128256, 2048)]
# Llama-3.2-1B prefill projections (M = 431 tokens).
LLAMA_PREFILL = [("gate_up", 8192, 2048), ("down", 2048, 8192), ("qkv", 3072, 2048)]
PREFILL_TOKENS = 431
# Qwen3-8B ternary projections.
QWEN3_TERNARY = [("gate_up", 12288, 4096), ("down", 4096, 12288), ("head", 151936, 4096)]
# Qwen3-30B-A3B MoE layer.
MOE = dict(d=2048, experts=128, fe=768, topk=8, group=32, tokens=404)


def q4_matrix(rng, n, k, group, scale_std=0.02):
    """(wq uint32 [n, k/8], ws fp16 [n, k/group]): scales first, then codes."""
    ws = np.abs(rng.normal(0.0, scale_std, size=(n, k // group))).astype(np.float16)
    wq = rng.integers(0, 1 << 32, size=(n, k // 8), dtype=np.uint32)
    return wq, ws


def ternary_matrix(rng, n, k, scale_std=0.05):
    """(w uint32 [k/16, n], s fp16 [k/128, n]) in the transposed layout: scales, then codes."""
    s = np.abs(rng.normal(0.0, scale_std, size=(k // 128, n))).astype(np.float16)
    r = rng.integers(0, 1 << 32, size=(k // 16, n), dtype=np.uint32)
    w = (r & np.uint32(0x55555555)) + ((r >> np.uint32(1)) & np.uint32(0x55555555))
    return w.astype(np.uint32), s


def gemv_config1(seed=0):
    """Q4_0 GEMV, Llama-3.2-1B MLP-up shape: x fp32 [1, 2048], W [8192, 2048], G = 32."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, 2048)).astype(np.float32)
    wq, ws = q4_matrix(rng, 8192, 2048, 32)
    return x, wq, ws


def llama_layer(batch=1, seed=0, rows=None, group=32):
    """The decode layer + head, G = 32: {name: (x fp32 [batch, k], wq, ws)}. `rows` limits every
    matrix to its first rows (for CPU-sized checks); the draws are made at full size regardless
    of batch so that batch-1 and batch-64 share weights."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, n, k in LLAMA_LAYER:
        x = rng.standard_normal((64, k)).astype(np.float32)[:batch]
        wq, ws = q4_matrix(rng, n, k, group)
        if rows is not None:
            wq, ws = wq[:rows], ws[:rows]
        out[name] = (np.ascontiguousarray(x), np.ascontiguousarray(wq), np.ascontiguousarray(ws))
    return out


def prefill(seed=0, tokens=PREFILL_TOKENS, group=32):
    """int4 prefill GEMM shapes: {name: (X fp16 [tokens, k], wq, ws)}."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, n, k in LLAMA_PREFILL:
        x = rng.standard_normal((tokens, k)).astype(np.float16)
        wq, ws = q4_matrix(rng, n, k, group)
        out[name] = (x, wq, ws)
    return out


def moe_layer(seed=0, tokens=MOE["tokens"], experts=MOE["experts"], d=MOE["d"], fe=MOE["fe"], group=MOE["group"]):
    """Qwen3-30B-A3B-shape MoE layer: x fp32 [T, d], router logits [T, E], gate|up experts
    [E * 2fe, d] (expert e: gate rows e*2fe .. +fe-1, up rows after) and down [E * d, fe], G = 32."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((tokens, d)).astype(np.float32)
    logits = rng.standard_normal((tokens, experts)).astype(np.float32)
    gu_wq, gu_ws = q4_matrix(rng, experts * 2 * fe, d, group)
    dn_wq, dn_ws = q4_matrix(rng, experts * d, fe, group)
    return dict(x=x, logits=logits, gu_wq=gu_wq, gu_ws=gu_ws, dn_wq=dn_wq, dn_ws=dn_ws)


def ternary(seed=0, which=None):
    """Qwen3-8B ternary GEMV shapes: {name: (x fp16 [1, k], w, s)}."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, n, k in QWEN3_TERNARY:
        x = rng.standard_normal((1, k)).astype(np.float16)
        w, s = ternary_matrix(rng, n, k)
        if which is None or name in which:
            out[name] = (x, w, s)
    return out
