"""Top-k MoE on int4 experts: routing, grouping and the SwiGLU expert layer (numpy restatements).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
import numpy as np

from . import q4


def route(logits, topk=8):
    """Per token the top-k experts (the lowest index among equal logits, in selection order) and
    their weights softmax(top logits) in fp32, max-subtracted: moek.mojo:156-197 (route) and
    :385-425 (p_route). logits [T, E] fp32 -> ids int32 [T, topk], weights fp32 [T, topk]."""
    lg = np.asarray(logits, np.float32)
    t, e = lg.shape
    order = np.lexsort((np.broadcast_to(np.arange(e), lg.shape), -lg), axis=-1)[:, :topk]
    top = np.take_along_axis(lg, order, -1)
    ex = np.exp((top - top[:, :1]).astype(np.float32)).astype(np.float32)
    tot = np.zeros(t, np.float32)
    for k in range(topk):  # the reference's serial fp32 sum
        tot = (tot + ex[:, k]).astype(np.float32)
    return order.astype(np.int32), (ex / tot[:, None]).astype(np.float32)


def expert_lists(ids, n_experts):
    """For each expert e the pair indices i = t * topk + k with ids[t, k] == e, in increasing i,
    and their counts: moek.mojo:432-442 (p_expert_lists). Returns (offsets [E+1], pairs)."""
    flat = np.asarray(ids, np.int64).reshape(-1)
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=n_experts)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    return offsets.astype(np.int32), order.astype(np.int32)


def silu(v):
    return v / (1.0 + np.exp(-v))


def moe_layer(x, ids, weights, gu_wq, gu_ws, dn_wq, dn_ws, group, fe):
    """y[t] = sum_k w[t, k] * W_down[e] (silu(W_gate[e] x_t) * (W_up[e] x_t)), e = ids[t, k], in
    float64 on the dequantised experts. Expert e's gate rows are e*2fe .. e*2fe+fe-1 and its up
    rows follow (qwen3moe/export.py:166-169); down rows e*d .. e*d+d-1. Restates moe_gate_up /
    moe_down (moek.mojo:200-223) and t_moe_gate_up / t_moe_down / p_moe_sum (:479-488,:560-608)."""
    x = np.atleast_2d(np.asarray(x, np.float64))
    t, d = x.shape
    ids = np.asarray(ids).reshape(t, -1)
    wts = np.asarray(weights, np.float64).reshape(t, -1)
    y = np.zeros((t, d), np.float64)
    for e in np.unique(ids):
        tok, slot = np.nonzero(ids == e)
        gu = q4.dequant(gu_wq[e * 2 * fe:(e + 1) * 2 * fe], gu_ws[e * 2 * fe:(e + 1) * 2 * fe], group).astype(np.float64)
        dn = q4.dequant(dn_wq[e * d:(e + 1) * d], dn_ws[e * d:(e + 1) * d], group).astype(np.float64)
        h = x[tok] @ gu.T
        a = silu(h[:, :fe]) * h[:, fe:]
        y[tok] += wts[tok, slot][:, None] * (a @ dn.T)
    return y
