"""Top-k MoE operators over libmq, named after the reference's kernels (qwen3moe/kernels/moek.mojo).

Expert weights use the reference's layout (qwen3moe/export.py:166-169): gate|up int4 words
[experts * 2fe, d/8] (expert e: gate rows e*2fe .. e*2fe+fe-1, then its up rows) and down
[experts * d, fe/8], each with fp16 scales per `group` weights of a row.
"""
import torch

from ._lib import MQError, lib
from .kernels import MQ_F16, MQ_F32, _need, _p, _stream, _WORDS

__all__ = ["gemv_f32", "p_gemv_f32", "router", "p_route", "route", "p_expert_lists", "route_group", "moe_gemv_q4",
           "moe_gate_up", "moe_down", "moe_forward", "moe_layer", "TILE_M"]

TILE_M = 64  # tokens per expert work tile of the grouped products


def p_gemv_f32(w, x, y, cols, rows=None, tokens=None):
    """y[t, r] = W[r] . x[t] in fp32 for the router W [rows, cols]: p_gemv_f32 (moek.mojo:284-295) and,
    for one token, gemv_f32 (:143-153). x [tokens, cols], y [tokens, rows]."""
    _need(w, "w", (torch.float32,))
    rows = w.numel() // cols if rows is None else rows
    _need(x, "x", (torch.float32,))
    tokens = x.numel() // cols if tokens is None else tokens
    _need(y, "y", (torch.float32,), tokens * rows)
    lib.call("mq_moe_router", _p(w), _p(x), _p(y), tokens, rows, cols, _stream())
    return y


def gemv_f32(w, x, y, cols):
    """The one-token router GEMV (moek.mojo:143-153)."""
    return p_gemv_f32(w, x, y, cols)


def router(w, x, ids, weights, topk=8, logits=None):
    """The MoE layer's routing on the device: fp32 router logits, then the top-k experts and their
    softmax weights (the model's gemv_f32 + route, qwen3moe/model.mojo:208-209)."""
    d = x.shape[-1]
    tokens = x.numel() // d
    experts = w.numel() // d
    logits = torch.empty(tokens, experts, dtype=torch.float32, device=x.device) if logits is None else logits
    p_gemv_f32(w, x, logits, d, experts, tokens)
    return p_route(logits, ids, weights, topk)


def p_route(logits, ids, weights, topk=8):
    """Per token row: the top-k experts (lowest index among equal logits) and softmax weights over
    them -- p_route(logits, ids, weights) of moek.mojo:385-425 (route, :156-197, is one row).
    logits: fp32 [tokens, experts]; ids: int32 [tokens, topk]; weights: fp32 [tokens, topk]."""
    _need(logits, "logits", (torch.float32,))
    tokens, experts = logits.shape
    _need(ids, "ids", (torch.int32,), tokens * topk)
    _need(weights, "weights", (torch.float32,), tokens * topk)
    lib.call("mq_moe_route", _p(logits), _p(ids), _p(weights), tokens, experts, topk, _stream())
    return ids, weights


def route(logits, ids, weights, topk=8):
    """route(logits, ids, weights) of moek.mojo:156-197: one token's top-k and weights."""
    return p_route(logits.reshape(1, -1), ids, weights, topk)


def p_expert_lists(ids, experts, tile=TILE_M):
    """The pairs grouped by expert, stable: p_expert_lists + p_expert_items (moek.mojo:432-442,
    548-557). ids: int32 [tokens, topk]. Returns (counts, offsets, order, slot_of, tiles, ntiles)
    as int32 device tensors; tiles has room for experts + ceil(pairs / tile) items of 3 ints."""
    _need(ids, "ids", (torch.int32,))
    tokens, topk = ids.shape
    pairs = tokens * topk
    dev = ids.device
    max_tiles = experts + (pairs + tile - 1) // tile
    counts = torch.empty(experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
    order = torch.empty(pairs, dtype=torch.int32, device=dev)
    slot_of = torch.empty(pairs, dtype=torch.int32, device=dev)
    tiles = torch.empty(max_tiles * 3, dtype=torch.int32, device=dev)
    ntiles = torch.empty(1, dtype=torch.int32, device=dev)
    lib.call("mq_moe_group", _p(ids), tokens, topk, experts, tile, _p(counts), _p(offsets), _p(order), _p(slot_of),
             _p(tiles), _p(ntiles), _stream())
    return counts, offsets, order, slot_of, tiles, ntiles


def route_group(w, x, ids, weights, topk=8, logits=None, tile=TILE_M, group=True):
    """The router chain fused on the device: router logits (fp32 W [experts, d] . x [tokens, d]),
    the top-k experts and softmax weights of each token, and (group=True) the stable grouping of the
    pairs by expert -- gemv_f32 + route + p_expert_lists / p_expert_items (moek.mojo:143-197,
    432-442, 548-557) in two launches, the logits kept on chip (written to `logits` when given).
    Returns (ids, weights) and, with group, p_expert_lists' (counts, offsets, order, slot_of, tiles,
    ntiles)."""
    _need(x, "x", (torch.float32,))
    d = x.shape[-1]
    tokens = x.numel() // d
    _need(w, "w", (torch.float32,))
    experts = w.numel() // d
    _need(ids, "ids", (torch.int32,), tokens * topk)
    _need(weights, "weights", (torch.float32,), tokens * topk)
    if logits is not None:
        _need(logits, "logits", (torch.float32,), tokens * experts)
    if not group:
        lib.call("mq_moe_route_group", _p(w), _p(x), _p(logits) if logits is not None else None, _p(ids), _p(weights),
                 tokens, experts, topk, d, tile, None, None, None, None, None, None, _stream())
        return ids, weights
    pairs = tokens * topk
    dev = x.device
    max_tiles = experts + (pairs + tile - 1) // tile
    counts = torch.empty(experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
    order = torch.empty(pairs, dtype=torch.int32, device=dev)
    slot_of = torch.empty(pairs, dtype=torch.int32, device=dev)
    tiles = torch.empty(max_tiles * 3, dtype=torch.int32, device=dev)
    ntiles = torch.empty(1, dtype=torch.int32, device=dev)
    lib.call("mq_moe_route_group", _p(w), _p(x), _p(logits) if logits is not None else None, _p(ids), _p(weights),
             tokens, experts, topk, d, tile, _p(counts), _p(offsets), _p(order), _p(slot_of), _p(tiles), _p(ntiles),
             _stream())
    return (ids, weights), (counts, offsets, order, slot_of, tiles, ntiles)


def moe_gemv_q4(wq, ws, ids, x, y, k, group_rows, rows_per_group=None, group=32, x_per_group=False):
    """The decode GEMV over selected experts: y[i, r] = W[ids[i] * group_rows + r] . x_i for
    i < len(ids), r < rows_per_group (default group_rows); x_i = x, or x[i] with x_per_group.
    wq: int4 words [wrows, k/8]; ws fp16 [wrows, k/group]; x fp32; y fp32 [len(ids), rows_per_group]."""
    rows_per_group = group_rows if rows_per_group is None else rows_per_group
    _need(wq, "wq", _WORDS)
    wrows = wq.numel() * 8 // k
    _need(ws, "ws", (torch.float16,), wrows * k // group)
    _need(ids, "ids", (torch.int32,))
    n = ids.numel()
    _need(x, "x", (torch.float32,), n * k if x_per_group else k)
    _need(y, "y", (torch.float32,), n * rows_per_group)
    lib.call("mq_moe_gemv_q4", _p(wq), _p(ws), wrows, _p(x), _p(y), _p(ids), n, group_rows, rows_per_group, k, group,
             int(bool(x_per_group)), _stream())
    return y


def moe_gate_up(wq, ws, ids, x, a, d, fe, group=32):
    """a[e, j] = silu(gate_e[j] . x) * (up_e[j] . x) for the selected experts ids[e]: moe_gate_up of
    moek.mojo:200-210 (one token), one launch with the SwiGLU fused. x fp32 [d]; a fp32 [topk, fe]."""
    _need(wq, "wq", _WORDS)
    wrows = wq.numel() * 8 // d
    _need(ws, "ws", (torch.float16,), wrows * d // group)
    _need(ids, "ids", (torch.int32,))
    _need(x, "x", (torch.float32,), d)
    topk = ids.numel()
    _need(a, "a", (torch.float32,), topk * fe)
    lib.call("mq_moe_gate_up_q4", _p(wq), _p(ws), wrows, _p(x), _p(a), _p(ids), topk, fe, d, group, _stream())
    return a


def moe_down(wq, ws, ids, weights, a, x, d, fe, group=32, z=None):
    """x[r] += sum_e weights[e] * W_down[ids[e]][r] . a[e]: moe_down of moek.mojo:213-223 (one token),
    k in order. a fp32 [topk, fe]; x fp32 [d] (the residual stream); z: optional fp32 [topk, d] scratch."""
    topk = ids.numel()
    z = torch.empty(topk, d, dtype=torch.float32, device=x.device) if z is None else z
    moe_gemv_q4(wq, ws, ids, a, z, fe, d, group=group, x_per_group=True)
    _need(weights, "weights", (torch.float32,), topk)
    _need(x, "x", (torch.float32,), d)
    lib.call("mq_moe_combine", _p(z), None, _p(weights), 1, topk, d, 1, _p(x), _stream())
    return x


def moe_forward(x, ids, weights, gu_wq, gu_ws, dn_wq, dn_ws, y, d, fe, group=32, add=False, workspace=None):
    """y (+)= the MoE layer of the routed tokens: for each token t and slot k with expert e = ids[t, k],
    weights[t, k] * down_e(silu(gate_e x_t) * up_e x_t) -- moe_gate_up + moe_down for one token
    (moek.mojo:200-223) and t_moe_gate_up + t_moe_down + p_moe_sum for a prompt (:479-488, 560-608).
    x: fp32/fp16 [tokens, d]; ids int32, weights fp32 [tokens, topk]; y fp32 [tokens, d]."""
    _need(x, "x", (torch.float32, torch.float16))
    tokens = x.numel() // d
    _need(ids, "ids", (torch.int32,))
    topk = ids.numel() // tokens
    _need(weights, "weights", (torch.float32,), tokens * topk)
    _need(gu_wq, "gu_wq", _WORDS)
    experts = gu_wq.numel() * 8 // d // (2 * fe)
    _need(gu_ws, "gu_ws", (torch.float16,), experts * 2 * fe * d // group)
    _need(dn_wq, "dn_wq", _WORDS, experts * d * fe // 8)
    _need(dn_ws, "dn_ws", (torch.float16,), experts * d * fe // group)
    _need(y, "y", (torch.float32,), tokens * d)
    nbytes = lib.mq_moe_workspace_size(tokens, experts, topk, d, fe)
    if workspace is None:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    if workspace.numel() < nbytes:
        raise MQError(-1, f"workspace: {workspace.numel()} bytes < {nbytes}")
    lib.call("mq_moe_forward", _p(x), MQ_F16 if x.dtype == torch.float16 else MQ_F32, _p(ids), _p(weights), _p(gu_wq),
             _p(gu_ws), _p(dn_wq), _p(dn_ws), _p(y), tokens, experts, topk, d, fe, group, int(bool(add)),
             _p(workspace), nbytes, _stream())
    return y


def moe_layer(x, router_w, gu_wq, gu_ws, dn_wq, dn_ws, y, d, fe, group=32, topk=8, ids=None, weights=None, logits=None,
              add=False, workspace=None):
    """y (+)= the MoE layer with its router on the device, as the model runs it (qwen3moe/model.mojo:
    208-274): the fused router chain (route_group) picks each token's experts and weights, then the
    experts run as in moe_forward. x fp32 [tokens, d]; router_w fp32 [experts, d]; ids int32 and
    weights fp32 [tokens, topk] receive the routing (made when None), logits fp32 [tokens, experts]
    the router logits when given. Returns (y, ids, weights)."""
    _need(x, "x", (torch.float32,))
    tokens = x.numel() // d
    _need(router_w, "router_w", (torch.float32,))
    experts = router_w.numel() // d
    _need(gu_wq, "gu_wq", _WORDS, experts * 2 * fe * d // 8)
    _need(gu_ws, "gu_ws", (torch.float16,), experts * 2 * fe * d // group)
    _need(dn_wq, "dn_wq", _WORDS, experts * d * fe // 8)
    _need(dn_ws, "dn_ws", (torch.float16,), experts * d * fe // group)
    _need(y, "y", (torch.float32,), tokens * d)
    ids = torch.empty(tokens, topk, dtype=torch.int32, device=x.device) if ids is None else ids
    weights = torch.empty(tokens, topk, dtype=torch.float32, device=x.device) if weights is None else weights
    _need(ids, "ids", (torch.int32,), tokens * topk)
    _need(weights, "weights", (torch.float32,), tokens * topk)
    if logits is not None:
        _need(logits, "logits", (torch.float32,), tokens * experts)
    nbytes = lib.mq_moe_workspace_size(tokens, experts, topk, d, fe)
    if workspace is None:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    if workspace.numel() < nbytes:
        raise MQError(-1, f"workspace: {workspace.numel()} bytes < {nbytes}")
    lib.call("mq_moe_layer", _p(x), _p(router_w), _p(gu_wq), _p(gu_ws), _p(dn_wq), _p(dn_ws), _p(y), _p(ids),
             _p(weights), _p(logits) if logits is not None else None, tokens, experts, topk, d, fe, group,
             int(bool(add)), _p(workspace), nbytes, _stream())
    return y, ids, weights
