"""Top-k MoE operators over libmq, named after the reference's kernels (qwen3moe/kernels/moek.mojo).

Expert weights use the reference's layout (qwen3moe/export.py:166-169): gate|up int4 words
[experts * 2fe, d/8] (expert e: gate rows e*2fe .. e*2fe+fe-1, then its up rows) and down
[experts * d, fe/8], each with fp16 scales per `group` weights of a row.
"""
import torch

from ._lib import MQError, lib
from .kernels import MQ_F16, MQ_F32, _need, _p, _stream, _WORDS

__all__ = ["p_route", "route", "p_expert_lists", "moe_forward", "TILE_M"]

TILE_M = 64  # tokens per expert work tile of the grouped products


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
