"""Expert-parallel MoE host logic on CPU: world_size 2 gloo ranks exchange rows through the same
ExpertParallelMoE code the GPU path runs, with the device steps replaced by the oracle
(plan = stable sort by owning rank, experts = the fp64 layer oracle). Each rank's output must equal
the one-device layer over the same tokens."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe as omoe

D, FE, E, TOPK, G = 256, 256, 8, 3, 32


class OracleOps:
    """ExpertParallelMoE's device steps, restated on CPU tensors with the oracle."""

    def plan(self, ids, tokens, topk, experts, world, capacity=0):
        per = experts // world
        flat = ids.reshape(-1).numpy().astype(np.int64)
        dest = flat // per
        order = np.argsort(dest, kind="stable")
        slot_of = np.empty_like(order)
        slot_of[order] = np.arange(order.size)
        counts = np.bincount(dest, minlength=world)
        local = (flat - dest * per)[order]
        if capacity:  # rank r's pairs at r * capacity + i, empty positions -1
            starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
            pos = dest[order] * capacity + (np.arange(order.size) - starts[dest[order]])
            porder = np.full(world * capacity, -1, np.int64)
            plocal = np.full(world * capacity, -1, np.int64)
            porder[pos], plocal[pos] = order, local
            slot_of[order] = pos
            order, local = porder, plocal
        return tuple(torch.from_numpy(a.astype(np.int32)) for a in (counts, order, slot_of, local))

    def gather(self, x, order, topk, d):
        o = order.long()
        rows = x[o.clamp(min=0) // topk].half()
        rows[o < 0] = 0  # empty positions of the fixed-capacity layout
        return rows

    def experts(self, rows, local_ids, gu_wq, gu_ws, dn_wq, dn_ws, d, fe, group):
        r = rows.shape[0]
        lid = local_ids.numpy().reshape(r, 1)
        live = lid[:, 0] >= 0
        y = np.zeros((r, d), np.float32)
        if live.any():
            y[live] = omoe.moe_layer(rows.float().numpy()[live], lid[live], np.ones((int(live.sum()), 1)), gu_wq, gu_ws,
                                     dn_wq, dn_ws, group, fe)
        return torch.from_numpy(y)

    def combine(self, ret, slot_of, weights, tokens, topk, d, add, y):
        z = ret.numpy()[slot_of.numpy()].reshape(tokens, topk, d).astype(np.float64)
        w = weights.numpy().reshape(tokens, topk).astype(np.float64)
        out = np.zeros((tokens, d))
        for k in range(topk):
            out += w[:, k:k + 1] * z[:, k]
        y.copy_(torch.from_numpy((y.numpy() if add else 0) + out).float())
        return y


def layer(seed=0):
    rng = np.random.default_rng(seed)
    gu_wq, gu_ws = oq4_matrix(rng, E * 2 * FE, D)
    dn_wq, dn_ws = oq4_matrix(rng, E * D, FE)
    return gu_wq, gu_ws, dn_wq, dn_ws


def oq4_matrix(rng, n, k):
    ws = np.abs(rng.normal(0, 0.02, (n, k // G))).astype(np.float16)
    wq = rng.integers(0, 1 << 32, (n, k // 8), dtype=np.uint32)
    return wq, ws


def tokens_of(rank, counts, seed=1):
    rng = np.random.default_rng(seed + rank)
    t = counts[rank]
    x = rng.standard_normal((t, D)).astype(np.float32)
    logits = rng.standard_normal((t, E)).astype(np.float32)
    if t:
        ids, w = omoe.route(logits, TOPK)
    else:
        ids, w = np.zeros((0, TOPK), np.int32), np.zeros((0, TOPK), np.float32)
    return x, ids, w


def _worker(rank, world, port, counts, add, max_tokens=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import mq

        gu_wq, gu_ws, dn_wq, dn_ws = layer()
        lo, hi = mq.expert_range(E, world, rank)
        moe = mq.ExpertParallelMoE(gu_wq[lo * 2 * FE:hi * 2 * FE], gu_ws[lo * 2 * FE:hi * 2 * FE], dn_wq[lo * D:hi * D],
                                   dn_ws[lo * D:hi * D], D, FE, E, topk=TOPK, group=G, ops=OracleOps(),
                                   max_tokens=max_tokens)
        x, ids, w = tokens_of(rank, counts)
        base = np.random.default_rng(9).standard_normal((counts[rank], D)).astype(np.float32)
        y = torch.from_numpy(base.copy()) if add else torch.full((counts[rank], D), float("nan"))
        moe(torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(w), y, add=add)
        if counts[rank]:
            xr = x.astype(np.float16).astype(np.float32)  # the rows travel in fp16
            ref = omoe.moe_layer(xr, ids, w, gu_wq, gu_ws, dn_wq, dn_ws, G, FE) + (base if add else 0)
            err = np.abs(y.numpy() - ref).max() / np.abs(ref).max()
            assert err < 1e-5, f"rank {rank}: normwise error {err}"
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("counts,add", [((5, 3), False), ((4, 0), True), ((1, 6), True)])
def test_expert_parallel_two_ranks_matches_one_device(counts, add):
    mp.spawn(_worker, args=(2, _port(), counts, add), nprocs=2, join=True)


@pytest.mark.parametrize("counts,add", [((5, 3), False), ((0, 6), True)])
def test_expert_parallel_fixed_capacity_two_ranks(counts, add):
    """The fixed-capacity exchange (static split sizes, no host read): the same layer."""
    mp.spawn(_worker, args=(2, _port(), counts, add, max(counts)), nprocs=2, join=True)


def test_expert_parallel_single_rank_is_the_layer():
    import mq

    gu_wq, gu_ws, dn_wq, dn_ws = layer()
    moe = mq.ExpertParallelMoE(gu_wq, gu_ws, dn_wq, dn_ws, D, FE, E, topk=TOPK, group=G, ops=OracleOps())
    x, ids, w = tokens_of(0, (7,))
    y = torch.zeros(7, D)
    moe(torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(w), y)
    ref = omoe.moe_layer(x.astype(np.float16).astype(np.float32), ids, w, gu_wq, gu_ws, dn_wq, dn_ws, G, FE)
    assert np.abs(y.numpy() - ref).max() / np.abs(ref).max() < 1e-5


def test_expert_range_rejects_uneven_split():
    import mq

    assert mq.expert_range(128, 8, 3) == (48, 64)
    with pytest.raises(mq.MQError):
        mq.expert_range(128, 3, 0)


def test_oracle_plan_fixed_capacity_layout():
    ids = torch.tensor([[7, 0, 4], [1, 6, 2]], dtype=torch.int32)
    counts, order, slot_of, local = OracleOps().plan(ids, 2, 3, 8, 2, capacity=4)
    assert counts.tolist() == [3, 3]
    assert order.tolist() == [1, 3, 5, -1, 0, 2, 4, -1]
    assert local.tolist() == [0, 1, 2, -1, 3, 0, 2, -1]
    assert slot_of.tolist() == [4, 0, 5, 1, 6, 2]


def test_oracle_plan_is_stable_by_owner():
    ids = torch.tensor([[7, 0, 4], [1, 6, 2]], dtype=torch.int32)
    counts, order, slot_of, local = OracleOps().plan(ids, 2, 3, 8, 2)
    assert counts.tolist() == [3, 3]
    assert order.tolist() == [1, 3, 5, 0, 2, 4]
    assert local.tolist() == [0, 1, 2, 3, 0, 2]
    assert slot_of[order.long()].tolist() == list(range(6))
