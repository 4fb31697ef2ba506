"""Expert-parallel MoE on the GPU: the dispatch plan bit-exact against the oracle, the layer at
world 1 through the device steps, and (with 2 visible GPUs) 2 ranks over NCCL."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import normwise
from oracle import moe as omoe
from test_ep_cpu import OracleOps

import mq
from mq import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,experts,topk,world", [(404, 128, 8, 8), (1, 128, 8, 2), (300, 60, 6, 4), (5, 8, 3, 1)])
def test_ep_plan_matches_oracle(cuda, tokens, experts, topk, world):
    rng = np.random.default_rng(tokens + world)
    ids = np.stack([rng.choice(experts, topk, replace=False) for _ in range(tokens)]).astype(np.int32)
    tids = torch.from_numpy(ids).to(cuda)
    counts, order, slot_of, local = mq.ep.DeviceOps().plan(tids, tokens, topk, experts, world)
    torch.cuda.synchronize()
    rc, ro, rs, rl = OracleOps().plan(torch.from_numpy(ids), tokens, topk, experts, world)
    for got, want in ((counts, rc), (order, ro), (slot_of, rs), (local, rl)):
        np.testing.assert_array_equal(got.cpu().numpy(), want.numpy())
    assert mq.device_status() == 0


def test_ep_plan_reports_out_of_range_ids(cuda):
    """An expert id past the layer is reported through the device status and left out of the plan."""
    ids = torch.tensor([[0, 9], [3, 1]], dtype=torch.int32, device=cuda)
    counts, order, slot_of, local = mq.ep.DeviceOps().plan(ids, 2, 2, 8, 2)
    torch.cuda.synchronize()
    assert mq.device_status() == 8
    assert counts.cpu().tolist() == [3, 0]
    assert order.cpu().tolist()[:3] == [0, 2, 3]


@pytest.mark.parametrize("tokens,experts,topk,world", [(404, 128, 8, 8), (1, 128, 8, 2), (37, 60, 6, 4)])
def test_ep_plan_fixed_capacity_matches_oracle(cuda, tokens, experts, topk, world):
    rng = np.random.default_rng(tokens + 7 * world)
    ids = np.stack([rng.choice(experts, topk, replace=False) for _ in range(tokens)]).astype(np.int32)
    cap = tokens * topk
    counts, order, slot_of, local = mq.ep.DeviceOps().plan(torch.from_numpy(ids).to(cuda), tokens, topk, experts, world, cap)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    rc, ro, rs, rl = OracleOps().plan(torch.from_numpy(ids), tokens, topk, experts, world, capacity=cap)
    for got, want in ((counts, rc), (order, ro), (slot_of, rs), (local, rl)):
        np.testing.assert_array_equal(got.cpu().numpy(), want.numpy())


def test_ep_plan_negative_ids_and_overflow(cuda):
    """-1 is "no expert": left out silently. A rank's pairs past the capacity are reported (9)."""
    ids = torch.tensor([[0, -1], [3, 1]], dtype=torch.int32, device=cuda)
    counts, order, slot_of, local = mq.ep.DeviceOps().plan(ids, 2, 2, 8, 2, 4)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    assert counts.cpu().tolist() == [3, 0] and slot_of.cpu().tolist() == [0, -1, 1, 2]
    counts, order, slot_of, local = mq.ep.DeviceOps().plan(ids, 2, 2, 8, 2, 2)
    torch.cuda.synchronize()
    assert mq.device_status() == 9
    assert slot_of.cpu().tolist() == [0, -1, 1, -1]


@pytest.mark.parametrize("max_tokens", [None, 37, 50])
def test_ep_single_rank_device_path(cuda, max_tokens):
    m = synth.moe_layer(seed=2, tokens=37)
    ids, w = omoe.route(m["logits"], 8)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a)).to(cuda)
    moe = mq.ExpertParallelMoE(t(m["gu_wq"]), t(m["gu_ws"]), t(m["dn_wq"]), t(m["dn_ws"]), 2048, 768, 128,
                               max_tokens=max_tokens)
    y = torch.full((37, 2048), float("nan"), device=cuda)
    moe(t(m["x"]), t(ids), t(w), y)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    ref = omoe.moe_layer(m["x"], ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 32, 768)
    assert normwise(y.cpu().numpy(), ref) <= 1e-3


@pytest.mark.parametrize("tokens", [1, 2, 3])
def test_ep_peer_small_and_grouped_owner_paths(cuda, tokens):
    """The peer form's owner step picks its path on the device: at most 16 received pairs run on the
    per-pair GEMVs over the compacted rows (1 and 2 tokens), more on the grouped products (3 tokens =
    24 pairs); both against the fp64 oracle, twice in a row."""
    m = synth.moe_layer(seed=10 + tokens, tokens=tokens)
    ids, w = omoe.route(m["logits"], 8)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a)).to(cuda)
    moe = mq.ExpertParallelMoE(t(m["gu_wq"]), t(m["gu_ws"]), t(m["dn_wq"]), t(m["dn_ws"]), 2048, 768, 128,
                               max_tokens=tokens)
    assert moe.exchange == "peer"
    ref = omoe.moe_layer(m["x"], ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 32, 768)
    for _ in range(2):
        y = torch.full((tokens, 2048), float("nan"), device=cuda)
        moe(t(m["x"]), t(ids), t(w), y)
        torch.cuda.synchronize()
        assert mq.device_status() == 0
        assert normwise(y.cpu().numpy(), ref) <= 1e-3


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("tokens,max_tokens", [("24,17", ""), ("0,9", ""), ("24,17", "24"), ("1,1", "1")])
def test_expert_parallel_two_gpus(cuda, tokens, max_tokens):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    worker = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ep_gpu_worker.py")
    env = dict(os.environ, EP_TOKENS=tokens, EP_MAX_TOKENS=max_tokens, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_port()), worker]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-4000:]
