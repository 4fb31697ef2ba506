"""MoE parity on the GPU through the C ABI: routing and grouping bit-exact against the oracle,
the layer within the 1e-3 normwise bar (fp16 x and fp16 q*scale, fp32 accumulation)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, normwise
from oracle import moe as omoe
from oracle import q4 as oq4

import mq
from mq import synth

pytestmark = pytest.mark.gpu
TOL = 1e-3


def t(a, dev):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(dev)


@pytest.mark.parametrize("tokens,experts,topk", [(404, 128, 8), (1, 128, 8), (33, 60, 6), (7, 256, 32)])
def test_route_matches_oracle(cuda, tokens, experts, topk):
    rng = np.random.default_rng(tokens + experts)
    logits = rng.standard_normal((tokens, experts)).astype(np.float32)
    logits[0, :8] = logits[0, 8]  # ties: the lowest index wins
    ids = torch.empty(tokens, topk, dtype=torch.int32, device=cuda)
    w = torch.empty(tokens, topk, device=cuda)
    mq.p_route(t(logits, cuda), ids, w, topk=topk)
    torch.cuda.synchronize()
    rid, rw = omoe.route(logits, topk)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("tokens,experts,topk", [(404, 128, 8), (1, 128, 8), (300, 7, 3)])
def test_group_matches_oracle(cuda, tokens, experts, topk):
    rng = np.random.default_rng(7 + tokens)
    ids = np.stack([rng.choice(experts, topk, replace=False) for _ in range(tokens)]).astype(np.int32)
    counts, offsets, order, slot_of, tiles, ntiles = mq.p_expert_lists(t(ids, cuda), experts, tile=64)
    torch.cuda.synchronize()
    ro, rorder = omoe.expert_lists(ids, experts)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ro)
    np.testing.assert_array_equal(order.cpu().numpy(), rorder)
    so = slot_of.cpu().numpy()
    np.testing.assert_array_equal(so[rorder], np.arange(tokens * topk))
    nt = int(ntiles.item())
    tl = tiles.cpu().numpy()[:3 * nt].reshape(nt, 3)
    cnt = np.diff(ro)
    assert nt == int(np.sum((cnt + 63) // 64))
    for e, r0, rows in tl:
        assert ro[e] <= r0 and r0 + rows <= ro[e + 1] and 1 <= rows <= 64


def run_forward(cuda, x, ids, w, gu_wq, gu_ws, dn_wq, dn_ws, d, fe, group, add_to=None):
    tokens = x.shape[0]
    y = torch.full((tokens, d), float("nan"), device=cuda) if add_to is None else t(add_to, cuda)
    mq.moe_forward(t(x, cuda), t(ids, cuda), t(w, cuda), t(gu_wq, cuda), t(gu_ws, cuda), t(dn_wq, cuda), t(dn_ws, cuda), y,
                   d, fe, group=group, add=add_to is not None)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    return y.cpu().numpy()


def test_moe_forward_matches_transformers_block(cuda):
    z = np.load(os.path.join(GOLDEN, "moe_block.npz"))
    y = run_forward(cuda, z["x"], z["ids"], z["weights"], z["gu_wq"], z["gu_ws"], z["dn_wq"], z["dn_ws"], int(z["d"]),
                    int(z["fe"]), int(z["group"]))
    assert normwise(y, z["y"]) <= TOL


@pytest.mark.parametrize("tokens", [404, 1, 2, 3])
def test_moe_forward_baseline_config(cuda, tokens):
    """Qwen3-30B-A3B MoE layer shapes (hidden 2048, 128 experts, top-8, FE 768,
    int4 G=32); 404 prompt tokens, and 1-token decode."""
    m = synth.moe_layer(seed=0, tokens=tokens)
    ids, w = omoe.route(m["logits"], 8)
    r = np.random.default_rng(1).standard_normal((tokens, 2048)).astype(np.float32)
    y = run_forward(cuda, m["x"], ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 2048, 768, 32, add_to=r.copy())
    ref = r + omoe.moe_layer(m["x"], ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 32, 768)
    assert normwise(y, ref) <= TOL


@pytest.mark.parametrize("tokens,topk", [(2, 8), (16, 1), (5, 3)])
def test_moe_forward_small_pairs_fp16(cuda, tokens, topk):
    """Up to 16 (token, expert) pairs run on the streaming GEMVs with each pair's own fp16 x (a small
    decode batch, an expert-parallel rank's rows): the layer oracle on the fp16-rounded x."""
    m = synth.moe_layer(seed=7, tokens=tokens)
    ids, w = omoe.route(m["logits"], topk)
    x16 = m["x"].astype(np.float16)
    y = run_forward(cuda, x16, ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 2048, 768, 32)
    ref = omoe.moe_layer(x16.astype(np.float32), ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 32, 768)
    assert normwise(y, ref) <= TOL


@pytest.mark.parametrize("group", [64, 128])
@pytest.mark.parametrize("tokens,x16", [(404, False), (1, False), (2, True)])
def test_moe_forward_groups(cuda, group, tokens, x16):
    """The layer with G = 64 and G = 128 scales (qwen3moe exports its experts at G = 128,
    qwen3moe/export.py:38-39,171-175) on each path: 404 tokens through the grouped tensor-core products,
    one fp32 token through the decode GEMVs, two fp16 tokens (16 pairs) through the small-pair GEMVs."""
    m = synth.moe_layer(seed=group + tokens, tokens=tokens, group=group)
    ids, w = omoe.route(m["logits"], 8)
    x = m["x"].astype(np.float16) if x16 else m["x"]
    y = run_forward(cuda, x, ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 2048, 768, group)
    ref = omoe.moe_layer(x.astype(np.float32), ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], group, 768)
    assert normwise(y, ref) <= TOL


@pytest.mark.parametrize("group,x_per_group", [(32, False), (32, True), (64, True), (128, False), (128, True)])
def test_moe_gemv_matches_oracle(cuda, group, x_per_group):
    """The expert-indirect decode GEMV: rows of the selected experts only, shared or per-expert x."""
    rng = np.random.default_rng(group + x_per_group)
    experts, rows, k, n = 16, 192, 768, 8
    wq, ws = synth.q4_matrix(rng, experts * rows, k, group)
    ids = rng.choice(experts, n, replace=False).astype(np.int32)
    ids[3] = ids[5]  # the same expert twice
    x = rng.standard_normal((n, k) if x_per_group else (k,)).astype(np.float32)
    y = torch.full((n, rows), float("nan"), device=cuda)
    mq.moe_gemv_q4(t(wq, cuda), t(ws, cuda), t(ids, cuda), t(x, cuda), y, k, rows, group=group, x_per_group=x_per_group)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    w = oq4.dequant(wq, ws, group).astype(np.float64).reshape(experts, rows, k)[ids]
    xx = np.broadcast_to(np.atleast_2d(x), (n, k)).astype(np.float64)
    ref = np.einsum("erk,ek->er", w, xx)
    assert normwise(y.cpu().numpy(), ref) <= TOL


def test_moe_gate_up_down_decode(cuda):
    """moe_gate_up then moe_down on one token (the reference's decode pair) against the layer oracle."""
    m = synth.moe_layer(seed=3, tokens=1)
    ids, w = omoe.route(m["logits"], 8)
    x = t(m["x"][0], cuda)
    a = torch.empty(8, 768, device=cuda)
    mq.moe_gate_up(t(m["gu_wq"], cuda), t(m["gu_ws"], cuda), t(ids[0], cuda), x, a, 2048, 768)
    r = np.random.default_rng(4).standard_normal(2048).astype(np.float32)
    res = t(r, cuda)
    mq.moe_down(t(m["dn_wq"], cuda), t(m["dn_ws"], cuda), t(ids[0], cuda), t(w[0], cuda), a, res, 2048, 768)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    ref = r + omoe.moe_layer(m["x"], ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], 32, 768)[0]
    assert normwise(res.cpu().numpy(), ref) <= TOL


def test_moe_gate_up_fused_is_the_unfused_pair(cuda):
    """The fused moe_gate_up (one launch) is bit-identical to the expert GEMV over the 2fe gate|up rows
    followed by the SwiGLU kernel: the same products in the same order."""
    m = synth.moe_layer(seed=5, tokens=1)
    ids, _ = omoe.route(m["logits"], 8)
    x = t(m["x"][0], cuda)
    gu_wq, gu_ws, tid = t(m["gu_wq"], cuda), t(m["gu_ws"], cuda), t(ids[0], cuda)
    a = torch.full((8, 768), float("nan"), device=cuda)
    mq.moe_gate_up(gu_wq, gu_ws, tid, x, a, 2048, 768)
    h = torch.empty(8, 2 * 768, device=cuda)
    mq.moe_gemv_q4(gu_wq, gu_ws, tid, x, h, 2048, 2 * 768)
    a2 = torch.empty(8, 768, device=cuda)
    mq.lib.call("mq_moe_silu_mul", h.data_ptr(), a2.data_ptr(), 8, 768, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    np.testing.assert_array_equal(a.cpu().numpy(), a2.cpu().numpy())


@pytest.mark.parametrize("tokens,experts,d", [(404, 128, 2048), (1, 128, 2048), (7, 60, 768), (33, 128, 4100)])
def test_router_logits_and_routing(cuda, tokens, experts, d):
    """The fp32 router GEMV against float64, then routing on its logits bit-exact against the oracle."""
    rng = np.random.default_rng(tokens + experts + d)
    w = (rng.standard_normal((experts, d)) * 0.02).astype(np.float32)
    x = rng.standard_normal((tokens, d)).astype(np.float32)
    logits = torch.empty(tokens, experts, device=cuda)
    ids = torch.empty(tokens, 8, dtype=torch.int32, device=cuda)
    wts = torch.empty(tokens, 8, device=cuda)
    mq.router(t(w, cuda), t(x, cuda), ids, wts, topk=8, logits=logits)
    torch.cuda.synchronize()
    got = logits.cpu().numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert normwise(got, ref) <= 1e-5
    rid, rw = omoe.route(got, 8)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(wts.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("tokens,experts,d,topk", [(404, 128, 2048, 8), (1, 128, 2048, 8), (7, 60, 768, 8),
                                                   (33, 128, 4100, 8), (17, 256, 512, 8), (5, 20, 64, 8),
                                                   (64, 128, 2048, 2), (3, 16, 256, 1)])
def test_route_group_fused_chain(cuda, tokens, experts, d, topk):
    """The fused router chain (one cluster kernel: router GEMV + top-k + softmax from distributed shared
    memory, then the grouping): logits against float64, routing bit-exact against the oracle on the
    chain's own logits, grouping bit-exact against the oracle's expert lists of those ids."""
    rng = np.random.default_rng(3 * tokens + experts + d)
    w = (rng.standard_normal((experts, d)) * 0.02).astype(np.float32)
    x = rng.standard_normal((tokens, d)).astype(np.float32)
    logits = torch.empty(tokens, experts, device=cuda)
    ids = torch.empty(tokens, topk, dtype=torch.int32, device=cuda)
    wts = torch.empty(tokens, topk, device=cuda)
    (_, _), (counts, offsets, order, slot_of, tiles, ntiles) = mq.route_group(t(w, cuda), t(x, cuda), ids, wts, topk=topk,
                                                                             logits=logits)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    got = logits.cpu().numpy()
    assert normwise(got, x.astype(np.float64) @ w.astype(np.float64).T) <= 1e-5
    rid, rw = omoe.route(got, topk)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(wts.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    ro, rorder = omoe.expert_lists(rid, experts)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ro)
    np.testing.assert_array_equal(counts.cpu().numpy(), np.diff(ro))
    np.testing.assert_array_equal(order.cpu().numpy(), rorder)
    np.testing.assert_array_equal(slot_of.cpu().numpy()[rorder], np.arange(tokens * topk))
    assert int(ntiles.item()) == int(np.sum((np.diff(ro) + 63) // 64))
    # without the grouping and without a logits buffer (a few tokens then take the cluster kernel too)
    ids2 = torch.empty_like(ids)
    wts2 = torch.empty_like(wts)
    mq.route_group(t(w, cuda), t(x, cuda), ids2, wts2, topk=topk, group=False)
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    if tokens > 4:  # the same kernel as above: the same routing, bit for bit
        np.testing.assert_array_equal(ids2.cpu().numpy(), rid)
        np.testing.assert_array_equal(wts2.cpu().numpy(), wts.cpu().numpy())
    else:  # the cluster kernel sums in another order: routing of near-equal logits may differ, so check
        # its weights against the oracle on the first logits where the chosen experts agree
        same = (ids2.cpu().numpy() == rid).all(axis=1)
        assert same.mean() >= 0.5
        np.testing.assert_allclose(wts2.cpu().numpy()[same], rw[same], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("tokens,group", [(404, 32), (1, 32), (2, 32), (3, 32), (404, 128), (1, 128)])
def test_moe_layer_with_router(cuda, tokens, group):
    """The whole layer with its router on the device (mq_moe_layer), in a CUDA graph replayed twice:
    the routing equals the oracle's on the chain's logits, the output the fp64 layer on that routing.
    1 token runs the decode GEMVs, 2 tokens (16 pairs) the small-pair GEMVs, 3 and 404 the grouped
    tensor-core products on the chain's grouping."""
    m = synth.moe_layer(seed=11, tokens=tokens, group=group)
    rw = (np.random.default_rng(5).standard_normal((128, 2048)) * 0.02).astype(np.float32)
    tx, trw = t(m["x"], cuda), t(rw, cuda)
    gw = [t(m[k], cuda) for k in ("gu_wq", "gu_ws", "dn_wq", "dn_ws")]
    y = torch.full((tokens, 2048), float("nan"), device=cuda)
    ids = torch.empty(tokens, 8, dtype=torch.int32, device=cuda)
    wts = torch.empty(tokens, 8, device=cuda)
    logits = torch.empty(tokens, 128, device=cuda)
    ws = torch.empty(mq.lib.mq_moe_workspace_size(tokens, 128, 8, 2048, 768), dtype=torch.uint8, device=cuda)
    mq.moe_layer(tx, trw, *gw, y, 2048, 768, group=group, ids=ids, weights=wts, logits=logits, workspace=ws)
    torch.cuda.synchronize()
    y.fill_(float("nan"))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        mq.moe_layer(tx, trw, *gw, y, 2048, 768, group=group, ids=ids, weights=wts, logits=logits, workspace=ws)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert mq.device_status() == 0
    rid, rwts = omoe.route(logits.cpu().numpy(), 8)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(wts.cpu().numpy(), rwts, rtol=2e-6, atol=1e-7)
    ref = omoe.moe_layer(m["x"], rid, rwts, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], group, 768)
    assert normwise(y.cpu().numpy(), ref) <= TOL
