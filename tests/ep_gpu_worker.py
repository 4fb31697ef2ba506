"""One rank of the 2-GPU expert-parallel MoE check (launched by tests/test_ep_gpu.py through
torch.distributed.run): Qwen3-30B-A3B layer shapes, each rank with its own tokens and its 64 experts;
with EP_MAX_TOKENS the peer-memory exchange (rows written into the owners' buffers over NVLink),
without it the compact NCCL all-to-all. The rank's output is compared with the fp64 oracle layer on
the full expert set, over two layers in a row, eagerly and replayed from a CUDA graph (peer form)."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [REPO, os.path.join(REPO, "mojo-adreno_b200")]

import mq  # noqa: E402
from mq import synth  # noqa: E402
from oracle import moe as omoe  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        d, fe, experts, topk, group = 2048, 768, 128, 8, 32
        counts = [int(c) for c in os.environ.get("EP_TOKENS", "24,17").split(",")]
        m = synth.moe_layer(seed=0, tokens=sum(counts))
        lo_t = sum(counts[:rank])
        x = m["x"][lo_t:lo_t + counts[rank]]
        ids, w = omoe.route(m["logits"][lo_t:lo_t + counts[rank]], topk) if counts[rank] else (
            np.zeros((0, topk), np.int32), np.zeros((0, topk), np.float32))
        lo, hi = mq.expert_range(experts, world, rank)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a)).to(dev)
        moe = mq.ExpertParallelMoE(t(m["gu_wq"][lo * 2 * fe:hi * 2 * fe]), t(m["gu_ws"][lo * 2 * fe:hi * 2 * fe]),
                                   t(m["dn_wq"][lo * d:hi * d]), t(m["dn_ws"][lo * d:hi * d]), d, fe, experts, topk=topk,
                                   group=group, max_tokens=int(os.environ.get("EP_MAX_TOKENS") or 0) or None)
        ys = []
        tx, tids, tw = t(x), t(ids), t(w)
        for _ in range(2):  # two layers in a row through the same buffers
            y = torch.full((counts[rank], d), float("nan"), device=dev)
            moe(tx, tids, tw, y)
            ys.append(y)
        if moe.exchange == "peer":  # the same layer captured once and replayed twice
            yg = torch.full((counts[rank], d), float("nan"), device=dev)
            g = torch.cuda.CUDAGraph()
            torch.cuda.synchronize()
            with torch.cuda.graph(g):
                moe(tx, tids, tw, yg)
            for _ in range(2):
                g.replay()
            torch.cuda.synchronize()
            ys.append(yg.clone())
            del g
        torch.cuda.synchronize()
        assert mq.device_status() == 0
        dist.barrier()
        moe.close()
        if counts[rank]:
            ref = omoe.moe_layer(x, ids, w, m["gu_wq"], m["gu_ws"], m["dn_wq"], m["dn_ws"], group, fe)
            for y in ys:
                err = np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max()
                assert err <= 1e-3, f"rank {rank}: normwise error {err}"
        print(f"rank {rank}: ok ({counts[rank]} tokens)", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
