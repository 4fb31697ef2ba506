"""Expert-parallel MoE layer over torch.distributed (NCCL over NVLink on a B200 node).

The reference runs the whole qwen3moe layer on one device (qwen3moe/kernels/moek.mojo:432-608). Here
the 128 experts are split into `world` contiguous ranges: rank r owns experts [r * E / world,
(r + 1) * E / world) and holds only their rows of the gate|up and down matrices (contiguous slices
of the reference's layout, qwen3moe/export.py:166-169). Each rank routes its own tokens; one layer
is then:

  1. plan (device): the rank's tokens * topk (token, slot) pairs grouped stably by owning rank
     (mq_ep_plan), with the expert id local to the owner.
  2. dispatch: counts, then fp16 activation rows and local expert ids, all-to-all.
  3. the owner runs its experts on the rows it received (mq_moe_forward with topk = 1, weight 1).
  4. combine: the fp32 expert outputs return all-to-all in the order they were sent, and the home
     rank sums them per token with the routing weights in slot order (mq_moe_combine), as p_moe_sum
     does (moek.mojo:479-488).

Every rank takes the same collective steps in the same order, also when it sends or receives no
rows. Three exchange forms:

- peer (the default when max_tokens is given): no NCCL on the data path. Each rank exports one
  device buffer through CUDA IPC and maps the others' (NVLink peer memory); a layer is then a chain
  of kernels on the stream -- mq_ep_plan, mq_ep_dispatch (the pairs' rows written straight into
  their owners' receive buffers, at fixed per-sender slots), mq_ep_expert_step (waits for the rows,
  runs the owner's experts, writes the outputs straight back into the senders' return buffers),
  mq_ep_combine (waits for them, sums per token) -- with epoch flags and bounded waits, no host
  read, so a whole layer can be captured in a CUDA graph. Only real pairs cross NVLink.

- compact (default): only the pairs travel; the split sizes are exchanged first and read on the host
  (one small device-to-host copy per layer), which the variable-size all-to-all needs.
- fixed capacity (max_tokens given): every rank sends max_tokens * topk row slots to every rank, its
  pairs first and empty slots (expert id -1, zero rows) after them. The split sizes are static, so
  the layer needs no host read and stays asynchronous on the stream; the price is the empty slots'
  bytes on NVLink (the experts skip them).
"""
import ctypes

import torch
import torch.distributed as dist

from ._lib import MQError, lib
from .kernels import MQ_F16, MQ_F32, _need, _p, _stream, _WORDS
from .moe import TILE_M  # noqa: F401  (same grouped-product tile as the one-device layer)

__all__ = ["ExpertParallelMoE", "expert_range"]


def expert_range(experts, world, rank):
    """[first, last) experts owned by `rank`."""
    if experts % world:
        raise MQError(-1, f"experts ({experts}) must be a multiple of world ({world})")
    per = experts // world
    return rank * per, (rank + 1) * per


class DeviceOps:
    """The layer's device steps, each one libmq entry point on the current CUDA stream."""

    def plan(self, ids, tokens, topk, experts, world, capacity=0):
        """capacity 0: the compact send order; > 0: the fixed-capacity layout (world * capacity slots)."""
        dev = ids.device
        pairs = tokens * topk
        slots = world * capacity if capacity else pairs
        counts = torch.empty(world, dtype=torch.int32, device=dev)
        offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
        order = torch.empty(slots, dtype=torch.int32, device=dev)
        slot_of = torch.empty(pairs, dtype=torch.int32, device=dev)
        local = torch.empty(slots, dtype=torch.int32, device=dev)
        lib.call("mq_ep_plan", _p(ids), tokens, topk, experts, world, capacity, _p(counts), _p(offsets), _p(order),
                 _p(slot_of), _p(local), _stream())
        return counts, order, slot_of, local

    def gather(self, x, order, topk, d):
        pairs = order.numel()
        xg = torch.empty(pairs, d, dtype=torch.float16, device=x.device)
        lib.call("mq_moe_gather", _p(x), MQ_F16 if x.dtype == torch.float16 else MQ_F32, _p(order), pairs, topk, d,
                 _p(xg), _stream())
        return xg

    def experts(self, rows, local_ids, gu_wq, gu_ws, dn_wq, dn_ws, d, fe, group):
        """Each row through its expert (local id); rows with id -1 are skipped (their outputs unused)."""
        from .moe import moe_forward

        r = rows.shape[0]
        out = torch.empty(r, d, dtype=torch.float32, device=rows.device)
        ones = self._ones.get((r, rows.device))
        if ones is None:
            ones = self._ones[(r, rows.device)] = torch.ones(r, dtype=torch.float32, device=rows.device)
        moe_forward(rows, local_ids, ones, gu_wq, gu_ws, dn_wq, dn_ws, out, d, fe, group=group)
        return out

    def __init__(self):
        self._ones = {}

    def combine(self, ret, slot_of, weights, tokens, topk, d, add, y):
        lib.call("mq_moe_combine", _p(ret), _p(slot_of), _p(weights), tokens, topk, d, int(bool(add)), _p(y), _stream())
        return y


class PeerBuffers:
    """One rank's exchange buffers for the peer form, and device tables of every rank's buffers.

    One allocation holds rows fp16 [world * cap, d] (received rows), ids int32 [world * cap], ret fp32
    [world * cap, d] (returned outputs), flags int32 [2, world], the epoch and two arrival counters, all
    zeroed. It is exported with mq_ipc_handle; the other ranks' allocations are mapped with mq_ipc_open
    (one mapping per peer). Table entry r of peer_* is rank r's buffer as this device addresses it."""

    def __init__(self, world, rank, cap, d, device, pg=None):
        slots = world * cap
        parts = [("rows", slots * d * 2), ("ids", slots * 4), ("ret", slots * d * 4), ("flags", 2 * world * 4),
                 ("epoch", 4), ("done", 8)]
        self.off, at = {}, 0
        for name, n in parts:
            self.off[name] = at
            at += (n + 255) // 256 * 256
        self.buf = torch.zeros(at, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)  # zeroed before any peer can write into it
        base = self.buf.data_ptr()
        self.opened = []
        bases = [base] * world
        if world > 1:
            handle, offset = (ctypes.c_char * 64)(), ctypes.c_int64()
            lib.call("mq_ipc_handle", base, ctypes.cast(handle, ctypes.c_void_p), ctypes.byref(offset))
            metas = [None] * world
            dist.all_gather_object(metas, (bytes(handle), offset.value), group=pg)
            for s_, (hb, ob) in enumerate(metas):
                if s_ == rank:
                    continue
                ptr = ctypes.c_void_p()
                hbuf = ctypes.create_string_buffer(hb, 64)
                lib.call("mq_ipc_open", ctypes.cast(hbuf, ctypes.c_void_p), ob, ctypes.byref(ptr))
                bases[s_] = ptr.value
                self.opened.append((ptr.value, ob))
            dist.barrier(group=pg)  # every rank mapped every buffer before any layer runs

        def table(name):
            return torch.tensor([b + self.off[name] for b in bases], dtype=torch.int64, device=device)

        self.peer_rows, self.peer_ids, self.peer_ret, self.peer_flags = (table(n) for n in ("rows", "ids", "ret", "flags"))
        self.ptr = {name: base + o for name, o in self.off.items()}
        self.ret = self.buf[self.off["ret"]:self.off["ret"] + slots * d * 4].view(torch.float32).view(slots, d)

    def close(self):
        for ptr, off in self.opened:
            lib.call("mq_ipc_close", ptr, off)
        self.opened = []


class ExpertParallelMoE:
    """One rank's share of an expert-parallel MoE layer.

    gu_wq / gu_ws / dn_wq / dn_ws hold only this rank's experts (expert_range): gate|up words
    [E_local * 2fe, d/8], down [E_local * d, fe/8], fp16 scales per `group`. `experts` is the
    layer's total. forward(x, ids, weights, y) takes this rank's tokens: x [T, d] fp32 or fp16, ids
    int32 and weights fp32 [T, topk] from the router, and writes (or adds into) y fp32 [T, d].
    share: another layer of the same shape (peer exchange) whose peer buffers and workspace this
    layer uses too -- the layers of a model run one after another on the stream, so one set of
    buffers serves them all; only the layer that made the buffers unmaps them (close).
    """

    def __init__(self, gu_wq, gu_ws, dn_wq, dn_ws, d, fe, experts, topk=8, group=32, pg=None, ops=None,
                 max_tokens=None, exchange=None, share=None):
        self.pg = pg
        self.world = dist.get_world_size(pg) if dist.is_initialized() else 1
        self.rank = dist.get_rank(pg) if dist.is_initialized() else 0
        self.first, self.last = expert_range(experts, self.world, self.rank)
        self.d, self.fe, self.experts, self.topk, self.group = d, fe, experts, topk, group
        self.capacity = max_tokens * topk if max_tokens else 0  # row slots per rank pair (fixed-capacity form)
        local = self.last - self.first
        self.ops = ops if ops is not None else DeviceOps()
        if ops is None:
            _need(gu_wq, "gu_wq", _WORDS, local * 2 * fe * d // 8)
            _need(gu_ws, "gu_ws", (torch.float16,), local * 2 * fe * d // group)
            _need(dn_wq, "dn_wq", _WORDS, local * d * fe // 8)
            _need(dn_ws, "dn_ws", (torch.float16,), local * d * fe // group)
        self.w = (gu_wq, gu_ws, dn_wq, dn_ws)
        # peer: device peer-memory exchange (needs the fixed capacity and the device path); nccl: all-to-alls
        self.exchange = exchange or ("peer" if self.capacity and ops is None else "nccl")
        if self.exchange == "peer":
            if not self.capacity or ops is not None:
                raise MQError(-1, "the peer exchange needs max_tokens and the device ops")
            dev = gu_wq.device
            self.local_experts = local
            rows = self.world * self.capacity
            if share is not None:
                if (share.exchange != "peer" or share.capacity != self.capacity or share.d != d or share.fe != fe
                        or share.local_experts != local or share.world != self.world):
                    raise MQError(-1, "share: the other layer must be a peer-exchange layer of the same shape")
                self.peer, self.workspace, self.empty_plan = share.peer, share.workspace, share.empty_plan
                self.owns_peer = False
            else:
                self.peer = PeerBuffers(self.world, self.rank, self.capacity, d, dev, pg)
                nbytes = lib.mq_ep_workspace_size(rows, local, d, fe)
                self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
                self.empty_plan = torch.full((rows,), -1, dtype=torch.int32, device=dev)
                self.owns_peer = True

    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.pg)
        return out

    def forward(self, x, ids, weights, y, add=False):
        d, topk = self.d, self.topk
        tokens = x.shape[0]
        if ids.numel() != tokens * topk or weights.numel() != tokens * topk:
            raise MQError(-1, f"ids / weights must hold tokens * topk = {tokens * topk} entries")
        if self.exchange == "peer":
            return self._forward_peer(x, ids, weights, y, add)
        if self.capacity:
            return self._forward_fixed(x, ids, weights, y, add)
        # 1. plan, and the rows to send, in send order (a rank without tokens still joins every exchange)
        if tokens > 0:
            counts, order, slot_of, local = self.ops.plan(ids, tokens, topk, self.experts, self.world)
            send = self.ops.gather(x, order, topk, d)
        else:
            counts = torch.zeros(self.world, dtype=torch.int32, device=x.device)
            slot_of = local = torch.empty(0, dtype=torch.int32, device=x.device)
            send = torch.empty(0, d, dtype=torch.float16, device=x.device)
        # 2. dispatch: counts first (the receivers' split sizes), then rows and local expert ids
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts, [1] * self.world, [1] * self.world)
        both = torch.cat([counts, recv_counts]).cpu().tolist()
        send_splits, recv_splits = both[:self.world], both[self.world:]
        r, sent = sum(recv_splits), sum(send_splits)  # sent < tokens * topk only if ids were out of range
        rows = torch.empty(r, d, dtype=send.dtype, device=send.device)
        self._a2a(rows, send[:sent], recv_splits, send_splits)
        rids = torch.empty(r, dtype=torch.int32, device=local.device)
        self._a2a(rids, local[:sent], recv_splits, send_splits)
        # 3. this rank's experts on the rows it received
        if r > 0:
            out = self.ops.experts(rows, rids, *self.w, d, self.fe, self.group)
        else:
            out = torch.empty(0, d, dtype=torch.float32, device=send.device)
        # 4. outputs back in send order, then the weighted per-token sum in slot order
        ret = torch.empty(sent, d, dtype=torch.float32, device=send.device)
        self._a2a(ret, out, send_splits, recv_splits)
        if tokens == 0:
            return y
        return self.ops.combine(ret, slot_of, weights, tokens, topk, d, add, y)

    def _forward_fixed(self, x, ids, weights, y, add):
        """The fixed-capacity exchange: static split sizes, no host read."""
        d, topk, world, cap = self.d, self.topk, self.world, self.capacity
        tokens = x.shape[0]
        if tokens * topk > cap:
            raise MQError(-1, f"{tokens} tokens exceed max_tokens = {cap // topk}")
        splits = [cap] * world
        if tokens > 0:
            _, order, slot_of, local = self.ops.plan(ids, tokens, topk, self.experts, world, cap)
            send = self.ops.gather(x, order, topk, d)
        else:
            order = local = torch.full((world * cap,), -1, dtype=torch.int32, device=x.device)
            send = torch.zeros(world * cap, d, dtype=torch.float16, device=x.device)
        rows = torch.empty_like(send)
        self._a2a(rows, send, splits, splits)
        rids = torch.empty_like(local)
        self._a2a(rids, local, splits, splits)
        out = self.ops.experts(rows, rids, *self.w, d, self.fe, self.group)
        ret = torch.empty_like(out)
        self._a2a(ret, out, splits, splits)
        if tokens == 0:
            return y
        return self.ops.combine(ret, slot_of, weights, tokens, topk, d, add, y)

    def _forward_peer(self, x, ids, weights, y, add):
        """The peer-memory exchange: every step a kernel on the current stream, no host read."""
        d, topk, world, rank, cap, B = self.d, self.topk, self.world, self.rank, self.capacity, self.peer
        tokens = x.shape[0]
        if tokens * topk > cap:
            raise MQError(-1, f"{tokens} tokens exceed max_tokens = {cap // topk}")
        st = _stream()
        if tokens > 0:
            _, order, slot_of, local = self.ops.plan(ids, tokens, topk, self.experts, world, cap)
        else:
            order = local = self.empty_plan
        lib.call("mq_ep_dispatch", _p(x) if tokens else None, MQ_F16 if x.dtype == torch.float16 else MQ_F32, _p(order),
                 _p(local), tokens, topk, d, world, rank, cap, _p(B.peer_rows), _p(B.peer_ids), _p(B.peer_flags),
                 B.ptr["epoch"], B.ptr["done"], st)
        gu_wq, gu_ws, dn_wq, dn_ws = self.w
        lib.call("mq_ep_expert_step", B.ptr["rows"], B.ptr["ids"], _p(gu_wq), _p(gu_ws), _p(dn_wq), _p(dn_ws),
                 world * cap, self.local_experts, d, self.fe, self.group, world, rank, cap, _p(B.peer_ret),
                 B.ptr["flags"], _p(B.peer_flags), B.ptr["epoch"], B.ptr["done"] + 4, _p(self.workspace),
                 self.workspace.numel(), st)
        if tokens == 0:  # still waits for the returns: every rank takes the same steps
            lib.call("mq_ep_wait", B.ptr["flags"], 1, world, B.ptr["epoch"], st)
            return y
        lib.call("mq_ep_combine", _p(B.ret), _p(slot_of), _p(weights), tokens, topk, d, int(bool(add)), _p(y),
                 B.ptr["flags"], world, B.ptr["epoch"], st)
        return y

    def close(self):
        """Unmaps the peers' buffers (call on every rank after the last layer, before the process group ends)."""
        if self.exchange == "peer" and self.owns_peer:
            self.peer.close()

    __call__ = forward
