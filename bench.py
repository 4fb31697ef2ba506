"""Benchmark of the weight-quantised matmul hot path on B200 (the driver's bench contract).

Headline workload: Q4_0 (G=32) decode GEMV over every matmul of one
Llama-3.2-1B layer (qkv 3072x2048, o 2048x2048, gate|up 16384x2048, down 2048x8192) plus the
128256x2048 lm_head, batch 1, fp32 activations. A step is one pass of the five GEMVs.
N GPUs shard every matrix column-parallel along its output rows (no communication), so the
total work is fixed as N grows ("scaling": "strong"). value = algorithmic bytes of the whole job
(packed weights + fp16 scales + fp32 x and y) / max-over-ranks time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mq|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...

--impl reference times the reference's CPU path for the same workload on this host's cores: its
dequantiser (Weights.int4 of qwen3moe/reference.py:53-65, restated in oracle/q4.py) followed by
a torch fp32 matmul (qwen3moe/reference.py:135), over the whole job every step, its row blocks
spread over every host thread.
"""
import argparse
import json
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "mojo-adreno_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
METRIC = "Q4_0 GEMV HBM GB/s (Llama-3.2-1B layer + lm_head decode, batch 1)"
GROUP = 32


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured (MEASURED_PEAKS.json)"
    return 6650.0, 1590.0, "fallback (no MEASURED_PEAKS.json)"


def q4_bytes(n, k, batch):
    """Algorithmic bytes of one int4 GEMV: packed weights, fp16 scales, fp32 x and y."""
    return n * k // 2 + n * (k // GROUP) * 2 + batch * k * 4 + batch * n * 4


class Clocks:
    """Samples the SM clock and the clock-event reasons of one GPU through NVML (read-only queries)
    every few milliseconds while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, index, period_s=0.004):
        self.index, self.period = index, period_s
        self.samples, self.max_mhz, self.nvml, self.handle = [], None, None, None

    def _open(self):
        import pynvml

        pynvml.nvmlInit()
        handle = None
        try:  # the CUDA device's own NVML handle (CUDA and NVML indices can differ)
            handle = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{torch.cuda.get_device_properties(self.index).uuid}")
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self.nvml, self.handle = pynvml, handle
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        self.reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

    def _sample(self):
        mhz = self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
        self.samples.append((mhz, int(self.reasons_fn(self.handle))))

    def _run(self):
        while not self.stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            self.stop.wait(self.period)

    def __enter__(self):
        import threading

        try:
            self._open()
            self._sample()
        except Exception:
            self.handle = None
            return self
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.handle is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self._sample()
                self.nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        sm = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = sorted(name for name, b in self.REASONS.items() if bits & b)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "source": "nvml"}


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def shard(n, world, rank):
    lo = n * rank // world
    hi = n * (rank + 1) // world
    return lo, hi


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def graph_of(fn):
    """A CUDA graph of the launches `fn` makes (warmed up once outside the capture)."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def time_graphs(graphs, reps, stream):
    """Average ms per replay over `reps` replays cycling through `graphs` (CUDA events)."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        graphs[i % len(graphs)].replay()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def rotating_copies(shard_bytes):
    """Weight copies per rank so that consecutive launches never find their weights in L2."""
    return max(2, -(-2 * L2_BYTES // shard_bytes))


DTYPE = ("int4 weights (fp16 scale per 32) x activations staged as 15-bit fixed point per 32-k group (two int8 "
         "limbs): exact integer products on the int8 tensor op, fp32 across groups")


def workload_config(world):
    """The workload both arms run (identical in the GPU and the reference line)."""
    from mq import synth

    return {"workload": "llama-3.2-1b decode layer + lm_head, Q4_0 G=32 GEMV, batch 1",
            "matrices": {nm: [n, k] for nm, n, k in synth.LLAMA_LAYER}, "batch": 1,
            "parallelism": f"column-parallel along output rows x{world} GPU(s), no communication; the reference "
                           "arm splits the same rows over host threads",
            "l2": "inputs larger than L2: rotating weight copies on the GPU (the reference arm streams host memory)"}


def run_mq(args):
    import mq
    from mq import synth

    world, rank, local = init_dist()
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    batch = 1
    layer = synth.llama_layer(batch=batch, seed=0)
    mats = []
    shard_bytes = 0
    for name, n, k in synth.LLAMA_LAYER:
        x, wq, ws = layer[name]
        lo, hi = shard(n, world, rank)
        mats.append(dict(name=name, n=hi - lo, k=k, x=torch.from_numpy(x).to(dev),
                         wq=torch.from_numpy(wq[lo:hi].view(np.int32)).to(dev), ws=torch.from_numpy(ws[lo:hi]).to(dev),
                         y=torch.empty(batch, hi - lo, device=dev)))
        shard_bytes += (hi - lo) * k // 2 + (hi - lo) * (k // GROUP) * 2
    copies = rotating_copies(shard_bytes)
    for m in mats:
        m["wqs"] = [m["wq"]] + [m["wq"].clone() for _ in range(copies - 1)]
        m["wss"] = [m["ws"]] + [m["ws"].clone() for _ in range(copies - 1)]
    job_bytes = sum(q4_bytes(n, k, batch) for _, n, k in synth.LLAMA_LAYER)

    def step(c):
        for m in mats:
            mq.gemv_q4(m["wqs"][c], m["wss"][c], m["x"], m["y"], m["k"], group=GROUP)

    # The decode step is recorded once per weight copy and replayed (the reference likewise records
    # its per-token dispatch plan once, llama/llama_vk.c:382-425).
    graphs = [graph_of(lambda c=c: step(c)) for c in range(copies)]
    for i in range(args.warmup):
        graphs[i % copies].replay()
    barrier(world)

    # ---- device-resident timed region ------------------------------------------------------
    with Clocks(local) as clk:
        barrier(world)
        ms_step = time_graphs(graphs, args.steps, stream)
    ms_step = max_over_ranks(ms_step, world)
    value = job_bytes / (ms_step * 1e-3) / 1e9

    # ---- dominant kernel: the lm_head GEMV (81% of the bytes), back to back in a graph --------
    head = mats[-1]
    reps_in_graph = 20
    head_graph = graph_of(lambda: [mq.gemv_q4(head["wqs"][i % copies], head["wss"][i % copies], head["x"], head["y"],
                                              head["k"], group=GROUP) for i in range(reps_in_graph)])
    head_ms = time_graphs([head_graph], max(5, args.steps // 100), stream) / reps_in_graph
    head_ms = max_over_ranks(head_ms, world)
    def cold(m):
        """Enough copies of one matrix that a graph cycling through them never finds its weights in L2."""
        mc = rotating_copies(m["wq"].numel() * 4 + m["ws"].numel() * 2)
        return [m["wq"]] + [m["wq"].clone() for _ in range(mc - 1)], [m["ws"]] + [m["ws"].clone() for _ in range(mc - 1)]

    per_matrix = {}
    for m in mats:
        cw, cs = cold(m)
        gm = graph_of(lambda m=m, cw=cw, cs=cs: [mq.gemv_q4(w_, s_, m["x"], m["y"], m["k"], group=GROUP)
                                                 for w_, s_ in zip(cw, cs)])
        per_matrix[m["name"]] = round(time_graphs([gm], 10, stream) / len(cw), 5)
        del gm, cw, cs

    # ---- BASELINE configs[0] on the GPU: the Q4_0 GEMV 8192x2048 (the CPU-runnable case), L2-cold
    cx, cwq, cws = synth.gemv_config1(seed=0)
    c0 = dict(wq=torch.from_numpy(cwq.view(np.int32)).to(dev), ws=torch.from_numpy(cws).to(dev))
    cw, cs = cold(c0)
    ctx_, cty = torch.from_numpy(cx).to(dev), torch.empty(1, 8192, device=dev)
    gc = graph_of(lambda: [mq.gemv_q4(w_, s_, ctx_, cty, 2048, group=GROUP) for w_, s_ in zip(cw, cs)])
    c0_ms = max_over_ranks(time_graphs([gc], 10, stream) / len(cw), world)
    config0 = {"shape": [8192, 2048], "ms": round(c0_ms, 5),
               "GB/s": round(q4_bytes(8192, 2048, 1) / (c0_ms * 1e-3) / 1e9, 1),
               "frac_of_measured_hbm": round(q4_bytes(8192, 2048, 1) / (c0_ms * 1e-3) / 1e9 / peaks()[0], 4),
               "frac_of_nominal_8tbs": round(q4_bytes(8192, 2048, 1) / (c0_ms * 1e-3) / 1e9 / 8000.0, 4)}
    del gc, cw, cs, c0

    # ---- end to end through the public API: x from pinned host, logits back, every step ------
    # The step's activations travel as one pinned block in one copy; each GEMV reads its slice. The
    # copies run on a second stream, double-buffered: step i+1's upload and step i's logits read
    # overlap the GEMVs, as a serving loop would run them. The GEMVs are issued two ways: eagerly
    # (five mq.gemv_q4 calls per step, which the host issues more slowly than they run) and as a CUDA graph of
    # those same calls, recorded once per (activation buffer, weight copy) and replayed per step,
    # as the device-resident step above is; the copies and the cross-stream waits stay per step.
    x_host = torch.cat([m["x"].reshape(-1) for m in mats]).cpu().pin_memory()
    x_dev = [torch.empty_like(x_host, device=dev) for _ in range(2)]
    x_views = [[], []]
    for b in range(2):
        at = 0
        for m in mats:
            x_views[b].append(x_dev[b][at:at + m["x"].numel()].view(m["x"].shape))
            at += m["x"].numel()
    y_dev = [torch.empty_like(mats[-1]["y"]) for _ in range(2)]
    y_host = [torch.empty(mats[-1]["y"].shape, dtype=torch.float32).pin_memory() for _ in range(2)]
    h2d = x_host.numel() * x_host.element_size()
    d2h = y_host[0].numel() * 4
    e2e_steps = max(100, args.steps // 4)  # enough steps that filling and draining the copy pipeline is a small part
    copy_stream = torch.cuda.Stream(device=dev)
    up_done = [torch.cuda.Event() for _ in range(2)]    # x_dev[b] filled
    used = [torch.cuda.Event() for _ in range(2)]       # the GEMVs that read x_dev[b] / wrote y_dev[b] are done
    read_done = [torch.cuda.Event() for _ in range(2)]  # y_dev[b] is on the host

    def issue_step(b, c):
        for j, (m, xv) in enumerate(zip(mats, x_views[b])):
            out = y_dev[b] if j == len(mats) - 1 else m["y"]
            mq.gemv_q4(m["wqs"][c], m["wss"][c], xv, out, m["k"], group=GROUP)

    def e2e_run(issue):
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_stream(stream)
            x_dev[0].copy_(x_host, non_blocking=True)
            up_done[0].record(copy_stream)
        for i in range(e2e_steps):
            b, nb = i % 2, (i + 1) % 2
            if i + 1 < e2e_steps:  # next step's upload, once the GEMVs of step i - 1 no longer read x_dev[nb]
                with torch.cuda.stream(copy_stream):
                    if i >= 1:
                        copy_stream.wait_event(used[nb])
                    x_dev[nb].copy_(x_host, non_blocking=True)
                    up_done[nb].record(copy_stream)
            stream.wait_event(up_done[b])
            if i >= 2:
                stream.wait_event(read_done[b])  # y_dev[b] of step i - 2 has reached the host
            issue(b, i % copies)
            used[b].record(stream)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(used[b])
                y_host[b].copy_(y_dev[b], non_blocking=True)
                read_done[b].record(copy_stream)
        stream.wait_stream(copy_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), world) / e2e_steps

    e2e_eager_ms = e2e_run(issue_step)
    step_graphs = [[graph_of(lambda b=b, c=c: issue_step(b, c)) for c in range(copies)] for b in range(2)]
    e2e_ms = e2e_run(lambda b, c: step_graphs[b][c].replay())
    del step_graphs
    e2e_value = job_bytes / (e2e_ms * 1e-3) / 1e9
    e2e_eager_value = job_bytes / (e2e_eager_ms * 1e-3) / 1e9

    # ---- secondary: ternary GEMV, Qwen3-8B shapes, N-sharded the same way
    tern = {}
    tsyn = synth.ternary(seed=0)
    for name, n, k in synth.QWEN3_TERNARY:
        x, w, s = tsyn[name]
        lo, hi = shard(n, world, rank)
        lo, hi = lo // 4 * 4, hi // 4 * 4
        tx = torch.from_numpy(x).to(dev)
        tw = torch.from_numpy(np.ascontiguousarray(w[:, lo:hi]).view(np.int32)).to(dev)
        ts = torch.from_numpy(np.ascontiguousarray(s[:, lo:hi])).to(dev)
        nb = (hi - lo) * k // 4 + (hi - lo) * (k // 128) * 2
        tc = rotating_copies(nb)
        tws = [tw] + [tw.clone() for _ in range(tc - 1)]
        tss = [ts] + [ts.clone() for _ in range(tc - 1)]
        ty = torch.empty(1, hi - lo, device=dev)
        gt = graph_of(lambda: [mq.project(tx, tws[i % tc], tss[i % tc], ty, hi - lo, k) for i in range(reps_in_graph)])
        tms = max_over_ranks(time_graphs([gt], 10, stream) / reps_in_graph, world)
        tbytes = n * k // 4 + n * (k // 128) * 2 + 2 * k + 4 * n
        gbs = tbytes / (tms * 1e-3) / 1e9  # the whole matrix over the slowest rank's time
        tern[name] = {"shape": [n, k], "ms": round(tms, 5), "GB/s_all_gpus": round(gbs, 1),
                      "GB/s_per_gpu": round(gbs / world, 1), "frac_of_measured_hbm_per_gpu": round(gbs / world / peaks()[0], 4)}
        del tws, tss

    # ---- secondary: the fused decode epilogues (one launch each) against their unfused forms -------
    fused = {}
    if world == 1:
        # gate|up with the SwiGLU inside the GEMV (gate_up_q4) vs the GEMV over 2f rows + the SwiGLU kernel
        gu = mats[2]
        f = gu["n"] // 2
        ga = torch.empty(1, f, device=dev)
        sm = torch.cuda.current_stream().cuda_stream
        cw, cs = cold(gu)
        g_f = graph_of(lambda: [mq.gate_up_q4(w_, s_, gu["x"], ga, gu["k"], f, group=GROUP) for w_, s_ in zip(cw, cs)])
        g_u = graph_of(lambda: [(mq.gemv_q4(w_, s_, gu["x"], gu["y"], gu["k"], group=GROUP),
                                 mq.lib.call("mq_moe_silu_mul", gu["y"].data_ptr(), ga.data_ptr(), 1, f, sm))
                                for w_, s_ in zip(cw, cs)])
        f_ms = time_graphs([g_f], 10, stream) / len(cw)
        u_ms = time_graphs([g_u], 10, stream) / len(cw)
        del cw, cs
        fused["gate_up_q4"] = {"shape": [2 * f, gu["k"]], "fused_ms": round(f_ms, 5), "unfused_ms": round(u_ms, 5),
                               "GB/s": round(q4_bytes(2 * f, gu["k"], 1) / (f_ms * 1e-3) / 1e9, 1)}
        del g_f, g_u
        # the ternary head with packed_head's argmax candidates + the device greedy, vs the logits alone
        hx, hw, hs = tsyn["head"]
        hn, hk = hw.shape[1], hx.shape[1]
        thx = torch.from_numpy(hx).to(dev)
        thw = [torch.from_numpy(hw.view(np.int32)).to(dev)]
        ths = [torch.from_numpy(hs).to(dev)]
        thw.append(thw[0].clone())
        ths.append(ths[0].clone())
        thy = torch.empty(1, hn, device=dev)
        thc = torch.empty(1, -(-hn // 512), 3, device=dev)
        thi = torch.empty(1, dtype=torch.int32, device=dev)
        g_h = graph_of(lambda: [(mq.packed_head(thx, thw[i % 2], ths[i % 2], thy, thc, hn, hk), mq.head_argmax(thc, thi))
                                for i in range(reps_in_graph)])
        g_p = graph_of(lambda: [mq.project(thx, thw[i % 2], ths[i % 2], thy, hn, hk) for i in range(reps_in_graph)])
        h_ms = time_graphs([g_h], 10, stream) / reps_in_graph
        p_ms = time_graphs([g_p], 10, stream) / reps_in_graph
        fused["packed_head_argmax"] = {"shape": [hn, hk], "head_and_greedy_ms": round(h_ms, 5),
                                       "logits_only_ms": round(p_ms, 5)}
        del g_h, g_p, thw, ths

    # ---- secondary: int4 prefill GEMM, Llama-3.2-1B shapes, 431 tokens -----
    hbm, tflops_peak, peak_src = peaks()
    prefill = {}
    psyn = synth.prefill(seed=0)
    for name, n, k in synth.LLAMA_PREFILL:
        x, wq, ws = psyn[name]
        lo, hi = shard(n, world, rank)
        px = torch.from_numpy(x).to(dev)
        pw = torch.from_numpy(np.ascontiguousarray(wq[lo:hi]).view(np.int32)).to(dev)
        ps = torch.from_numpy(np.ascontiguousarray(ws[lo:hi])).to(dev)
        py = torch.empty(x.shape[0], hi - lo, device=dev)
        gp = graph_of(lambda: [mq.p_gemm_q4(pw, ps, px, py, hi - lo, k, x.shape[0], group=GROUP) for _ in range(10)])
        pms = max_over_ranks(time_graphs([gp], 10, stream) / 10, world)
        flops = 2.0 * x.shape[0] * n * k
        tf = flops / (pms * 1e-3) / 1e12  # the whole GEMM over the slowest rank's time
        prefill[name] = {"shape": [n, k], "tokens": x.shape[0], "ms": round(pms, 5),
                         "TFLOP/s_all_gpus": round(tf, 1), "TFLOP/s_per_gpu": round(tf / world, 1),
                         "frac_of_measured_bf16_peak_per_gpu": round(tf / world / tflops_peak, 4)}
        del gp

    # ---- secondary: ternary prefill GEMM (p_gemm_t2), Qwen3-8B projections, 512 rows, fp16 x -----------
    tprefill = {}
    trng = np.random.default_rng(11)
    for name, n, k in synth.QWEN3_TERNARY[:2]:
        lo, hi = shard(n, world, rank)
        tw_, ts_ = synth.ternary_matrix(trng, n, k)
        tx_ = torch.from_numpy(trng.standard_normal((512, k)).astype(np.float16)).to(dev)
        tw_d = torch.from_numpy(np.ascontiguousarray(tw_[:, lo:hi]).view(np.int32)).to(dev)
        ts_d = torch.from_numpy(np.ascontiguousarray(ts_[:, lo:hi])).to(dev)
        ty_ = torch.empty(512, hi - lo, device=dev)
        gt_ = graph_of(lambda: [mq.p_gemm_t2(tx_, tw_d, ts_d, ty_, hi - lo, k, 512) for _ in range(10)])
        tms = max_over_ranks(time_graphs([gt_], 10, stream) / 10, world)
        flops = 2.0 * 512 * n * k
        tf = flops / (tms * 1e-3) / 1e12
        tprefill[name] = {"shape": [n, k], "rows": 512, "ms": round(tms, 5), "TFLOP/s_all_gpus": round(tf, 1),
                          "TFLOP/s_per_gpu": round(tf / world, 1),
                          "frac_of_measured_bf16_peak_per_gpu": round(tf / world / tflops_peak, 4)}
        del gt_
        if name == synth.QWEN3_TERNARY[0][0]:  # the tile and split choice across prompt lengths
            sweep = {}
            for rows in (64, 128, 256, 1024, 2048):
                sx_ = torch.from_numpy(trng.standard_normal((rows, k)).astype(np.float16)).to(dev)
                sy_ = torch.empty(rows, hi - lo, device=dev)
                gs_ = graph_of(lambda: [mq.p_gemm_t2(sx_, tw_d, ts_d, sy_, hi - lo, k, rows) for _ in range(10)])
                sms_ = max_over_ranks(time_graphs([gs_], 10, stream) / 10, world)
                stf = 2.0 * rows * n * k / (sms_ * 1e-3) / 1e12
                sweep[str(rows)] = {"ms": round(sms_, 5), "TFLOP/s_per_gpu": round(stf / world, 1),
                                    "frac_of_measured_bf16_peak_per_gpu": round(stf / world / tflops_peak, 4)}
                del gs_
            tprefill[name]["rows_sweep"] = sweep
            tprefill[name]["rows_sweep_note"] = "weights L2-resident (the 12.6 MB shard stays in L2 across launches)"

    # ---- secondary: the decode layer at batch 64 through the tensor-core path
    b64 = synth.llama_layer(batch=64, seed=0)
    b64_graphs = []
    b64_bufs = []
    for m_ in mats:
        x64 = torch.from_numpy(b64[m_["name"]][0]).to(dev).half()
        y64 = torch.empty(64, m_["n"], device=dev)
        b64_bufs.append((x64, y64))
    for c in range(copies):
        b64_graphs.append(graph_of(lambda c=c: [mq.gemv_q4(m_["wqs"][c], m_["wss"][c], xb, yb, m_["k"], group=GROUP)
                                                for m_, (xb, yb) in zip(mats, b64_bufs)]))
    b64_ms = max_over_ranks(time_graphs(b64_graphs, 50, stream), world)
    b64_bytes = sum(q4_bytes(n, k, 64) for _, n, k in synth.LLAMA_LAYER)
    b64_gbs = b64_bytes / (b64_ms * 1e-3) / 1e9
    decode64 = {"ms_per_step": round(b64_ms, 5), "GB/s_all_gpus": round(b64_gbs, 1), "GB/s_per_gpu": round(b64_gbs / world, 1),
                "x": "fp16 [64, k] per matrix", "path": "tcgen05 GEMM (batch > 4)"}
    del b64_graphs

    # ---- secondary: Qwen3-30B-A3B MoE layer: 404-token prefill, 1-token decode
    moe_res = moe_bench(mq, synth, dev, stream, world, rank) if world == 1 else \
        moe_bench_ep(mq, synth, dev, stream, world, rank)

    head_bytes = q4_bytes(head["n"], head["k"], batch) * (world if world > 1 else 1)
    achieved = q4_bytes(head["n"], head["k"], batch) / (head_ms * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(REPO, "profiles", "gemv_q4_lm_head_traffic.json")
    if os.path.exists(tpath) and world == 1:
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(budget_s=args.cpu_seconds)
    config = workload_config(world)

    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded; BASELINE configs[1] distributions)",
            "config": config,
            "timing": {"step": "the 5 GEMVs of a decode step, recorded once as a CUDA graph and replayed",
                       "weight_copies_per_rank": copies, "clock": "CUDA events, max over ranks"},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "the step's five mq.gemv_q4 API calls recorded once per (activation buffer, weight "
                            "copy) as a CUDA graph and replayed per step; every step the step's x vectors from "
                            "pinned host in one copy and the lm_head logits to pinned host, on a copy stream "
                            "double-buffered against the GEMVs",
                    "eager_value": round(e2e_eager_value, 1),
                    "eager_note": "the same loop with the five mq.gemv_q4 calls issued eagerly each step"},
            "roofline": {"bound": "hbm", "kernel": "gemv_q4_kernel<32,1,true> (lm_head shard)",
                         "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "frac_of_nominal_8tbs": round(achieved / 8000.0, 4),
                         "traffic": traffic, "algorithmic_bytes_per_launch": q4_bytes(head["n"], head["k"], batch),
                         "peak_source": peak_src, "launch_ms": round(head_ms, 5)},
            "per_matrix_ms": per_matrix,
            "gemv_config0": config0,
            "ternary_gemv": tern,
            "fused_decode_epilogues": fused,
            "prefill_gemm": prefill,
            "ternary_prefill_gemm": tprefill,
            "decode_batch64": decode64,
            "moe": moe_res,
            "gpu_launches": args.steps * len(mats),
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graphs, head_graph
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def device_route(mq, logits, dev, topk=8):
    """Routes synthetic router logits on the device (mq.p_route): the MoE layer's ids and weights."""
    tl = torch.from_numpy(logits).to(dev)
    ids = torch.empty(tl.shape[0], topk, dtype=torch.int32, device=dev)
    w = torch.empty(tl.shape[0], topk, device=dev)
    mq.p_route(tl, ids, w, topk=topk)
    return ids, w


def moe_bench(mq, synth, dev, stream, world, rank):
    """Tokens/s of the MoE layer (routing given, computed once on the device) with every expert on
    this GPU. Each CUDA graph holds several layers in a row, as a model's graph does, so the time per
    layer carries no host launch cost; the layers cycle through enough copies of the expert weights
    that the experts a layer touches are never found in L2."""
    out = {}
    for tokens in (404, 1):
        m = synth.moe_layer(seed=0, tokens=tokens)
        tx = torch.from_numpy(m["x"]).to(dev)
        tids, tw = device_route(mq, m["logits"], dev)
        ids = tids.cpu().numpy()
        gw = [torch.from_numpy(m[k].view(np.int32) if m[k].dtype == np.uint32 else m[k]).to(dev)
              for k in ("gu_wq", "gu_ws", "dn_wq", "dn_ws")]
        used = np.unique(ids)
        active_bytes = len(used) * (1536 * 2048 + 2048 * 768) * 9 // 16  # int4 + fp16 scales per G=32
        copies = rotating_copies(active_bytes)
        gws = [gw] + [[a.clone() for a in gw] for _ in range(copies - 1)]
        y = torch.zeros(tokens, 2048, device=dev)
        ws = torch.empty(mq.lib.mq_moe_workspace_size(tokens, 128, 8, 2048, 768), dtype=torch.uint8, device=dev)
        layers = max(copies, 8)
        g = graph_of(lambda: [mq.moe_forward(tx, tids, tw, *gws[i % copies], y, 2048, 768, group=32, workspace=ws)
                              for i in range(layers)])
        ms = max_over_ranks(time_graphs([g], 10, stream) / layers, world)
        # the router (fp32 [128, 2048] GEMV) and routing on the device, timed on their own
        rw = torch.from_numpy((np.random.default_rng(5).standard_normal((128, 2048)) * 0.02).astype(np.float32)).to(dev)
        rl = torch.empty(tokens, 128, device=dev)
        rids = torch.empty(tokens, 8, dtype=torch.int32, device=dev)
        rwts = torch.empty(tokens, 8, device=dev)
        reps = 20
        gr = graph_of(lambda: [mq.router(rw, tx, rids, rwts, 8, rl) for _ in range(reps)])
        router_ms = max_over_ranks(time_graphs([gr], 10, stream) / reps, world)
        # the fused chain: router GEMV + top-k + softmax in one cluster kernel, then the grouping
        gf = graph_of(lambda: [mq.route_group(rw, tx, rids, rwts, 8, logits=rl, group=tokens * 8 > 16)
                               for _ in range(reps)])
        fused_ms = max_over_ranks(time_graphs([gf], 10, stream) / reps, world)
        gfr = graph_of(lambda: [mq.route_group(rw, tx, rids, rwts, 8, logits=rl, group=False) for _ in range(reps)])
        fused_route_ms = max_over_ranks(time_graphs([gfr], 10, stream) / reps, world)
        # the whole layer with its router (mq_moe_layer): routing, grouping and experts
        gl = graph_of(lambda: [mq.moe_layer(tx, rw, *gws[i % copies], y, 2048, 768, group=32, ids=rids, weights=rwts,
                                            workspace=ws) for i in range(layers)])
        layer_ms = max_over_ranks(time_graphs([gl], 10, stream) / layers, world)
        out[f"tokens_{tokens}"] = {"ms": round(ms, 5), "tokens/s": round(tokens / (ms * 1e-3), 1),
                                   "router_and_route_ms": round(router_ms, 5),
                                   "router_and_route_fused_ms": round(fused_route_ms, 5),
                                   "router_route_and_grouping_fused_ms": round(fused_ms, 5),
                                   "layer_with_router_ms": round(layer_ms, 5),
                                   "experts_touched": int(len(used)),
                                   "expert_weight_GB/s": round(active_bytes / (ms * 1e-3) / 1e9, 1),
                                   "timing": f"{layers} layers per CUDA graph over {copies} weight copies"}
        del g, gr, gf, gfr, gl, gws
    return out


def moe_bench_ep(mq, synth, dev, stream, world, rank, steps=50):
    """Tokens/s of the expert-parallel MoE layer (BASELINE configs[3] at N GPUs): rank r owns experts
    [r * 128 / N, (r + 1) * 128 / N) and routes its share of the tokens; rows travel to their experts'
    owners and back through NVLink peer memory (mq.ExpertParallelMoE's peer exchange: kernels only, no
    NCCL, no host read), the whole layer recorded once as a CUDA graph and replayed. Timed with CUDA
    events, max over ranks; every rank checks its tokens' outputs against the fp64 oracle layer, and
    the line reports the largest normwise error over the ranks (asserted <= 1e-3)."""
    from oracle import moe as omoe

    d, fe, experts, topk = 2048, 768, 128, 8
    out = {}
    for tokens in (404, 1):
        m = synth.moe_layer(seed=0, tokens=tokens)
        lo_t, hi_t = shard(tokens, world, rank)
        lo, hi = mq.expert_range(experts, world, rank)
        parts = (m["gu_wq"][lo * 2 * fe:hi * 2 * fe], m["gu_ws"][lo * 2 * fe:hi * 2 * fe], m["dn_wq"][lo * d:hi * d],
                 m["dn_ws"][lo * d:hi * d])
        gw = [torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a)).to(dev)
              for a in parts]
        # Enough weight copies that the experts a layer touches on any rank are never found in L2 (the
        # same count on every rank: the global routing is known to all of them).
        used = np.unique(device_route(mq, m["logits"], dev, topk)[0].cpu().numpy())
        per_expert = (2 * fe * d + d * fe) * 9 // 16  # int4 + fp16 scales per G=32
        copies = max(rotating_copies(max(1, int(np.sum((used >= r * experts // world) & (used < (r + 1) * experts // world))))
                                     * per_expert) for r in range(world))
        gws = [gw] + [[a.clone() for a in gw] for _ in range(copies - 1)]
        max_tokens = max(hi_ - lo_ for lo_, hi_ in (shard(tokens, world, r) for r in range(world)))
        layers = [mq.ExpertParallelMoE(*gws[0], d, fe, experts, topk=topk, group=32, max_tokens=max_tokens)]
        layers += [mq.ExpertParallelMoE(*g, d, fe, experts, topk=topk, group=32, max_tokens=max_tokens, share=layers[0])
                   for g in gws[1:]]
        tx = torch.from_numpy(np.ascontiguousarray(m["x"][lo_t:hi_t])).to(dev)
        if hi_t > lo_t:
            tids, tw = device_route(mq, np.ascontiguousarray(m["logits"][lo_t:hi_t]), dev)
        else:
            tids = torch.empty(0, topk, dtype=torch.int32, device=dev)
            tw = torch.empty(0, topk, device=dev)
        y = torch.empty(hi_t - lo_t, d, device=dev)
        # per-phase device times: the layer's steps captured in one CUDA graph with timing events between
        # them (external events, so that they are recorded on every replay)
        L0 = layers[0]
        B = L0.peer
        ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(5)]

        def phased():
            st = mq.kernels._stream()
            ev[0].record()
            if hi_t > lo_t:
                _, order, slot_of, local = L0.ops.plan(tids, hi_t - lo_t, topk, experts, world, L0.capacity)
            else:
                order = local = slot_of = L0.empty_plan
            ev[1].record()
            mq.lib.call("mq_ep_dispatch", tx.data_ptr(), 0, order.data_ptr(), local.data_ptr(), hi_t - lo_t, topk, d,
                        world, rank, L0.capacity, B.peer_rows.data_ptr(), B.peer_ids.data_ptr(), B.peer_flags.data_ptr(),
                        B.ptr["epoch"], B.ptr["done"], st)
            ev[2].record()
            g0 = L0.w
            mq.lib.call("mq_ep_expert_step", B.ptr["rows"], B.ptr["ids"], g0[0].data_ptr(), g0[1].data_ptr(),
                        g0[2].data_ptr(), g0[3].data_ptr(), world * L0.capacity, L0.local_experts, d, fe, 32, world, rank,
                        L0.capacity, B.peer_ret.data_ptr(), B.ptr["flags"], B.peer_flags.data_ptr(), B.ptr["epoch"],
                        B.ptr["done"] + 4, L0.workspace.data_ptr(), L0.workspace.numel(), st)
            ev[3].record()
            if hi_t > lo_t:
                mq.lib.call("mq_ep_combine", B.ret.data_ptr(), slot_of.data_ptr(), tw.data_ptr(), hi_t - lo_t, topk, d,
                            0, y.data_ptr(), B.ptr["flags"], world, B.ptr["epoch"], st)
            else:
                mq.lib.call("mq_ep_wait", B.ptr["flags"], 1, world, B.ptr["epoch"], st)
            ev[4].record()

        gph = graph_of(phased)
        barrier(world)
        acc = [0.0] * 4
        for _ in range(10):
            gph.replay()
            torch.cuda.synchronize()
            for i in range(4):
                acc[i] += ev[i].elapsed_time(ev[i + 1]) / 10
        names = ("plan", "dispatch", "wait_rows_experts_and_return", "wait_returns_and_combine")
        phases = {nm: round(a * 1e3, 2) for nm, a in zip(names, acc)}
        del gph
        # several layers in a row as one CUDA graph (as a model's graph holds them), cycling through the
        # weight copies, replayed back to back
        nl = max(copies, 8)
        graph = graph_of(lambda: [layers[i % copies](tx, tids, tw, y) for i in range(nl)])
        for i in range(2):
            graph.replay()
        torch.cuda.synchronize()
        barrier(world)
        reps = max(2, steps // nl)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / (reps * nl), world)
        status = int(max_over_ranks(float(mq.device_status()), world))
        err = 0.0
        if hi_t > lo_t:
            ids_np = tids.cpu().numpy()
            ref = omoe.moe_layer(m["x"][lo_t:hi_t], ids_np, tw.cpu().numpy(), m["gu_wq"], m["gu_ws"], m["dn_wq"],
                                 m["dn_ws"], 32, fe)
            err = float(np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max())
        err = max_over_ranks(err, world)
        assert err <= 1e-3 and status == 0, f"expert-parallel layer: normwise error {err}, device status {status}"
        out[f"tokens_{tokens}"] = {"ms": round(ms, 5), "tokens/s": round(tokens / (ms * 1e-3), 1),
                                   "phases_us": phases, "parity_normwise_max_over_ranks": err,
                                   "parallelism": f"expert-parallel x{world} ({experts // world} experts per GPU), "
                                                  "peer-memory dispatch and return over NVLink (no NCCL on the data "
                                                  f"path), capacity {max_tokens * topk} rows per rank pair",
                                   "timing": f"{nl} layers per CUDA graph over {copies} weight copies, max over ranks; "
                                             "phases from one layer's graph with events between its steps"}
        del graph
        torch.cuda.synchronize()
        barrier(world)
        for L in layers:
            L.close()
        del layers, gws
    return out


class CpuJob:
    """The reference's CPU path for the decode step: each matrix dequantised as Weights.int4 does
    (oracle/q4.py restates qwen3moe/reference.py:53-65 in numpy) and multiplied by x with torch in
    fp32 (qwen3moe/reference.py:135). Row blocks of every matrix are spread over `threads` host
    threads (numpy and torch release the interpreter lock in their loops); `rows` limits every matrix
    to its first rows (a sample), None runs the whole job."""

    BLOCK = 4096  # rows per task at k = 2048 (fewer for longer rows)

    def __init__(self, threads, rows=None):
        from concurrent.futures import ThreadPoolExecutor

        from mq import synth

        layer = synth.llama_layer(batch=1, seed=0, rows=rows)
        self.mats = [(layer[nm][0], layer[nm][1], layer[nm][2]) for nm, _, _ in synth.LLAMA_LAYER]
        self.xs = [torch.from_numpy(x) for x, _, _ in self.mats]
        self.bytes = sum(q4_bytes(wq.shape[0], wq.shape[1] * 8, 1) for _, wq, _ in self.mats)
        self.rows = sum(wq.shape[0] for _, wq, _ in self.mats)
        self.threads = threads
        self.pool = ThreadPoolExecutor(max_workers=threads)

    def _block(self, i, r0, r1, parts):
        from oracle import q4

        _, wq, ws = self.mats[i]
        t0 = time.perf_counter()
        w = torch.from_numpy(q4.dequant(wq[r0:r1], ws[r0:r1], GROUP))
        t1 = time.perf_counter()
        y = self.xs[i] @ w.T
        t2 = time.perf_counter()
        parts.append((t1 - t0, t2 - t1))
        return y

    def run(self, parts=None):
        """Seconds for one pass over the job (per-block dequantise and matmul thread-seconds into `parts`)."""
        parts = [] if parts is None else parts
        t0 = time.perf_counter()
        futs = []
        for i, (_, wq, _) in enumerate(self.mats):
            block = self.BLOCK * 2048 // (wq.shape[1] * 8)  # about 8 M weights per task
            futs += [self.pool.submit(self._block, i, r0, min(r0 + block, wq.shape[0]), parts)
                     for r0 in range(0, wq.shape[0], block)]
        ys = [f.result() for f in futs]
        dt = time.perf_counter() - t0
        assert all(bool(torch.isfinite(y).all()) for y in ys)
        return dt


def cpu_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def cpu_baseline(budget_s=10.0):
    """The reference's CPU path on the GPU box's host cores, the whole job per pass."""
    threads = cpu_threads()
    torch.set_num_threads(1)  # the parallelism is over row blocks
    job = CpuJob(threads)
    dt = job.run()  # warm-up and sizing
    reps = min(20, max(3, int(budget_s / max(dt, 1e-3))))
    parts = []
    times = [job.run(parts) for _ in range(reps)]
    med = statistics.median(times)
    return {"value": round(job.bytes / med / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "ms_per_step": round(1e3 * med, 3),
            "dequantise_thread_s": round(sum(p[0] for p in parts) / reps, 3),
            "matmul_thread_s": round(sum(p[1] for p in parts) / reps, 3),
            "sample": f"the whole step ({job.rows} rows of the five matrices) per pass, median of {reps}: numpy "
                      f"dequantise + torch fp32 matmul per block of about 8 M weights, blocks over {threads} threads",
            "cpu": platform_cpu()}


def platform_cpu():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    torch.set_num_threads(1)  # the parallelism is over row blocks
    job = CpuJob(threads)
    # Every step is the whole job while warmup + steps of it fit in about three minutes; past that each
    # step runs the same leading rows of every matrix, and the line says so.
    per_step = job.run()
    rows = None
    if per_step * (args.steps + args.warmup) > 180.0:
        frac = 180.0 / (per_step * (args.steps + args.warmup))
        rows = max(CpuJob.BLOCK, int(128256 * frac) // CpuJob.BLOCK * CpuJob.BLOCK)
        job = CpuJob(threads, rows=rows)
    for _ in range(args.warmup):
        job.run()
    times = [job.run() for _ in range(args.steps)]
    med = statistics.median(times)
    value = job.bytes / med / 1e9
    sample = (f"the whole step per step ({job.rows} rows of the five matrices)" if rows is None else
              f"the first {rows} rows of every matrix per step ({job.rows} rows)") + \
        f": numpy dequantise + torch fp32 matmul per block of about 8 M weights, blocks over {threads} threads"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * med, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights dequantised to fp32, fp32 matmul", "data": "synthetic (seeded; BASELINE configs[1] distributions)",
        "config": workload_config(world),
        "timing": {"clock": "host perf_counter per step, median", "sample": sample},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
                         "cpu": platform_cpu()},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def profile_case(name, launches):
    """A few launches of one kernel on one workload, for ncu captures (no timing, no JSON line).
    Cases: gemv_lm_head (configs[1] head, batch 1), tgemv_head (configs[4] head), gemm_gate_up
    (configs[2] 8192x2048, 431 tokens), gemm_decode64_head (configs[1] head, batch 64), moe_prefill
    and moe_decode (configs[3], 404 tokens and 1 token), gemm_t2_gate_up / gemm_t2_down (the ternary
    prefill GEMM on the Qwen3-8B projections, 512 rows), route_group_404 / route_group_1 (the fused
    router chain on configs[3]'s router at 404 tokens and 1 token)."""
    import mq
    from mq import synth

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    if name in ("gemv_lm_head", "gemm_decode64_head"):
        batch = 1 if name == "gemv_lm_head" else 64
        x, wq, ws = synth.llama_layer(batch=batch, seed=0)["lm_head"]
        tw = torch.from_numpy(wq.view(np.int32)).to(dev)
        ts = torch.from_numpy(ws).to(dev)
        tx = torch.from_numpy(x).to(dev)
        if batch > 4:
            tx = tx.half()
        ty = torch.empty(batch, wq.shape[0], device=dev)
        for _ in range(launches):
            mq.gemv_q4(tw, ts, tx, ty, 2048, group=GROUP)
    elif name == "tgemv_head":
        x, w, s = synth.ternary(seed=0, which=("head",))["head"]
        n, k = w.shape[1], w.shape[0] * 16
        tx, tw, ts = (torch.from_numpy(a).to(dev) for a in (x, w.view(np.int32), s))
        ty = torch.empty(1, n, device=dev)
        for _ in range(launches):
            mq.project(tx, tw, ts, ty, n, k)
    elif name == "gemm_gate_up":
        x, wq, ws = synth.prefill(seed=0)["gate_up"]
        tw = torch.from_numpy(wq.view(np.int32)).to(dev)
        ts, tx = torch.from_numpy(ws).to(dev), torch.from_numpy(x).to(dev)
        ty = torch.empty(x.shape[0], wq.shape[0], device=dev)
        for _ in range(launches):
            mq.p_gemm_q4(tw, ts, tx, ty, wq.shape[0], 2048, x.shape[0], group=GROUP)
    elif name in ("gemm_t2_gate_up", "gemm_t2_down"):
        n, k = {a: (b, c) for a, b, c in synth.QWEN3_TERNARY}[name[len("gemm_t2_"):]]
        rng = np.random.default_rng(11)
        w, s = synth.ternary_matrix(rng, n, k)
        tx = torch.from_numpy(rng.standard_normal((512, k)).astype(np.float16)).to(dev)
        tw, ts = torch.from_numpy(w.view(np.int32)).to(dev), torch.from_numpy(s).to(dev)
        ty = torch.empty(512, n, device=dev)
        for _ in range(launches):
            mq.p_gemm_t2(tx, tw, ts, ty, n, k, 512)
    elif name in ("route_group_404", "route_group_1"):
        tokens = 404 if name.endswith("404") else 1
        rng = np.random.default_rng(5)
        rw = torch.from_numpy((rng.standard_normal((128, 2048)) * 0.02).astype(np.float32)).to(dev)
        tx = torch.from_numpy(rng.standard_normal((tokens, 2048)).astype(np.float32)).to(dev)
        ids = torch.empty(tokens, 8, dtype=torch.int32, device=dev)
        wts = torch.empty(tokens, 8, device=dev)
        for _ in range(launches):
            mq.route_group(rw, tx, ids, wts, 8, group=tokens > 2)
    elif name in ("moe_prefill", "moe_decode"):
        tokens = 404 if name == "moe_prefill" else 1
        m = synth.moe_layer(seed=0, tokens=tokens)
        t = {k: torch.from_numpy(m[k].view(np.int32) if m[k].dtype == np.uint32 else m[k]).to(dev)
             for k in ("x", "gu_wq", "gu_ws", "dn_wq", "dn_ws")}
        tids, tw = device_route(mq, m["logits"], dev)
        y = torch.zeros(tokens, 2048, device=dev)
        for _ in range(launches):
            mq.moe_forward(t["x"], tids, tw, t["gu_wq"], t["gu_ws"], t["dn_wq"], t["dn_ws"], y, 2048, 768, group=32)
    else:
        raise SystemExit(f"unknown profile case {name}")
    torch.cuda.synchronize()
    assert mq.device_status() == 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["mq", "reference"], default="mq")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--profile-case", default=None, help="run a few launches of one kernel for ncu and exit")
    ap.add_argument("--launches", type=int, default=3)
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case, args.launches)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mq(args)


if __name__ == "__main__":
    main()
