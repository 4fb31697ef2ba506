"""Reference-named operators over libmq (torch tensors as device buffers).

Each function keeps the argument order of the reference kernel it replaces (cited per function)
and adds what the reference fixed at compile time (group size, batch). Shapes are taken from the
buffers. Every operator is asynchronous on the current torch CUDA stream; failures raise MQError
with the library's message, as the reference's helpers return a non-zero status.
"""
import ctypes

import torch

from ._lib import MQError, lib

MQ_F32, MQ_F16 = 0, 1

__all__ = ["MQ_F32", "MQ_F16", "MQError", "gemv_q4", "gemv_add_q4", "gate_up_q4", "p_gemm_q4", "p_gemm_t2", "unpack_q4",
           "project", "packed_head", "head_argmax", "device_status"]


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream():
    """The current device's current CUDA stream as a raw handle (building a torch Stream object costs
    about 3 us per call, as much as the launch itself)."""
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return t.data_ptr()


def _need(t, name, dtypes, numel=None):
    if not isinstance(t, torch.Tensor):
        raise MQError(-1, f"{name}: expected a torch.Tensor")
    if not t.is_cuda:
        raise MQError(-1, f"{name}: must be a CUDA tensor (there is no CPU path)")
    if t.dtype not in dtypes:
        raise MQError(-1, f"{name}: dtype {t.dtype} not in {dtypes}")
    if not t.is_contiguous():
        raise MQError(-1, f"{name}: must be contiguous")
    if numel is not None and t.numel() != numel:
        raise MQError(-1, f"{name}: has {t.numel()} elements, expected {numel}")


_WORDS = (torch.int32, torch.uint32)


def gemv_q4(wq, ws, x, y, cols, group=64, add=False):
    """y[b, r] (+)= sum_c W[r, c] x[b, c] for the int4 word-layout W.

    Mirrors gemv_q4(wq, ws, x, y, cols) of llama/kernels/gemv_q4.mojo:13-30 (one row per
    workgroup there; here the rows come from wq's size). wq: int32/uint32 [rows, cols/8];
    ws: fp16 [rows, cols/group]; x: fp32 or fp16 [batch, cols]; y: fp32 [batch, rows].
    group: 64 (llama), 32 (Q4_0 / GGUF, lfm2/kernels/lk.mojo:26), 128 (qwen3moe experts).
    """
    _need(wq, "wq", _WORDS)
    rows = wq.numel() * 8 // cols
    _need(ws, "ws", (torch.float16,), rows * cols // group)
    _need(x, "x", (torch.float32, torch.float16))
    batch = x.numel() // cols
    if batch * cols != x.numel():
        raise MQError(-1, f"x: {x.numel()} elements is not a whole number of rows of {cols}")
    _need(y, "y", (torch.float32,), batch * rows)
    if batch > 4 and x.dtype == torch.float32:  # the tensor-core path takes fp32 x through a workspace
        return p_gemm_q4(wq, ws, x, y, rows, cols, batch, group=group, add=add)
    lib.call("mq_gemv_q4", _p(wq), _p(ws), _p(x), MQ_F16 if x.dtype == torch.float16 else MQ_F32, _p(y),
             rows, cols, group, batch, int(bool(add)), _stream())
    return y


def p_gemm_q4(wq, ws, x, y, n, k, rows=None, group=64, add=False):
    """Y[t, r] (+)= sum_c W[r, c] X[t, c] on the tcgen05 tensor cores: p_gemm_q4(wq, ws, x, y, n, k) of
    llama/kernels/prefill/p_gemm_q4.mojo:26-62 (there X's rows are padded to 128; here `rows` is the
    true token count, default x's). wq: int32/uint32 [n, k/8]; ws: fp16 [n, k/group]; x: fp16 or fp32
    [rows, k]; y: fp32 [rows, n]."""
    _need(wq, "wq", _WORDS, n * k // 8)
    _need(ws, "ws", (torch.float16,), n * k // group)
    _need(x, "x", (torch.float32, torch.float16))
    if rows is None:
        rows = x.numel() // k
    if x.numel() < rows * k:
        raise MQError(-1, f"x: {x.numel()} elements < rows * k = {rows * k}")
    _need(y, "y", (torch.float32,))
    if y.numel() < rows * n:
        raise MQError(-1, f"y: {y.numel()} elements < rows * n = {rows * n}")
    dt = MQ_F16 if x.dtype == torch.float16 else MQ_F32
    nbytes = lib.mq_gemm_q4_workspace_size(rows, k, dt)
    work = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x.device) if nbytes else None
    lib.call("mq_gemm_q4", _p(wq), _p(ws), _p(x), dt, _p(y), n, k, rows, group, int(bool(add)),
             _p(work) if work is not None else None, nbytes, _stream())
    return y


def gemv_add_q4(wq, ws, x, y, cols, group=64):
    """y += W x: gemv_add_q4 of llama/kernels/gemv_add_q4.mojo:13-30 (the residual)."""
    return gemv_q4(wq, ws, x, y, cols, group, add=True)


def gate_up_q4(wq, ws, x, a, cols, f, group=32):
    """a[b, j] = silu(W[j] . x_b) * (W[f + j] . x_b): gate_up_q4(wq, ws, x, a, cols, f) of
    lfm2/kernels/lk.mojo:154-167, the SwiGLU fused into the GEMV. wq: int32/uint32 [2f, cols/8] (gate
    rows, then up rows); ws: fp16 [2f, cols/group]; x: fp32 or fp16 [batch <= 4, cols]; a: fp32 [batch, f]."""
    _need(wq, "wq", _WORDS, 2 * f * cols // 8)
    _need(ws, "ws", (torch.float16,), 2 * f * cols // group)
    _need(x, "x", (torch.float32, torch.float16))
    batch = x.numel() // cols
    if batch * cols != x.numel():
        raise MQError(-1, f"x: {x.numel()} elements is not a whole number of rows of {cols}")
    _need(a, "a", (torch.float32,), batch * f)
    lib.call("mq_gate_up_q4", _p(wq), _p(ws), _p(x), MQ_F16 if x.dtype == torch.float16 else MQ_F32, _p(a), f, cols,
             group, batch, _stream())
    return a


def unpack_q4(wq, ws, cols, group, q=None, s=None):
    """The bit-exact decode hook: int8 q [rows, cols] = ((nib ^ 8) - 8) and the scales unchanged
    (the integer step of qwen3moe/reference.py:53-65)."""
    _need(wq, "wq", _WORDS)
    rows = wq.numel() * 8 // cols
    _need(ws, "ws", (torch.float16,), rows * cols // group)
    if q is None:
        q = torch.empty(rows, cols, dtype=torch.int8, device=wq.device)
    _need(q, "q", (torch.int8,), rows * cols)
    if s is not None:
        _need(s, "s", (torch.float16,), ws.numel())
    lib.call("mq_unpack_q4", _p(wq), _p(ws), _p(q), _p(s) if s is not None else None, rows, cols, group, _stream())
    return q, s


def project(x, w, s, y, n, k):
    """y = W x for the ternary transposed layout: the reference's project() =
    packed_linear + packed_reduce (qwen3/model.mojo:128-135; bonsai/kernels/kernels.mojo:283-325,
    437-448), argument order (input, words, scales, output, n, k). x: fp16 [batch, k] (or the
    fp16-pair int32 [batch, k/2] buffer the reference passes); w: int32/uint32 [k/16, n];
    s: fp16 [k/128, n]; y: fp32 [batch, n]."""
    _need(x, "x", (torch.float16, torch.int32, torch.uint32))
    batch = x.numel() * x.element_size() // 2 // k
    _need(w, "w", _WORDS, k // 16 * n)
    _need(s, "s", (torch.float16,), k // 128 * n)
    _need(y, "y", (torch.float32,), batch * n)
    lib.call("mq_tgemv", _p(x), _p(w), _p(s), _p(y), n, k, batch, _stream())
    return y


CAND_BLOCK = 512  # logits per argmax candidate


def packed_head(x, w, s, y, candidates, n, k, select=True):
    """The ternary vocab head: packed_head(x, w, params, y, candidates, width, reduction, select) of
    bonsai/kernels/kernels.mojo:451-517. y = W x as `project`; with select, candidates [batch, ceil(n/512), 3]
    fp32 get (best logit, its index, non-finite flag) per 512 logits, the lowest index among equal values."""
    if not select:
        return project(x, w, s, y, n, k)
    _need(x, "x", (torch.float16, torch.int32, torch.uint32))
    batch = x.numel() * x.element_size() // 2 // k
    _need(w, "w", _WORDS, k // 16 * n)
    _need(s, "s", (torch.float16,), k // 128 * n)
    _need(y, "y", (torch.float32,), batch * n)
    _need(candidates, "candidates", (torch.float32,), batch * -(-n // CAND_BLOCK) * 3)
    lib.call("mq_tgemv_head", _p(x), _p(w), _p(s), _p(y), _p(candidates), n, k, batch, _stream())
    return y, candidates


def head_argmax(candidates, index=None):
    """The greedy token of each token's candidates [batch, ncand, 3] on the device (best_of,
    lfm2/kernels/dsk.mojo:442-465; greedy() of bonsai/bonsai_vk.c:506-515): int32 [batch], -1 where a
    candidate is flagged non-finite."""
    _need(candidates, "candidates", (torch.float32,))
    batch = candidates.shape[0] if candidates.dim() == 3 else 1
    ncand = candidates.numel() // 3 // batch
    if index is None:
        index = torch.empty(batch, dtype=torch.int32, device=candidates.device)
    _need(index, "index", (torch.int32,), batch)
    lib.call("mq_head_argmax", _p(candidates), ncand, batch, _p(index), _stream())
    return index


def p_gemm_t2(x, w, s, y, n, k, rows=None, add=False):
    """Y[t, c] (+)= sum_k X[t, k] W[c, k] for ternary W on the tcgen05 tensor cores: p_gemm_t2(x, w, params,
    y, n, k) of bonsai/kernels/prefill.mojo:155-164. x: fp32 or fp16 [rows, k]; w: int32/uint32
    [k/16, n]; s: fp16 [k/128, n]; y: fp32 [rows, n]."""
    _need(x, "x", (torch.float32, torch.float16))
    rows = x.numel() // k if rows is None else rows
    _need(w, "w", _WORDS, k // 16 * n)
    _need(s, "s", (torch.float16,), k // 128 * n)
    _need(y, "y", (torch.float32,))
    if y.numel() < rows * n:
        raise MQError(-1, f"y: {y.numel()} elements < rows * n = {rows * n}")
    dt = MQ_F16 if x.dtype == torch.float16 else MQ_F32
    nbytes = lib.mq_gemm_q4_workspace_size(rows, k, dt)
    work = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x.device) if nbytes else None
    lib.call("mq_gemm_t2", _p(x), dt, _p(w), _p(s), _p(y), n, k, rows, int(bool(add)),
             _p(work) if work is not None else None, nbytes, _stream())
    return y


def device_status(reset=True):
    """The device status word set by kernels whose bounded waits ran out (0 = none)."""
    return lib.call("mq_device_status", int(bool(reset)), _stream())
