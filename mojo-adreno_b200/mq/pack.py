"""Weight packers on the device (libmq), named after the reference converters they replace.

Each produces the exact bytes of the reference's offline tool: quantize4 / st2bin (max/7 int4),
qwen3moe's convert.c (searched-scale int4), lfm2's convert.c (GGUF Q4_0 -> words), qwen3's
convert.cpp (ternary transpose) and qwen3k.mojo's pack_half (fp32 -> fp16 pairs).
"""
import torch

from ._lib import MQError, lib
from .kernels import MQ_F16, MQ_F32, _need, _p, _stream

MQ_BF16 = 2
MQ_Q4_MAX7, MQ_Q4_SEARCH = 0, 1

__all__ = ["MQ_BF16", "MQ_Q4_MAX7", "MQ_Q4_SEARCH", "quantize_q4", "quantize4", "q4_0_to_words", "pack_ternary",
           "pack_half"]

_DT = {torch.float32: MQ_F32, torch.float16: MQ_F16, torch.bfloat16: MQ_BF16}


def quantize_q4(w, group=64, method=MQ_Q4_MAX7, wq=None, ws=None):
    """w: fp32 / fp16 / bf16 [n, k] on the device -> (wq int32 [n, k/8], ws fp16 [n, k/group]).
    method MQ_Q4_MAX7: llama/run.py:56-70, llama/st2bin.c:54-70; MQ_Q4_SEARCH: qwen3moe/convert.c:124-157."""
    _need(w, "w", tuple(_DT))
    if w.dim() != 2:
        raise MQError(-1, "w: expected a [n, k] matrix")
    n, k = w.shape
    wq = torch.empty(n, k // 8, dtype=torch.int32, device=w.device) if wq is None else wq
    ws = torch.empty(n, k // group, dtype=torch.float16, device=w.device) if ws is None else ws
    _need(wq, "wq", (torch.int32, torch.uint32), n * k // 8)
    _need(ws, "ws", (torch.float16,), n * k // group)
    lib.call("mq_quantize_q4", _p(w), _DT[w.dtype], n, k, group, method, _p(wq), _p(ws), _stream())
    return wq, ws


def quantize4(w16, group=64):
    """The packed words and fp16 scales of quantize4 (llama/run.py:56-70) for an fp16 matrix."""
    return quantize_q4(w16, group, MQ_Q4_MAX7)


def q4_0_to_words(blocks):
    """GGUF Q4_0 blocks (uint8, 18 bytes each) -> (wq int32 [nblocks * 4], ws fp16 [nblocks]):
    lfm2/convert.c:58-71. Reshape to [rows, cols / 8] and [rows, cols / 32] for a matrix."""
    _need(blocks, "blocks", (torch.uint8,))
    if blocks.numel() % 18:
        raise MQError(-1, "blocks: size is not a whole number of 18-byte Q4_0 blocks")
    nb = blocks.numel() // 18
    wq = torch.empty(nb * 4, dtype=torch.int32, device=blocks.device)
    ws = torch.empty(nb, dtype=torch.float16, device=blocks.device)
    lib.call("mq_q4_0_to_words", _p(blocks), nb, _p(wq), _p(ws), _stream())
    return wq, ws


def pack_ternary(codes, scales, biases=None):
    """MLX 2-bit rows -> the ternary GEMV's transposed layout (qwen3/convert.cpp:39-74): codes int32
    [n, k/16], scales / biases fp16 [n, k/128] -> (w int32 [k/16, n], s fp16 [k/128, n]). Raises
    MQError "not ternary" when a bias differs from -scale."""
    _need(codes, "codes", (torch.int32, torch.uint32))
    n, kw = codes.shape
    k = kw * 16
    _need(scales, "scales", (torch.float16,), n * k // 128)
    if biases is not None:
        _need(biases, "biases", (torch.float16,), n * k // 128)
    w = torch.empty(kw, n, dtype=torch.int32, device=codes.device)
    s = torch.empty(k // 128, n, dtype=torch.float16, device=codes.device)
    lib.call("mq_pack_ternary", _p(codes), _p(scales), _p(biases) if biases is not None else None, n, k, _p(w), _p(s),
             _stream())
    return w, s


def pack_half(x, q=None):
    """fp32 x [.., n] -> fp16 pairs as int32 [.., n/2] (pack_half, qwen3/kernels/qwen3k.mojo:45-48)."""
    _need(x, "x", (torch.float32,))
    q = torch.empty(*x.shape[:-1], x.shape[-1] // 2, dtype=torch.int32, device=x.device) if q is None else q
    _need(q, "q", (torch.int32, torch.uint32), x.numel() // 2)
    lib.call("mq_pack_half", _p(x), _p(q), x.numel(), _stream())
    return q
