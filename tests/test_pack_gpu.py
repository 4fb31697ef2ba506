"""The device packers byte-for-byte against the reference converters' own outputs (tests/golden,
made by make_golden.py from llama/run.py, llama/st2bin.c, qwen3moe/convert.c, lfm2/convert.c and
qwen3/convert.cpp), and against the oracle restatements at sizes the fixtures do not reach."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import q4, ternary

import mq

pytestmark = pytest.mark.gpu


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def dev(a, cuda):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to(cuda)


def u32(t):
    return t.cpu().numpy().view(np.uint32)


def u16(t):
    return t.cpu().numpy().view(np.uint16)


def test_quantize4_matches_run_py(cuda):
    z = load("quantize4.npz")
    wq, ws = mq.quantize4(dev(z["w16"], cuda), 64)
    np.testing.assert_array_equal(u32(wq), z["packed"])
    np.testing.assert_array_equal(u16(ws), z["s16"].view(np.uint16))


def test_max7_bf16_matches_st2bin_c(cuda):
    z = load("st2bin_q4.npz")
    w = dev(z["bf16"], cuda).view(torch.bfloat16)
    wq, ws = mq.quantize_q4(w, 64, mq.MQ_Q4_MAX7)
    np.testing.assert_array_equal(u32(wq), z["words"])
    np.testing.assert_array_equal(u16(ws), z["scales"].view(np.uint16))


@pytest.mark.parametrize("g", [32, 64, 128])
def test_search_matches_qwen3moe_convert_c(cuda, g):
    z = load(f"qwen3moe_q4_g{g}.npz")
    w = dev(z["bf16"], cuda).view(torch.bfloat16)
    wq, ws = mq.quantize_q4(w, g, mq.MQ_Q4_SEARCH)
    np.testing.assert_array_equal(u16(ws), z["scales"].view(np.uint16))
    np.testing.assert_array_equal(u32(wq), z["words"])


@pytest.mark.parametrize("method,dtype", [(0, torch.float32), (1, torch.float32), (1, torch.float16), (0, torch.bfloat16)])
def test_quantize_large_matches_oracle(cuda, method, dtype):
    """A 1024 x 4096 matrix with zero groups, tiny and large magnitudes, every dtype."""
    rng = np.random.default_rng(method)
    w = (rng.standard_normal((1024, 4096)) * 0.05).astype(np.float32)
    w[3, :64] = 0.0
    w[5, 64:96] = 1e-7
    w[7] *= 300.0
    t = torch.from_numpy(w).to(cuda).to(dtype)
    vals = t.float().cpu().numpy()
    wq, ws = mq.quantize_q4(t, 32, method)
    ref = q4.quantize_max7(vals.astype(np.float16), 32) if method == 0 else q4.quantize_search(vals, 32)
    np.testing.assert_array_equal(u16(ws), ref[1].view(np.uint16))
    np.testing.assert_array_equal(u32(wq), ref[0])


def test_q4_0_to_words_matches_lfm2_convert_c(cuda):
    z = load("lfm2_q4.npz")
    wq, ws = mq.q4_0_to_words(dev(z["blocks"].reshape(-1), cuda))
    np.testing.assert_array_equal(u32(wq).reshape(z["words"].shape), z["words"])
    np.testing.assert_array_equal(u16(ws).reshape(z["scales"].shape), z["scales"].view(np.uint16))


def test_q4_0_to_words_large_matches_oracle(cuda):
    blocks = np.random.default_rng(5).integers(0, 256, (20000, 18), dtype=np.uint8)
    blocks[:, :2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    wq, ws = mq.q4_0_to_words(dev(blocks.reshape(-1), cuda))
    rw, rd = q4.q4_0_to_words(blocks)
    np.testing.assert_array_equal(u32(wq), rw.reshape(-1))
    np.testing.assert_array_equal(u16(ws), rd.view(np.uint16))


def test_pack_ternary_matches_qwen3_convert_cpp(cuda):
    z = load("qwen3_pack.npz")
    w, s = mq.pack_ternary(dev(z["codes"], cuda), dev(z["scales"], cuda).view(torch.float16),
                           dev(z["biases"], cuda).view(torch.float16))
    np.testing.assert_array_equal(u32(w), z["w"])
    np.testing.assert_array_equal(u16(s), z["s"].view(np.uint16))
    with pytest.raises(mq.MQError, match="not ternary"):
        mq.pack_ternary(dev(z["codes"], cuda), dev(z["scales"], cuda).view(torch.float16),
                        dev(z["bad_biases"], cuda).view(torch.float16))


def test_pack_ternary_large_matches_oracle(cuda):
    rng = np.random.default_rng(6)
    n, k = 1000, 4096
    codes = rng.integers(0, 1 << 32, (n, k // 16), dtype=np.uint32)
    sc = np.abs(rng.standard_normal((n, k // 128))).astype(np.float16)
    w, s = mq.pack_ternary(dev(codes, cuda), dev(sc, cuda).view(torch.float16), dev(-sc, cuda).view(torch.float16))
    rw, rs = ternary.pack_transposed(codes, sc, -sc)
    np.testing.assert_array_equal(u32(w), rw)
    np.testing.assert_array_equal(u16(s), rs.view(np.uint16))


def test_pack_half_matches_fp16_rounding(cuda):
    x = np.random.default_rng(7).standard_normal((3, 4096)).astype(np.float32) * 1000
    q = mq.pack_half(torch.from_numpy(x).to(cuda))
    np.testing.assert_array_equal(q.cpu().numpy().view(np.float16), x.astype(np.float16))


def test_packed_weights_feed_the_gemv(cuda):
    """quantize on the device, then the GEMV on those words: the layer's numbers, end to end."""
    rng = np.random.default_rng(8)
    w = (rng.standard_normal((512, 2048)) * 0.02).astype(np.float16)
    wq, ws = mq.quantize4(torch.from_numpy(w).to(cuda), 64)
    x = rng.standard_normal((1, 2048)).astype(np.float32)
    y = torch.empty(1, 512, device=cuda)
    mq.gemv_q4(wq, ws, torch.from_numpy(x).to(cuda), y, 2048, group=64)
    rq, rs = q4.quantize_max7(w, 64)
    ref = q4.dequant(rq, rs, 64).astype(np.float64) @ x[0].astype(np.float64)
    assert np.abs(y.cpu().numpy()[0] - ref).max() / np.abs(ref).max() <= 1e-3
