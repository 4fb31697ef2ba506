"""The oracle's restatements against the reference's own outputs (tests/golden, made by
tests/golden/make_golden.py from the reference's Python and its compiled C/C++ converters)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import q4, ternary


def load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.mark.parametrize("g", [32, 64, 128])
def test_dequant_matches_weights_int4(g):
    z = load(f"int4_dequant_g{g}.npz")
    got = q4.dequant(z["wq"], z["ws"], g)
    assert got.dtype == np.float32
    np.testing.assert_array_equal(got, z["deq"])
    np.testing.assert_array_equal(q4.dequant(z["wq"][3:8], z["ws"][3:8], g), z["deq_rows_3_8"])


def test_unpack_values_and_roundtrip():
    z = load("int4_dequant_g32.npz")
    q = q4.unpack(z["wq"])
    assert q.min() >= -8 and q.max() <= 7
    np.testing.assert_array_equal(q4.pack_words(q), z["wq"])


def test_quantize_max7_matches_run_py_quantize4():
    z = load("quantize4.npz")
    wq, ws = q4.quantize_max7(z["w16"], 64)
    np.testing.assert_array_equal(wq, z["packed"])
    np.testing.assert_array_equal(ws.view(np.uint16), z["s16"].view(np.uint16))
    np.testing.assert_array_equal(q4.dequant(wq, ws, 64), z["deq"])


def test_quantize_max7_matches_st2bin_c():
    z = load("st2bin_q4.npz")
    vals = (z["bf16"].astype(np.uint32) << 16).view(np.float32)
    wq, ws = q4.quantize_max7(vals.astype(np.float16), 64)  # st2bin rounds bf16 -> fp16 first
    np.testing.assert_array_equal(wq, z["words"])
    np.testing.assert_array_equal(ws.view(np.uint16), z["scales"].view(np.uint16))


@pytest.mark.parametrize("g", [32, 64, 128])
def test_quantize_search_matches_qwen3moe_convert_c(g):
    z = load(f"qwen3moe_q4_g{g}.npz")
    vals = (z["bf16"].astype(np.uint32) << 16).view(np.float32)
    wq, ws = q4.quantize_search(vals, g)
    np.testing.assert_array_equal(ws.view(np.uint16), z["scales"].view(np.uint16))
    np.testing.assert_array_equal(wq, z["words"])


def test_q4_0_to_words_matches_lfm2_convert_c():
    z = load("lfm2_q4.npz")
    words, d = q4.q4_0_to_words(z["blocks"])
    np.testing.assert_array_equal(words.reshape(z["words"].shape), z["words"])
    np.testing.assert_array_equal(d.view(np.uint16).reshape(z["scales"].shape), z["scales"].view(np.uint16))


def test_q4_0_dequant_matches_lfm2_weights_py():
    z = load("q4_0_dequant.npz")
    rows, cols = int(z["rows"]), int(z["cols"])
    np.testing.assert_array_equal(q4.dequant_q4_0(z["blocks"], rows, cols), z["deq"])
    # the words repack keeps the numbers: dequant(words, d) == ggml's dequant
    words, d = q4.q4_0_to_words(z["blocks"])
    np.testing.assert_array_equal(q4.dequant(words.reshape(rows, cols // 8), d.reshape(rows, cols // 32), 32), z["deq"])


def test_ternary_pack_matches_qwen3_convert_cpp():
    z = load("qwen3_pack.npz")
    w, s = ternary.pack_transposed(z["codes"], z["scales"], z["biases"])
    np.testing.assert_array_equal(w, z["w"])
    np.testing.assert_array_equal(s.view(np.uint16), z["s"].view(np.uint16))
    assert int(z["bad_rc"]) == 1 and "bias != -scale" in str(z["bad_msg"])
    with pytest.raises(ValueError, match="bias != -scale"):
        ternary.pack_transposed(z["codes"], z["scales"], z["bad_biases"])


def test_ternary_codes_layout_and_exact_gemv():
    z = load("qwen3_pack.npz")
    n, k = z["codes"].shape[0], z["codes"].shape[1] * 16
    c = ternary.codes(z["w"], n, k)
    # row layout of the MLX codes: element i of a row at bits 2(i % 16) of word i / 16
    rowc = (z["codes"][:, :, None] >> (np.arange(16, dtype=np.uint32) * 2)) & 3
    np.testing.assert_array_equal(c, rowc.reshape(n, k))
    assert set(np.unique(c)) <= {0, 1, 2}
    x = np.random.default_rng(0).standard_normal((1, k)).astype(np.float16)
    y = ternary.tgemv(x, z["w"], z["s"], n, k)
    w = (c.astype(np.float64) - 1) * np.repeat(z["scales"].astype(np.float64), 128, axis=1)
    np.testing.assert_allclose(y[0], w @ x[0].astype(np.float64), rtol=1e-12, atol=1e-12)
    # the reference's fp16-chain arithmetic stays close to exact (its documented few-1e-3 level)
    yf = ternary.tgemv_fp16_chains(x, z["w"], z["s"], n, k)
    assert np.abs(yf - y[0]).max() / np.abs(y[0]).max() < 5e-3


def test_gemv_reference_order_close_to_exact():
    z = load("int4_dequant_g64.npz")
    x = np.random.default_rng(1).standard_normal((1, 512)).astype(np.float32)
    a = q4.gemv_reference_order(z["wq"], z["ws"], x, 64)
    b = q4.gemv(z["wq"], z["ws"], x, 64)[0]
    assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()


def test_moe_oracle_matches_transformers_block():
    """oracle.moe (routing and the SwiGLU expert layer) against transformers' Qwen3MoeSparseMoeBlock
    run on the same int4 experts (the reference's own check, qwen3moe/reference.py:94-147)."""
    from oracle import moe

    z = load("moe_block.npz")
    ids, w = moe.route(z["logits"], int(z["topk"]))
    np.testing.assert_array_equal(ids, z["ids"])
    np.testing.assert_allclose(w, z["weights"], rtol=2e-6, atol=1e-7)
    y = moe.moe_layer(z["x"], ids, w, z["gu_wq"], z["gu_ws"], z["dn_wq"], z["dn_ws"], int(z["group"]), int(z["fe"]))
    assert np.abs(y - z["y"]).max() <= 1e-5 * np.abs(z["y"]).max()


def test_route_ties_prefer_lowest_index():
    from oracle import moe

    logits = np.zeros((3, 16), np.float32)
    logits[0, [3, 7, 9]] = 1.0          # three-way tie for the top: 3, 7, 9
    logits[1, :] = np.arange(16)[::-1]  # strictly decreasing
    logits[2, [5, 2]] = [2.0, 2.0]
    ids, w = moe.route(logits, 4)
    assert ids[0].tolist()[:3] == [3, 7, 9] and ids[0][3] == 0
    assert ids[1].tolist() == [0, 1, 2, 3]
    assert ids[2].tolist()[:2] == [2, 5]
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)


def test_expert_lists_stable():
    from oracle import moe

    ids = np.array([[3, 1], [1, 0], [3, 2], [1, 3]], np.int32)
    offsets, order = moe.expert_lists(ids, 4)
    assert offsets.tolist() == [0, 1, 4, 5, 8]
    assert order.tolist() == [3, 1, 2, 6, 5, 0, 4, 7]
